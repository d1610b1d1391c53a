"""Typed views of the model's ``config.json`` and the synthetic configuration this build runs on.

The reference reads every dimension from the checkpoint's ``config.json`` (src/config.rs:21-66,
src/config.rs:127-135). No checkpoint exists here, so :func:`synthetic_config` writes one with the
dimensions the reference's own profiling code hard-codes for EmbeddingGemma 2 (hidden 512, 24
layers, 4 heads, head_dim 256 / 512 on global layers, one global layer in six) and the values that
live only in the absent file (vocab, eps, RoPE thetas, layer placement) chosen as stated below.
The same file feeds the CPU oracle and the CUDA library.
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path


@dataclass
class TextConfig:
    """Mirror of ``TextConfig`` (src/config.rs:21-41)."""

    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    hidden_size_per_layer_input: int
    embedding_dim: int
    sliding_window: int
    rms_norm_eps: float
    layer_types: list
    rope_parameters: dict
    per_layer_config: dict = field(default_factory=dict)
    attention_bias: bool = False
    pad_token_id: int = 0

    def is_sliding(self, layer: int) -> bool:
        """src/config.rs:44-46."""
        return self.layer_types[layer] == "sliding_attention"

    def layer_dims(self, layer: int) -> tuple[int, int]:
        """``(head_dim, n_kv)`` with per-layer overrides (src/config.rs:48-61)."""
        ov = self.per_layer_config.get(f"{layer:02d}") or self.per_layer_config.get(str(layer))
        if ov is None:
            return self.head_dim, self.num_key_value_heads
        return (ov.get("head_dim") or self.head_dim, ov.get("num_key_value_heads") or self.num_key_value_heads)

    def rope_theta(self, layer: int) -> float:
        """src/config.rs:63-66."""
        key = "sliding_attention" if self.is_sliding(layer) else "full_attention"
        return float(self.rope_parameters[key]["rope_theta"])


@dataclass
class VisionConfig:
    """Mirror of ``VisionConfig`` (src/config.rs:69-86)."""

    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    patch_size: int
    pooling_kernel_size: int
    position_embedding_size: int
    rms_norm_eps: float
    rope_parameters: dict
    standardize: bool = False
    use_clipped_linears: bool = False


@dataclass
class ModelConfig:
    text: TextConfig
    vision: VisionConfig | None
    raw: dict

    @staticmethod
    def load(path: str | Path) -> "ModelConfig":
        """Read ``config.json`` (a directory or the file itself), as src/config.rs:127-135 does."""
        p = Path(path)
        if p.is_dir():
            p = p / "config.json"
        raw = json.loads(p.read_text())
        tc = dict(raw["text_config"])
        if tc.get("attention_bias"):
            raise ValueError("attention_bias=true is not supported")
        known = set(TextConfig.__dataclass_fields__)
        text = TextConfig(**{k: v for k, v in tc.items() if k in known})
        vision = None
        if raw.get("vision_config"):
            vk = set(VisionConfig.__dataclass_fields__)
            vision = VisionConfig(**{k: v for k, v in raw["vision_config"].items() if k in vk})
        return ModelConfig(text=text, vision=vision, raw=raw)


def synthetic_config(num_hidden_layers: int = 24, global_every: int = 6, vision_layers: int = 16) -> dict:
    """The EmbeddingGemma 2 configuration used throughout this build.

    Dimensions pinned by the reference's code: hidden 512 ("GEMM ple_model 512->12288",
    src/gpu/text.rs:361), 24 layers, intermediate 2048 and PLE width 512 (examples/profile_ops.rs:18-28),
    4 query heads with 2 K/V heads of 256 on sliding layers and 1 K/V head of 512 on global ones
    (examples/check_attention.rs:66-72), window radius 512 (src/ops.rs:353), output 768.

    Chosen here because they live only in the absent checkpoint config: vocab 262144, eps 1e-6,
    RoPE theta 1e4 (sliding) / 1e6 (global), layer ``i`` global iff ``i % 6 == 5`` (20 sliding : 4
    global), vision position table 10240 entries and vision RoPE theta 100.
    """
    layer_types = [
        "full_attention" if (i % global_every) == global_every - 1 else "sliding_attention"
        for i in range(num_hidden_layers)
    ]
    per_layer = {
        f"{i:02d}": {"head_dim": 512, "num_key_value_heads": 1}
        for i, t in enumerate(layer_types)
        if t == "full_attention"
    }
    return {
        "architectures": ["EmbeddingGemma2Model"],
        "text_config": {
            "vocab_size": 262144,
            "hidden_size": 512,
            "intermediate_size": 2048,
            "num_hidden_layers": num_hidden_layers,
            "num_attention_heads": 4,
            "num_key_value_heads": 2,
            "head_dim": 256,
            "hidden_size_per_layer_input": 512,
            "embedding_dim": 768,
            "sliding_window": 512,
            "rms_norm_eps": 1e-6,
            "attention_bias": False,
            "pad_token_id": 0,
            "layer_types": layer_types,
            "per_layer_config": per_layer,
            "rope_parameters": {
                "sliding_attention": {"rope_theta": 10000.0, "rope_type": "default"},
                "full_attention": {"rope_theta": 1000000.0, "rope_type": "default"},
            },
        },
        "vision_config": {
            "hidden_size": 768,
            "intermediate_size": 3072,
            "num_hidden_layers": vision_layers,
            "num_attention_heads": 12,
            "num_key_value_heads": 12,
            "head_dim": 64,
            "patch_size": 16,
            "pooling_kernel_size": 3,
            "position_embedding_size": 10240,
            "rms_norm_eps": 1e-6,
            "standardize": False,
            "use_clipped_linears": False,
            "rope_parameters": {"rope_theta": 100.0, "rope_type": "axial"},
        },
        "image_token_id": 258880,
        "audio_token_id": 258881,
        "video_token_id": 258884,
        "boi_token_id": 255999,
        "eoi_token_id": 258882,
        "boa_token_id": 256000,
        "eoa_token_index": 258883,
    }


def write_config(dirpath: str | Path, cfg: dict | None = None) -> Path:
    d = Path(dirpath)
    d.mkdir(parents=True, exist_ok=True)
    p = d / "config.json"
    p.write_text(json.dumps(cfg or synthetic_config(), indent=1))
    return p
