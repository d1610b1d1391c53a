"""Safetensors reading and writing, and the seeded random-init checkpoint this build runs on.

The layout and tensor names are the reference's (reader: src/weights.rs:46-185; names:
src/text.rs:74-111 and src/vision.rs:184-217). Tensors are stored BF16, the checkpoint's own dtype,
and widened to f32 on load exactly as ``bf16_to_f32`` does (src/weights.rs:189-191).

Random init follows the workload definition: every matrix (projections, the token-embedding table
and the vision position table) is N(0, 0.02); every norm weight and ``layer_scalar`` is 1, except the
per-head ``q_norm`` / ``k_norm`` weights, which are ``head_dim ** -0.25`` (bf16-rounded). The reference
applies no 1/sqrt(d) attention scale (scale 1.0, src/text.rs:181): the learned q/k norm weights carry
it. With unit q/k norms the logits have standard deviation sqrt(head_dim) (16 to 23), attention is
argmax-like and the random network is chaotic -- a 1e-7 relative perturbation of the input moves a
700-token embedding by 6e-3 -- so no two implementations, even two f32 ones, could agree to any
tolerance. ``head_dim ** -0.25`` on both gives logits of unit scale, and then a 1e-4 perturbation
moves the embedding by ~1e-5. Each tensor draws from its own generator seeded by
``(seed, crc32(name))`` so the values do not depend on the order tensors are generated in.
"""
from __future__ import annotations

import json
import struct
import zlib
from pathlib import Path

import numpy as np

from .config import TextConfig, synthetic_config, write_config

_DT = {"BF16": (np.uint16, 2), "F16": (np.float16, 2), "F32": (np.float32, 4)}


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bit patterns (NaN-free inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


class SafeTensors:
    """Memory-mapped ``.safetensors`` reader with the checks of src/weights.rs:46-86."""

    def __init__(self, path: str | Path):
        self.path = Path(path)
        raw = np.memmap(self.path, dtype=np.uint8, mode="r")
        if raw.size < 8:
            raise ValueError("safetensors file too small")
        (hlen,) = struct.unpack("<Q", bytes(raw[:8]))
        if hlen > raw.size - 8:
            raise ValueError(f"corrupt safetensors header length in {self.path}")
        header = json.loads(bytes(raw[8 : 8 + hlen]))
        self._raw = raw
        self._start = 8 + hlen
        self.index: dict[str, tuple[str, list[int], int, int]] = {}
        for name, info in header.items():
            if name == "__metadata__":
                continue
            dt = info["dtype"]
            if dt not in _DT:
                raise ValueError(f"tensor {name}: unsupported dtype {dt}")
            s, e = info["data_offsets"]
            n = int(np.prod(info["shape"], dtype=np.int64)) if info["shape"] else 1
            if e < s or self._start + e > raw.size or n * _DT[dt][1] != e - s:
                raise ValueError(f"tensor {name}: bad offsets")
            self.index[name] = (dt, list(info["shape"]), s, e)

    def __contains__(self, name: str) -> bool:
        return name in self.index

    def raw(self, name: str) -> np.ndarray:
        dt, shape, s, e = self.index[name]
        np_t, _ = _DT[dt]
        return self._raw[self._start + s : self._start + e].view(np_t).reshape(shape)

    def f32(self, name: str, shape: list[int] | tuple[int, ...] | None = None) -> np.ndarray:
        if name not in self.index:
            raise KeyError(f"missing tensor `{name}`")
        dt, sh, _, _ = self.index[name]
        if shape is not None and list(shape) != sh:
            raise ValueError(f"tensor `{name}` has shape {sh}, expected {list(shape)}")
        r = self.raw(name)
        if dt == "BF16":
            return bf16_bits_to_f32(r).reshape(sh)
        return np.asarray(r, dtype=np.float32).reshape(sh)

    def scalar(self, name: str) -> float:
        v = self.f32(name).reshape(-1)
        if v.size != 1:
            raise ValueError(f"tensor `{name}` is not a scalar")
        return float(v[0])


def write_safetensors(path: str | Path, tensors: dict[str, np.ndarray]) -> None:
    """Write bf16 (uint16 bit patterns) or f32 arrays in the safetensors layout."""
    header: dict = {}
    off = 0
    order = sorted(tensors)
    for name in order:
        a = tensors[name]
        dt = "BF16" if a.dtype == np.uint16 else "F32"
        nb = a.size * a.itemsize
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + nb]}
        off += nb
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for name in order:
            f.write(np.ascontiguousarray(tensors[name]).tobytes())


def _normal_bf16(seed: int, name: str, shape: tuple[int, ...], std: float = 0.02) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64([seed, zlib.crc32(name.encode())]))
    x = rng.standard_normal(int(np.prod(shape)), dtype=np.float32) * np.float32(std)
    return f32_to_bf16_bits(x).reshape(shape)


_ONE_BF16 = np.uint16(0x3F80)


def text_tensor_specs(cfg: dict) -> list[tuple[str, tuple[int, ...], str]]:
    """(name, shape, init) for every text-tower tensor, names as src/text.rs:74-111."""
    t = cfg["text_config"]
    known = set(TextConfig.__dataclass_fields__)
    c = TextConfig(**{k: v for k, v in t.items() if k in known})
    h, p, ff, nh = c.hidden_size, c.hidden_size_per_layer_input, c.intermediate_size, c.num_attention_heads
    specs: list[tuple[str, tuple[int, ...], str]] = [
        ("language_model.embed_tokens.weight", (c.vocab_size, h), "normal"),
        ("language_model.norm.weight", (h,), "ones"),
        ("language_model.ple.per_layer_model_projection.weight", (c.num_hidden_layers * p, h), "normal"),
        ("language_model.ple.per_layer_projection_norm.weight", (p,), "ones"),
        ("language_model.embedding_projection.weight", (c.embedding_dim, h), "normal"),
    ]
    for i in range(c.num_hidden_layers):
        hd, nkv = c.layer_dims(i)
        pre = f"language_model.layers.{i}"
        specs += [
            (f"{pre}.input_layernorm.weight", (h,), "ones"),
            (f"{pre}.post_attention_layernorm.weight", (h,), "ones"),
            (f"{pre}.pre_feedforward_layernorm.weight", (h,), "ones"),
            (f"{pre}.post_feedforward_layernorm.weight", (h,), "ones"),
            (f"{pre}.self_attn.q_proj.weight", (nh * hd, h), "normal"),
            (f"{pre}.self_attn.k_proj.weight", (nkv * hd, h), "normal"),
            (f"{pre}.self_attn.v_proj.weight", (nkv * hd, h), "normal"),
            (f"{pre}.self_attn.o_proj.weight", (h, nh * hd), "normal"),
            (f"{pre}.self_attn.q_norm.weight", (hd,), "qk"),
            (f"{pre}.self_attn.k_norm.weight", (hd,), "qk"),
            (f"{pre}.mlp.gate_proj.weight", (ff, h), "normal"),
            (f"{pre}.mlp.up_proj.weight", (ff, h), "normal"),
            (f"{pre}.mlp.down_proj.weight", (h, ff), "normal"),
            (f"{pre}.ple_block.per_layer_input_gate.weight", (p, h), "normal"),
            (f"{pre}.ple_block.per_layer_projection.weight", (h, p), "normal"),
            (f"{pre}.ple_block.post_per_layer_input_norm.weight", (h,), "ones"),
            (f"{pre}.layer_scalar", (1,), "ones"),
        ]
    return specs


def vision_tensor_specs(cfg: dict) -> list[tuple[str, tuple[int, ...], str]]:
    """(name, shape, init) for every vision-tower tensor, names as src/vision.rs:184-217."""
    v = cfg["vision_config"]
    h, hd, nh, nkv, ff = v["hidden_size"], v["head_dim"], v["num_attention_heads"], v["num_key_value_heads"], v["intermediate_size"]
    th = cfg["text_config"]["hidden_size"]
    specs: list[tuple[str, tuple[int, ...], str]] = [
        ("vision_tower.patch_embedder.position_embedding_table", (2, v["position_embedding_size"], h), "normal"),
        ("vision_tower.patch_embedder.input_proj.weight", (h, 3 * v["patch_size"] ** 2), "normal"),
        ("embed_vision.embedding_projection.weight", (th, h), "normal"),
    ]
    for i in range(v["num_hidden_layers"]):
        p = f"vision_tower.encoder.layers.{i}"
        specs += [
            (f"{p}.self_attn.q_proj.linear.weight", (nh * hd, h), "normal"),
            (f"{p}.self_attn.k_proj.linear.weight", (nkv * hd, h), "normal"),
            (f"{p}.self_attn.v_proj.linear.weight", (nkv * hd, h), "normal"),
            (f"{p}.self_attn.o_proj.linear.weight", (h, nh * hd), "normal"),
            (f"{p}.self_attn.q_norm.weight", (hd,), "qk"),
            (f"{p}.self_attn.k_norm.weight", (hd,), "qk"),
            (f"{p}.mlp.gate_proj.linear.weight", (ff, h), "normal"),
            (f"{p}.mlp.up_proj.linear.weight", (ff, h), "normal"),
            (f"{p}.mlp.down_proj.linear.weight", (h, ff), "normal"),
            (f"{p}.input_layernorm.weight", (h,), "ones"),
            (f"{p}.post_attention_layernorm.weight", (h,), "ones"),
            (f"{p}.pre_feedforward_layernorm.weight", (h,), "ones"),
            (f"{p}.post_feedforward_layernorm.weight", (h,), "ones"),
        ]
    return specs


def make_random_checkpoint(
    dirpath: str | Path, seed: int = 0, cfg: dict | None = None, vision: bool = True, unit_qk_norms: bool = False
) -> Path:
    """Write ``config.json`` + ``model.safetensors`` (BF16) with seeded random-init weights.

    ``unit_qk_norms=True`` writes the workload's literal init (every norm weight 1, q/k norms included):
    the chaotic checkpoint described in the module docstring, kept for the test that shows why the
    default scales the q/k norms."""
    cfg = cfg or synthetic_config()
    d = Path(dirpath)
    write_config(d, cfg)
    specs = text_tensor_specs(cfg) + (vision_tensor_specs(cfg) if vision else [])
    tensors: dict[str, np.ndarray] = {}
    for name, shape, init in specs:
        if init == "ones":
            tensors[name] = np.full(shape, _ONE_BF16, dtype=np.uint16)
        elif init == "qk" and unit_qk_norms:
            tensors[name] = np.full(shape, _ONE_BF16, dtype=np.uint16)
        elif init == "qk":
            tensors[name] = np.full(shape, f32_to_bf16_bits(np.float32(shape[0] ** -0.25))[()], dtype=np.uint16)
        else:
            tensors[name] = _normal_bf16(seed, name, shape)
    out = d / "model.safetensors"
    write_safetensors(out, tensors)
    return out
