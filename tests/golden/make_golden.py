"""Generate the golden vectors that pin the CPU oracle.

The reference's own golden dumps (testdata/ref_text.json, testdata/image/*.soft.bin) were produced by
PyTorch / sentence-transformers on Google's real weights (tools/ref_text.py), which are not available.
This script reproduces that source of truth on the seeded random-init checkpoint instead: the text
backbone is assembled from transformers' own ``Gemma4`` modules (``Gemma4TextDecoderLayer``,
``Gemma4RMSNorm``, ``Gemma4TextRotaryEmbedding``), the modules src/text.rs restates, and the vision
tower from ``Gemma4VisionModel`` pieces where they exist. Outputs go to ``golden_text.json``.

Run (CPU, about a minute):  python tests/golden/make_golden.py
"""
from __future__ import annotations

import importlib
import json
import math
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
cfgmod = importlib.import_module("embeddinggemma2-rust_b200.config")
wmod = importlib.import_module("embeddinggemma2-rust_b200.weights")

from transformers.models.gemma4 import modeling_gemma4 as G  # noqa: E402
from transformers.models.gemma4.configuration_gemma4 import Gemma4TextConfig  # noqa: E402

SEED = 0
# Token-id cases: lengths at tile edges, a packed batch, and a document longer than the window
# radius (so the sliding-window mask and the global layers differ).
CASES = [
    {"name": "query17", "lens": [17]},
    {"name": "packed3", "lens": [3, 27, 100]},
    {"name": "doc700", "lens": [700]},
]
TRUNC = (512, 256, 128)


def hf_text_configs(tc: dict) -> tuple[Gemma4TextConfig, Gemma4TextConfig]:
    common = dict(
        vocab_size=tc["vocab_size"], hidden_size=tc["hidden_size"], intermediate_size=tc["intermediate_size"],
        num_hidden_layers=tc["num_hidden_layers"], num_attention_heads=tc["num_attention_heads"],
        head_dim=tc["head_dim"], global_head_dim=512, hidden_activation="gelu_pytorch_tanh",
        rms_norm_eps=tc["rms_norm_eps"], sliding_window=tc["sliding_window"], layer_types=tc["layer_types"],
        hidden_size_per_layer_input=tc["hidden_size_per_layer_input"], vocab_size_per_layer_input=8,
        attention_k_eq_v=False, num_kv_shared_layers=0, enable_moe_block=False, use_double_wide_mlp=False,
        attention_bias=False,
        rope_parameters={
            "sliding_attention": {"rope_type": "default", "rope_theta": tc["rope_parameters"]["sliding_attention"]["rope_theta"]},
            "full_attention": {"rope_type": "default", "rope_theta": tc["rope_parameters"]["full_attention"]["rope_theta"]},
        },
    )
    sliding = Gemma4TextConfig(num_key_value_heads=2, **common)
    glob = Gemma4TextConfig(num_key_value_heads=1, **common)
    for c in (sliding, glob):
        c._attn_implementation = "eager"
    return sliding, glob


def rope_tables(L: int, inv_freq: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin ``[1, L, hd]`` from transformers' inverse frequencies, evaluated as src/ops.rs:298-314
    does: the angle ``pos * inv_freq`` rounded to f32, then a correctly rounded f32 sin and cos (the
    reference's libm ``sin_cos``). transformers' own vectorised cos differs from that by up to ~16 ulp,
    and a 24-layer stack with random weights amplifies such table differences into the 1e-4 range."""
    inv = inv_freq.numpy().astype(np.float32)
    f = (np.arange(L, dtype=np.float32)[:, None] * inv[None, :]).astype(np.float32)
    c = np.vectorize(lambda a: np.float32(math.cos(float(a))), otypes=[np.float32])(f)
    s_ = np.vectorize(lambda a: np.float32(math.sin(float(a))), otypes=[np.float32])(f)
    c, s_ = np.concatenate([c, c], 1), np.concatenate([s_, s_], 1)
    return torch.from_numpy(c)[None], torch.from_numpy(s_)[None]


def load_linear(st, name: str) -> torch.nn.Linear:
    w = torch.from_numpy(st.f32(name).copy())
    lin = torch.nn.Linear(w.shape[1], w.shape[0], bias=False)
    lin.weight.data.copy_(w)
    return lin


def build_text(st, tc: dict):
    sl_cfg, gl_cfg = hf_text_configs(tc)
    layers = []
    for i in range(tc["num_hidden_layers"]):
        cfg = sl_cfg if tc["layer_types"][i] == "sliding_attention" else gl_cfg
        layer = G.Gemma4TextDecoderLayer(cfg, i).eval()
        sd = {}
        pre = f"language_model.layers.{i}"
        for k in layer.state_dict():
            if k == "layer_scalar":
                sd[k] = torch.tensor([st.scalar(f"{pre}.layer_scalar")])
                continue
            src = k.replace("per_layer_input_gate", "ple_block.per_layer_input_gate").replace(
                "per_layer_projection", "ple_block.per_layer_projection").replace(
                "post_per_layer_input_norm", "ple_block.post_per_layer_input_norm")
            sd[k] = torch.from_numpy(st.f32(f"{pre}.{src}").copy())
        layer.load_state_dict(sd)
        layers.append(layer)
    # A rotary module per head width: the sliding one from the sliding config, the global one from a
    # config whose head_dim is the global 512 (the reference rotates the whole 512-wide head with
    # theta_full, src/text.rs:158-161).
    rot_sl = G.Gemma4TextRotaryEmbedding(sl_cfg)
    gl_rot_cfg = Gemma4TextConfig(**{**gl_cfg.to_dict(), "head_dim": 512})
    rot_gl = G.Gemma4TextRotaryEmbedding(gl_rot_cfg)
    h, p, nl = tc["hidden_size"], tc["hidden_size_per_layer_input"], tc["num_hidden_layers"]
    ple_proj = load_linear(st, "language_model.ple.per_layer_model_projection.weight")
    ple_norm = G.Gemma4RMSNorm(p, eps=tc["rms_norm_eps"])
    ple_norm.weight.data.copy_(torch.from_numpy(st.f32("language_model.ple.per_layer_projection_norm.weight").copy()))
    final_norm = G.Gemma4RMSNorm(h, eps=tc["rms_norm_eps"])
    final_norm.weight.data.copy_(torch.from_numpy(st.f32("language_model.norm.weight").copy()))
    emb_proj = load_linear(st, "language_model.embedding_projection.weight")

    @torch.no_grad()
    def forward_one(x: torch.Tensor) -> torch.Tensor:
        """One sequence [L, h] -> per-token states [L, 768]."""
        L = x.shape[0]
        xb = x[None]
        ple = ple_proj(xb) * (h**-0.5)
        ple = ple_norm(ple.reshape(1, L, nl, p))
        cs_sl = rope_tables(L, rot_sl.sliding_attention_inv_freq)
        cs_gl = rope_tables(L, rot_gl.full_attention_inv_freq)
        idx = torch.arange(L)
        band = (idx[:, None] - idx[None, :]).abs() <= tc["sliding_window"]
        m_sl = torch.zeros(L, L).masked_fill(~band, float("-inf"))[None, None]
        m_gl = torch.zeros(1, 1, L, L)
        hs = xb
        for i, layer in enumerate(layers):
            sliding = tc["layer_types"][i] == "sliding_attention"
            hs = layer(hs, per_layer_input=ple[:, :, i, :], position_embeddings=cs_sl if sliding else cs_gl,
                       attention_mask=m_sl if sliding else m_gl)
        return emb_proj(final_norm(hs))[0]

    return forward_one


def main() -> None:
    torch.set_num_threads(8)
    cfg = cfgmod.synthetic_config()
    tc = cfg["text_config"]
    out: dict = {"seed": SEED, "config": "synthetic_config()", "generator": "transformers "
                 + __import__("transformers").__version__ + " Gemma4 modules", "cases": []}
    with tempfile.TemporaryDirectory() as d:
        wmod.make_random_checkpoint(d, seed=SEED, cfg=cfg, vision=False)
        st = wmod.SafeTensors(Path(d) / "model.safetensors")
        fwd = build_text(st, tc)
        table = st.raw("language_model.embed_tokens.weight")
        rng = np.random.default_rng(1234)
        for case in CASES:
            lens = case["lens"]
            ids = [rng.integers(0, tc["vocab_size"], size=l).tolist() for l in lens]
            embs, hidden_rows = [], []
            for seq_ids in ids:
                # Scaled embedding gather (src/text.rs:53-64), in torch.
                e = torch.from_numpy(wmod.bf16_bits_to_f32(table[np.asarray(seq_ids)])) * torch.tensor(float(np.sqrt(np.float32(512))), dtype=torch.float32)
                hs = fwd(e)
                pooled = torch.nn.functional.normalize(hs.double().mean(0), dim=0).float()
                entry = {"emb": pooled.tolist()}
                for dcut in TRUNC:
                    entry[f"emb{dcut}"] = torch.nn.functional.normalize(pooled[:dcut].double(), dim=0).float().tolist()
                embs.append(entry)
                hidden_rows.append({"first": hs[0].tolist(), "last": hs[-1].tolist()})
            out["cases"].append({"name": case["name"], "lens": lens, "ids": ids, "outputs": embs, "rows": hidden_rows})
            print(case["name"], "done", file=sys.stderr)
    path = Path(__file__).with_name("golden_text.json")
    path.write_text(json.dumps(out))
    print("wrote", path, path.stat().st_size, "bytes", file=sys.stderr)


if __name__ == "__main__":
    main()
