"""Generate the golden vectors that pin the CPU oracle's vision tower.

Same approach as make_golden.py for the text backbone: the reference's own image dumps
(testdata/image/*.soft.bin) were produced with Google's real weights, which are not available, so the
source of truth is rebuilt on the seeded random-init checkpoint from transformers' own Gemma4 vision
modules (``Gemma4VisionModel`` = patch embedder + encoder + pooler, and ``Gemma4MultimodalEmbedder``),
the modules src/vision.rs restates. The one substitution, as for the text: the rotary cos/sin tables are
evaluated the way the reference builds them (src/vision.rs:114-136; f32 angle, correctly rounded sin and
cos per axis) instead of by torch's vectorised cos. Outputs go to ``golden_vision.json``.

Run (CPU, under a minute):  python tests/golden/make_golden_vision.py
"""
from __future__ import annotations

import base64
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
from transformers.models.gemma4.configuration_gemma4 import Gemma4TextConfig, Gemma4VisionConfig  # noqa: E402

SEED = 0
# Patch grids (rows x columns): square, non-square, and one that pools to a single soft token.
CASES = [(6, 6), (3, 9), (3, 3)]


def hf_vision_config(vc: dict) -> Gemma4VisionConfig:
    c = Gemma4VisionConfig(
        hidden_size=vc["hidden_size"], intermediate_size=vc["intermediate_size"],
        num_hidden_layers=vc["num_hidden_layers"], num_attention_heads=vc["num_attention_heads"],
        num_key_value_heads=vc["num_key_value_heads"], head_dim=vc["head_dim"], rms_norm_eps=vc["rms_norm_eps"],
        pooling_kernel_size=vc["pooling_kernel_size"], patch_size=vc["patch_size"],
        position_embedding_size=vc["position_embedding_size"], use_clipped_linears=False, standardize=False,
        rope_parameters={"rope_type": "default", "rope_theta": vc["rope_parameters"]["rope_theta"]},
    )
    c._attn_implementation = "eager"
    return c


def reference_rope(pos: np.ndarray, inv_freq: np.ndarray) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin [1, n, head_dim]: per axis (x then y) the angles pos * inv_freq rounded to f32, their
    correctly rounded cos / sin, duplicated halves (the rotate-half layout)."""
    inv = inv_freq.astype(np.float32)
    cs, sn = [], []
    for axis in range(2):
        f = (pos[:, axis].astype(np.float32)[:, None] * inv[None, :]).astype(np.float32)
        c = np.vectorize(lambda a: np.float32(math.cos(float(a))), otypes=[np.float32])(f)
        s = np.vectorize(lambda a: np.float32(math.sin(float(a))), otypes=[np.float32])(f)
        cs += [c, c]
        sn += [s, s]
    return torch.from_numpy(np.concatenate(cs, 1))[None], torch.from_numpy(np.concatenate(sn, 1))[None]


def main() -> None:
    torch.set_num_threads(8)
    cfg = cfgmod.synthetic_config()
    vc = cfg["vision_config"]
    hcfg = hf_vision_config(vc)
    tcfg = Gemma4TextConfig(hidden_size=cfg["text_config"]["hidden_size"])
    out: dict = {"seed": SEED, "config": "synthetic_config()", "generator": "transformers "
                 + __import__("transformers").__version__ + " Gemma4VisionModel + Gemma4MultimodalEmbedder",
                 "cases": []}
    with tempfile.TemporaryDirectory() as d:
        wmod.make_random_checkpoint(d, seed=SEED, cfg=cfg, vision=True)
        st = wmod.SafeTensors(Path(d) / "model.safetensors")
        model = G.Gemma4VisionModel(hcfg).eval()
        model.load_state_dict({k: torch.from_numpy(st.f32(f"vision_tower.{k}").copy())
                               for k in model.state_dict()})
        emb = G.Gemma4MultimodalEmbedder(hcfg, tcfg).eval()
        emb.load_state_dict({k: torch.from_numpy(st.f32(f"embed_vision.{k}").copy()) for k in emb.state_dict()})
        inv_freq = model.encoder.rotary_emb.inv_freq.numpy()
        rng = np.random.default_rng(4321)
        for gh, gw in CASES:
            n = gh * gw
            patches = rng.random((n, 3 * vc["patch_size"] ** 2), dtype=np.float32)
            pos = np.array([[x, y] for y in range(gh) for x in range(gw)], dtype=np.int64)
            tables = reference_rope(pos, inv_freq)
            model.encoder.rotary_emb.forward = lambda x, position_ids, t=tables: t
            with torch.no_grad():
                pooled = model(pixel_values=torch.from_numpy(patches)[None],
                               pixel_position_ids=torch.from_numpy(pos)[None]).last_hidden_state
                soft = emb(pooled)
            # Patches as base64 of little-endian f32 (exact and compact).
            out["cases"].append({"grid": [gh, gw], "patches_f32_b64": base64.b64encode(patches.astype("<f4").tobytes()).decode(),
                                 "positions": pos.tolist(),
                                 "pooled": pooled.reshape(-1, vc["hidden_size"]).tolist(),
                                 "soft": soft.reshape(-1, cfg["text_config"]["hidden_size"]).tolist()})
            print(gh, gw, "done", file=sys.stderr)
    path = Path(__file__).with_name("golden_vision.json")
    path.write_text(json.dumps(out))
    print("wrote", path, path.stat().st_size, "bytes", file=sys.stderr)


if __name__ == "__main__":
    main()
