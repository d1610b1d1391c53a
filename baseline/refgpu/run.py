"""Time the reference's own CUDA backend (cuBLAS + its CUDA kernels, built by baseline/refgpu/Makefile
into baseline/_ref/librefgpu.so) on this GPU, as a baseline beside bench.py's numbers.

What runs is the reference's bf16 path as its EmbeddingGemma2::embed_prepared drives it: consecutive
inputs packed greedily into passes of at most PACK_TOKENS = 2,048 rows, a longer input a pass of its
own (src/model.rs:157-158, :508-521); per pass GpuText::forward_packed (host embeddings in, per-token
states out, src/gpu/text.rs:436-529); mean pool and L2 on the host (src/model.rs:530-535). The
embedding gather is the reference's host code (src/text.rs:53-64), restated in numpy.

Checks first that the harness computes the model: the pooled embeddings of the first C3 documents
against the CPU oracle's (tests/golden/oracle_fixtures.npz) under the bf16 profile. Then times
(1) 64 documents of 2,208 tokens (the bench metric's workload; 64 passes), (2) C3's 64 mixed-length
documents, (3) one 17-token query per call (eager: the reference's CUDA-graph replay of short passes
is not restated). Prints one JSON line.

    python baseline/refgpu/run.py [--docs 64]
"""
from __future__ import annotations

import argparse
import ctypes as C
import importlib
import json
import statistics
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests" / "golden"))
W = importlib.import_module("embeddinggemma2-rust_b200.weights")
CFG = importlib.import_module("embeddinggemma2-rust_b200.config")
LIB = ROOT / "baseline" / "_ref" / "librefgpu.so"
PACK_TOKENS = 2048
BF16_MAX_ABS, BF16_MIN_COS = 4e-3, 0.99991  # src/verify.rs:104-110


def reference_pack(lens):
    """embed_prepared's greedy pack (src/model.rs:513-521)."""
    packs, start = [], 0
    while start < len(lens):
        end, rows = start + 1, lens[start]
        while end < len(lens) and rows + lens[end] <= PACK_TOKENS:
            rows += lens[end]
            end += 1
        packs.append(list(range(start, end)))
        start = end
    return packs


class RefGpu:
    def __init__(self, model_dir: Path, device: int = 0):
        self.lib = C.CDLL(str(LIB))
        self.lib.refgpu_error.restype = C.c_char_p
        cfg = CFG.ModelConfig.load(model_dir).text
        st = W.SafeTensors(Path(model_dir) / "model.safetensors")
        self.cfg, self.st = cfg, st
        nl = cfg.num_hidden_layers
        keep = []

        def bits(name):
            a = np.ascontiguousarray(st.raw(name))
            keep.append(a)
            return a

        def f32(name):
            a = np.ascontiguousarray(st.f32(name), dtype=np.float32)
            keep.append(a)
            return a

        ptrs = []
        for i in range(nl):
            P = f"language_model.layers.{i}."
            qkv = np.ascontiguousarray(np.concatenate([st.raw(P + f"self_attn.{x}_proj.weight") for x in "qkv"], axis=0))
            gu = np.ascontiguousarray(np.concatenate([st.raw(P + "mlp.gate_proj.weight"), st.raw(P + "mlp.up_proj.weight")], axis=0))
            keep += [qkv, gu]
            arrs = [qkv, bits(P + "self_attn.o_proj.weight"), gu, bits(P + "mlp.down_proj.weight"),
                    bits(P + "ple_block.per_layer_input_gate.weight"), bits(P + "ple_block.per_layer_projection.weight"),
                    f32(P + "input_layernorm.weight"), f32(P + "post_attention_layernorm.weight"),
                    f32(P + "pre_feedforward_layernorm.weight"), f32(P + "post_feedforward_layernorm.weight"),
                    f32(P + "self_attn.q_norm.weight"), f32(P + "self_attn.k_norm.weight"),
                    f32(P + "ple_block.post_per_layer_input_norm.weight")]
            ptrs += [a.ctypes.data for a in arrs]
        glob = [bits("language_model.ple.per_layer_model_projection.weight"), bits("language_model.embedding_projection.weight"),
                f32("language_model.ple.per_layer_projection_norm.weight"), f32("language_model.norm.weight")]
        dims = (C.c_int * 6)(cfg.hidden_size, cfg.hidden_size_per_layer_input, nl, cfg.num_attention_heads,
                             cfg.intermediate_size, cfg.embedding_dim)
        hd = (C.c_int * nl)(*[cfg.layer_dims(i)[0] for i in range(nl)])
        nkv = (C.c_int * nl)(*[cfg.layer_dims(i)[1] for i in range(nl)])
        win = (C.c_int * nl)(*[cfg.sliding_window if cfg.is_sliding(i) else -1 for i in range(nl)])
        th = (C.c_double * nl)(*[cfg.rope_theta(i) for i in range(nl)])
        ls = (C.c_float * nl)(*[st.scalar(f"language_model.layers.{i}.layer_scalar") for i in range(nl)])
        lw = (C.c_void_p * len(ptrs))(*ptrs)
        gw = (C.c_void_p * 4)(*[a.ctypes.data for a in glob])
        h = C.c_void_p()
        rc = self.lib.refgpu_open(device, dims, C.c_float(cfg.rms_norm_eps), hd, nkv, win, th, ls, lw, gw, C.byref(h))
        if rc != 0:
            raise RuntimeError(f"refgpu_open failed ({rc})")
        self.h = h
        self.table = st.raw("language_model.embed_tokens.weight")
        self.scale = np.float32(np.sqrt(np.float32(cfg.hidden_size)))

    def embed_tokens(self, ids):
        """src/text.rs:53-64: bf16 row widened to f32, times sqrt(hidden) in f32."""
        return W.bf16_bits_to_f32(self.table[np.asarray(ids, dtype=np.int64)]) * self.scale

    def forward_packed(self, embeds, lens):
        rows = int(sum(lens))
        out = np.empty((rows, self.cfg.embedding_dim), np.float32)
        ms = C.c_float()
        l = (C.c_int * len(lens))(*[int(x) for x in lens])
        rc = self.lib.refgpu_forward(self.h, np.ascontiguousarray(embeds, np.float32).ctypes.data_as(C.c_void_p), l,
                                     len(lens), out.ctypes.data_as(C.c_void_p), C.byref(ms))
        if rc != 0:
            raise RuntimeError(f"refgpu_forward failed: {self.lib.refgpu_error(self.h).decode()}")
        return out, ms.value

    def embed_prepared(self, seqs):
        """Returns (pooled [n, 768], device ms summed over passes)."""
        out, dev_ms = [], 0.0
        for pack in reference_pack([len(s) for s in seqs]):
            lens = [len(seqs[i]) for i in pack]
            e = self.embed_tokens(np.concatenate([seqs[i] for i in pack]))
            hidden, ms = self.forward_packed(e, lens)
            dev_ms += ms
            off = 0
            for n in lens:
                v = hidden[off:off + n].astype(np.float64).mean(axis=0)
                out.append((v / max(np.linalg.norm(v), 1e-12)).astype(np.float32))
                off += n
        return np.stack(out), dev_ms

    def close(self):
        self.lib.refgpu_close(self.h)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--docs", type=int, default=64)
    ap.add_argument("--parity-docs", type=int, default=8)
    args = ap.parse_args()
    import make_oracle_fixtures as M

    with tempfile.TemporaryDirectory() as d:
        W.make_random_checkpoint(d, seed=0, vision=False)
        r = RefGpu(Path(d))
        try:
            fx = np.load(ROOT / "tests" / "golden" / "oracle_fixtures.npz")
            c3 = M.case_ids("c3")
            got, _ = r.embed_prepared(c3[: args.parity_docs])
            want = fx["c3_emb"][: args.parity_docs]
            max_abs = float(np.abs(got - want).max())
            cos = float(((got * want).sum(1) / (np.linalg.norm(got, axis=1) * np.linalg.norm(want, axis=1))).min())
            parity = {"docs": args.parity_docs, "max_abs": max_abs, "min_cos": cos,
                      "passes_bf16_profile": bool(max_abs <= BF16_MAX_ABS and cos >= BF16_MIN_COS)}

            rng = np.random.default_rng(1000)
            docs = [rng.integers(0, 262144, size=2208).astype(np.uint32) for _ in range(args.docs)]
            r.embed_prepared(docs[:3])  # warm-up
            t0 = time.perf_counter()
            _, dev_ms = r.embed_prepared(docs)
            wall = time.perf_counter() - t0
            t0 = time.perf_counter()
            _, c3_dev_ms = r.embed_prepared(c3)
            c3_wall = time.perf_counter() - t0
            q = [np.random.default_rng(17).integers(0, 262144, size=17).astype(np.uint32)]
            for _ in range(3):
                r.embed_prepared(q)
            ts = []
            for _ in range(20):
                t0 = time.perf_counter()
                r.embed_prepared(q)
                ts.append(time.perf_counter() - t0)
        finally:
            r.close()
    line = {
        "baseline": "reference GPU backend (cuBLAS GemmEx + the reference's CUDA kernels, bf16), sm_100",
        "docs_2208": {"docs": args.docs, "passes": args.docs, "device_docs_per_s": round(args.docs / (dev_ms / 1e3), 2),
                      "e2e_docs_per_s": round(args.docs / wall, 2), "device_ms_per_doc": round(dev_ms / args.docs, 3),
                      "e2e_ms_per_doc": round(wall * 1e3 / args.docs, 3)},
        "mixed_c3": {"docs": len(c3), "passes": len(reference_pack([len(s) for s in c3])),
                     "device_docs_per_s": round(len(c3) / (c3_dev_ms / 1e3), 2), "e2e_docs_per_s": round(len(c3) / c3_wall, 2)},
        "query_17_ms_per_call": round(statistics.median(ts) * 1e3, 3),
        "parity_vs_oracle": parity,
        "timing": "device: CUDA events around each pass's enqueued layers; e2e: wall clock of embed_prepared "
                  "(host gather, H2D, pass, D2H, host pool), 1 GPU",
    }
    print(json.dumps(line))


if __name__ == "__main__":
    main()
