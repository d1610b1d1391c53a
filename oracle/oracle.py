"""ctypes front end of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Loads ``oracle/_build/libeg2_oracle.so`` (built by ``oracle/Makefile``) and exposes the reference's
CPU f32 path on a checkpoint in the reference's safetensors layout:

* :class:`OracleText` -- ``TextModel::forward_packed`` (src/text.rs:136-235) and the embedding
  gather ``embed_tokens`` (src/text.rs:53-64);
* :class:`OracleVision` -- ``VisionTower::encode`` (src/vision.rs:223-273);
* :func:`pool`, :func:`truncate_and_normalize` -- src/model.rs:530-535, :677-688;
* :func:`sgemm_nt`, :func:`attention_packed` -- single ops for the GEMM sweep and attention checks.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may use this module. The
product library never calls it.
"""
from __future__ import annotations

import ctypes as C
import importlib
import os
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
LIB_PATH = HERE / "_build" / "libeg2_oracle.so"

if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
pkg = importlib.import_module("embeddinggemma2-rust_b200")
from_cfg = importlib.import_module("embeddinggemma2-rust_b200.config")
wmod = importlib.import_module("embeddinggemma2-rust_b200.weights")

_F = C.POINTER(C.c_float)
_FF = C.POINTER(_F)


def build() -> Path:
    """Compile the oracle with its Makefile (gcc + OpenMP)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        l = C.CDLL(str(LIB_PATH))
        l.eg2o_sgemm_nt.argtypes = [C.c_int, C.c_int, C.c_int, _F, _F, _F]
        l.eg2o_attention_packed.argtypes = [_F, _F, _F, C.POINTER(C.c_int64), C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _F]
        l.eg2o_text_forward_packed.argtypes = [C.c_void_p, _F, C.POINTER(C.c_int64), C.c_int, _F]
        l.eg2o_text_forward_packed.restype = C.c_int
        l.eg2o_vision_encode.argtypes = [C.c_void_p, _F, C.POINTER(C.c_int32), C.c_int, C.c_int, _F, _F]
        l.eg2o_vision_encode.restype = C.c_int
        l.eg2o_pool.argtypes = [_F, C.POINTER(C.c_int64), C.c_int, C.c_int, _F]
        l.eg2o_l2_normalize.argtypes = [_F, C.c_int]
        l.eg2o_embed_tokens.argtypes = [C.POINTER(C.c_uint16), C.c_long, C.c_int, C.POINTER(C.c_uint32), C.c_long, _F]
        l.eg2o_embed_tokens.restype = C.c_int
        l.eg2o_gelu_tanh.argtypes = [C.c_float]
        l.eg2o_gelu_tanh.restype = C.c_float
        l.eg2o_num_threads.restype = C.c_int
        l.eg2o_set_threads.argtypes = [C.c_int]
        l.eg2o_rms_norm.argtypes = [_F, C.c_long, C.c_int, _F, C.c_float]
        _lib = l
    return _lib


def _fp(a: np.ndarray) -> _F:
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_F)


def set_threads(n: int) -> None:
    lib().eg2o_set_threads(int(n))


def num_threads() -> int:
    return int(lib().eg2o_num_threads())


def sgemm_nt(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """``x[m,k] . w[n,k]^T`` in f32 (src/ops.rs:131-137)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    m, k = x.shape
    n = w.shape[0]
    out = np.empty((m, n), dtype=np.float32)
    lib().eg2o_sgemm_nt(m, n, k, _fp(x), _fp(w), _fp(out))
    return out


def attention_packed(q, k, v, lens, nh: int, nkv: int, hd: int, window: int | None) -> np.ndarray:
    """Block-diagonal attention (src/ops.rs:364-444, src/text.rs:183-202). ``window=None`` is global."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    lens_a = np.ascontiguousarray(lens, dtype=np.int64)
    out = np.zeros((int(lens_a.sum()), nh * hd), dtype=np.float32)
    lib().eg2o_attention_packed(
        _fp(q), _fp(k), _fp(v), lens_a.ctypes.data_as(C.POINTER(C.c_int64)), len(lens_a), nh, nkv, hd,
        -1 if window is None else int(window), _fp(out),
    )
    return out


def gelu_tanh(x: float) -> float:
    return float(lib().eg2o_gelu_tanh(float(x)))


def pool(hidden: np.ndarray, lens) -> np.ndarray:
    """Mean over each sequence's rows, then L2 (src/model.rs:530-535)."""
    hidden = np.ascontiguousarray(hidden, dtype=np.float32)
    lens_a = np.ascontiguousarray(lens, dtype=np.int64)
    dim = hidden.shape[1]
    out = np.empty((len(lens_a), dim), dtype=np.float32)
    lib().eg2o_pool(_fp(hidden), lens_a.ctypes.data_as(C.POINTER(C.c_int64)), len(lens_a), dim, _fp(out))
    return out


def truncate_and_normalize(v: np.ndarray, dim: int) -> np.ndarray:
    """Matryoshka: keep the first ``dim`` components and re-normalise (src/model.rs:677-688)."""
    n = v.shape[-1]
    if dim == 0 or dim > n:
        raise ValueError(f"truncate_dim {dim} out of range 1..={n}")
    out = np.ascontiguousarray(v[..., :dim], dtype=np.float32).copy()
    if dim < n:
        for row in out.reshape(-1, dim):
            r = np.ascontiguousarray(row)
            lib().eg2o_l2_normalize(_fp(r), dim)
            row[:] = r
    return out


class _Text(C.Structure):
    _fields_ = [
        ("hidden", C.c_int), ("ple_dim", C.c_int), ("n_layers", C.c_int), ("n_heads", C.c_int),
        ("emb_dim", C.c_int), ("inter", C.c_int), ("window", C.c_int), ("eps", C.c_float),
        ("head_dim", C.POINTER(C.c_int)), ("n_kv", C.POINTER(C.c_int)), ("sliding", C.POINTER(C.c_int)),
        ("theta", C.POINTER(C.c_double)), ("layer_scalar", _F),
    ] + [(n, _FF) for n in (
        "input_ln", "post_attn_ln", "pre_ff_ln", "post_ff_ln", "q_proj", "k_proj", "v_proj", "o_proj",
        "q_norm", "k_norm", "gate_proj", "up_proj", "down_proj", "ple_gate", "ple_proj", "ple_post_norm",
    )] + [(n, _F) for n in ("final_norm", "ple_model_proj", "ple_norm", "embed_proj")]


_TEXT_PER_LAYER = {
    "input_ln": "input_layernorm.weight",
    "post_attn_ln": "post_attention_layernorm.weight",
    "pre_ff_ln": "pre_feedforward_layernorm.weight",
    "post_ff_ln": "post_feedforward_layernorm.weight",
    "q_proj": "self_attn.q_proj.weight",
    "k_proj": "self_attn.k_proj.weight",
    "v_proj": "self_attn.v_proj.weight",
    "o_proj": "self_attn.o_proj.weight",
    "q_norm": "self_attn.q_norm.weight",
    "k_norm": "self_attn.k_norm.weight",
    "gate_proj": "mlp.gate_proj.weight",
    "up_proj": "mlp.up_proj.weight",
    "down_proj": "mlp.down_proj.weight",
    "ple_gate": "ple_block.per_layer_input_gate.weight",
    "ple_proj": "ple_block.per_layer_projection.weight",
    "ple_post_norm": "ple_block.post_per_layer_input_norm.weight",
}


class OracleText:
    """``TextModel`` (src/text.rs:39-235) on the CPU oracle, loaded from a checkpoint directory."""

    def __init__(self, model_dir: str | Path):
        d = Path(model_dir)
        self.cfg = from_cfg.ModelConfig.load(d).text
        self.st = wmod.SafeTensors(d / "model.safetensors")
        c = self.cfg
        self._keep: list = []
        s = _Text()
        s.hidden, s.ple_dim, s.n_layers = c.hidden_size, c.hidden_size_per_layer_input, c.num_hidden_layers
        s.n_heads, s.emb_dim, s.inter, s.window = c.num_attention_heads, c.embedding_dim, c.intermediate_size, c.sliding_window
        s.eps = c.rms_norm_eps
        nl = c.num_hidden_layers
        dims = [c.layer_dims(i) for i in range(nl)]
        hd = (C.c_int * nl)(*[d_[0] for d_ in dims])
        nkv = (C.c_int * nl)(*[d_[1] for d_ in dims])
        sl = (C.c_int * nl)(*[1 if c.is_sliding(i) else 0 for i in range(nl)])
        th = (C.c_double * nl)(*[c.rope_theta(i) for i in range(nl)])
        ls = np.array([self.st.scalar(f"language_model.layers.{i}.layer_scalar") for i in range(nl)], dtype=np.float32)
        self._keep += [hd, nkv, sl, th, ls]
        s.head_dim, s.n_kv, s.sliding, s.theta, s.layer_scalar = hd, nkv, sl, th, _fp(ls)
        for field, suffix in _TEXT_PER_LAYER.items():
            arrs = [np.ascontiguousarray(self.st.f32(f"language_model.layers.{i}.{suffix}")) for i in range(nl)]
            ptrs = (_F * nl)(*[_fp(a) for a in arrs])
            self._keep += [arrs, ptrs]
            setattr(s, field, ptrs)
        for field, name in (
            ("final_norm", "language_model.norm.weight"),
            ("ple_model_proj", "language_model.ple.per_layer_model_projection.weight"),
            ("ple_norm", "language_model.ple.per_layer_projection_norm.weight"),
            ("embed_proj", "language_model.embedding_projection.weight"),
        ):
            a = np.ascontiguousarray(self.st.f32(name))
            self._keep.append(a)
            setattr(s, field, _fp(a))
        self._s = s

    def embed_tokens(self, ids) -> np.ndarray:
        """Scaled token embeddings (src/text.rs:53-64)."""
        table = np.ascontiguousarray(self.st.raw("language_model.embed_tokens.weight"))
        ids_a = np.ascontiguousarray(ids, dtype=np.uint32)
        h = self.cfg.hidden_size
        out = np.empty((len(ids_a), h), dtype=np.float32)
        rc = lib().eg2o_embed_tokens(
            table.ctypes.data_as(C.POINTER(C.c_uint16)), table.shape[0], h,
            ids_a.ctypes.data_as(C.POINTER(C.c_uint32)), len(ids_a), _fp(out),
        )
        if rc != 0:
            raise ValueError("token id out of range")
        return out

    def forward_packed(self, embeds: np.ndarray, lens) -> np.ndarray:
        """Per-token states ``[rows, embedding_dim]`` (src/text.rs:136-235)."""
        embeds = np.ascontiguousarray(embeds, dtype=np.float32)
        lens_a = np.ascontiguousarray(lens, dtype=np.int64)
        rows = int(lens_a.sum())
        if embeds.shape != (rows, self.cfg.hidden_size):
            raise ValueError(f"embeds shape {embeds.shape} does not match {rows} rows")
        out = np.empty((rows, self.cfg.embedding_dim), dtype=np.float32)
        rc = lib().eg2o_text_forward_packed(C.byref(self._s), _fp(embeds), lens_a.ctypes.data_as(C.POINTER(C.c_int64)), len(lens_a), _fp(out))
        if rc != 0:
            raise ValueError("empty token sequence")
        return out

    def embed_ids(self, ids_list) -> np.ndarray:
        """Pooled, L2-normalised 768-d embeddings of token-id sequences packed into one pass."""
        lens = [len(x) for x in ids_list]
        emb = self.embed_tokens(np.concatenate([np.asarray(x, dtype=np.uint32) for x in ids_list]))
        return pool(self.forward_packed(emb, lens), lens)


class _Vision(C.Structure):
    _fields_ = [
        ("hidden", C.c_int), ("inter", C.c_int), ("n_layers", C.c_int), ("n_heads", C.c_int), ("n_kv", C.c_int),
        ("head_dim", C.c_int), ("patch_dim", C.c_int), ("pool_k", C.c_int), ("pos_size", C.c_int),
        ("text_hidden", C.c_int), ("eps", C.c_float), ("theta", C.c_double),
        ("pos_table", _F), ("input_proj", _F), ("embed_proj", _F),
    ] + [(n, _FF) for n in (
        "q_proj", "k_proj", "v_proj", "o_proj", "q_norm", "k_norm", "gate_proj", "up_proj", "down_proj",
        "input_ln", "post_attn_ln", "pre_ff_ln", "post_ff_ln",
    )]


_VISION_PER_LAYER = {
    "q_proj": "self_attn.q_proj.linear.weight",
    "k_proj": "self_attn.k_proj.linear.weight",
    "v_proj": "self_attn.v_proj.linear.weight",
    "o_proj": "self_attn.o_proj.linear.weight",
    "q_norm": "self_attn.q_norm.weight",
    "k_norm": "self_attn.k_norm.weight",
    "gate_proj": "mlp.gate_proj.linear.weight",
    "up_proj": "mlp.up_proj.linear.weight",
    "down_proj": "mlp.down_proj.linear.weight",
    "input_ln": "input_layernorm.weight",
    "post_attn_ln": "post_attention_layernorm.weight",
    "pre_ff_ln": "pre_feedforward_layernorm.weight",
    "post_ff_ln": "post_feedforward_layernorm.weight",
}


class OracleVision:
    """``VisionTower`` (src/vision.rs:41-273) on the CPU oracle."""

    def __init__(self, model_dir: str | Path):
        d = Path(model_dir)
        mc = from_cfg.ModelConfig.load(d)
        self.cfg = mc.vision
        self.st = wmod.SafeTensors(d / "model.safetensors")
        v = self.cfg
        s = _Vision()
        s.hidden, s.inter, s.n_layers, s.n_heads, s.n_kv = v.hidden_size, v.intermediate_size, v.num_hidden_layers, v.num_attention_heads, v.num_key_value_heads
        s.head_dim, s.patch_dim, s.pool_k, s.pos_size = v.head_dim, 3 * v.patch_size**2, v.pooling_kernel_size, v.position_embedding_size
        s.text_hidden, s.eps, s.theta = mc.text.hidden_size, v.rms_norm_eps, float(v.rope_parameters["rope_theta"])
        self._keep: list = []
        nl = v.num_hidden_layers
        for field, suffix in _VISION_PER_LAYER.items():
            arrs = [np.ascontiguousarray(self.st.f32(f"vision_tower.encoder.layers.{i}.{suffix}")) for i in range(nl)]
            ptrs = (_F * nl)(*[_fp(a) for a in arrs])
            self._keep += [arrs, ptrs]
            setattr(s, field, ptrs)
        for field, name in (
            ("pos_table", "vision_tower.patch_embedder.position_embedding_table"),
            ("input_proj", "vision_tower.patch_embedder.input_proj.weight"),
            ("embed_proj", "embed_vision.embedding_projection.weight"),
        ):
            a = np.ascontiguousarray(self.st.f32(name))
            self._keep.append(a)
            setattr(s, field, _fp(a))
        self._s = s

    def encode(self, patches: np.ndarray, positions: np.ndarray, grid_h: int, grid_w: int):
        """Returns ``(pooled [n/k^2, 768] before the embedder, soft tokens [n/k^2, 512])``."""
        patches = np.ascontiguousarray(patches, dtype=np.float32)
        pos = np.ascontiguousarray(positions, dtype=np.int32)
        k = self.cfg.pooling_kernel_size
        n_out = (grid_h // k) * (grid_w // k)
        pooled = np.empty((n_out, self.cfg.hidden_size), dtype=np.float32)
        soft = np.empty((n_out, int(self._s.text_hidden)), dtype=np.float32)
        rc = lib().eg2o_vision_encode(C.byref(self._s), _fp(patches), pos.ctypes.data_as(C.POINTER(C.c_int32)), grid_h, grid_w, _fp(pooled), _fp(soft))
        if rc != 0:
            raise ValueError(f"malformed patched image (code {rc})")
        return pooled, soft
