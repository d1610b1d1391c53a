"""Host-side mirror of the reference's backend interface over the B200 library.

The reference dispatches the towers through ``TextBackend`` / ``VisionBackend`` (src/backend.rs:57-96):
``embed_tokens(ids, out)``, ``forward_packed(embeds, lens) -> [rows, embedding_dim]`` and
``encode(img) -> soft tokens``. :class:`TextBackend` and :class:`VisionBackend` keep those names,
argument meanings and error behaviour (errors raise :class:`lib.Eg2Error`; an empty token sequence
is rejected like src/model.rs:522), backed by one device context (:class:`Device`). The pooled
path of ``EmbeddingGemma2::embed_ids`` + ``truncate_and_normalize`` (src/model.rs:498-540, :677-688)
is :meth:`TextBackend.embed_ids`.
"""
from __future__ import annotations

import ctypes as C
import json
from pathlib import Path

import numpy as np

from . import lib as L
from . import shard
from .config import ModelConfig

MATRYOSHKA_DIMS = (512, 256, 128)


class Device:
    """One CUDA device context with the model loaded (``eg2_open``)."""

    def __init__(self, model_dir: str | Path, device: int = 0, precision: str | int = "bf16"):
        self._lib = L.load()
        prec = L.PRECISIONS[precision] if isinstance(precision, str) else int(precision)
        h = C.c_void_p()
        rc = self._lib.eg2_open(int(device), prec, str(model_dir).encode(), C.byref(h))
        if rc != 0:
            msg = self._lib.eg2_last_error(None)
            raise L.Eg2Error(rc, msg.decode() if msg else "")
        self.handle = h
        self.device = int(device)
        self.precision = prec
        hidden, emb, layers = C.c_int(), C.c_int(), C.c_int()
        vocab = C.c_int64()
        L.check(self._lib.eg2_text_dims(h, C.byref(hidden), C.byref(emb), C.byref(vocab), C.byref(layers)), h)
        self.hidden, self.embedding_dim, self.vocab, self.layers = hidden.value, emb.value, vocab.value, layers.value
        self.cfg = ModelConfig.load(model_dir)

    def close(self) -> None:
        if getattr(self, "handle", None):
            self._lib.eg2_close(self.handle)
            self.handle = None

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass

    def check(self, rc: int) -> None:
        L.check(rc, self.handle)

    def set_stream(self, stream_ptr: int | None) -> None:
        self.check(self._lib.eg2_set_stream(self.handle, C.c_void_p(stream_ptr or 0)))

    def pass_policy(self) -> tuple[int, int]:
        """``(max_rows, precise_max)`` of this context's pass policy (:func:`plan_passes`)."""
        rows, pmax = C.c_int64(), C.c_int()
        self.check(self._lib.eg2_pass_policy(self.handle, C.byref(rows), C.byref(pmax)))
        return rows.value, pmax.value

    def profile(self, enable: bool) -> None:
        self.check(self._lib.eg2_profile(self.handle, 1 if enable else 0))

    def profile_read(self) -> dict:
        buf = C.create_string_buffer(1 << 16)
        self.check(self._lib.eg2_profile_read(self.handle, buf, len(buf)))
        return json.loads(buf.value.decode())


def plan_passes(lens, max_rows: int, precise_max: int = 0) -> list[tuple[list[int], bool]]:
    """The library's pass policy (``eg2_plan_passes``): ``[(sequence indices, runs_in_tf32), ...]``.

    Consecutive sequences in call order share a pass of at most ``max_rows`` rows, as the reference's
    ``embed_prepared`` packs inputs into passes of at most ``PACK_TOKENS`` rows (src/model.rs:508-521);
    sequences of at most ``precise_max`` tokens form their own (TF32) passes."""
    lens_l = [int(x) for x in lens]
    n = len(lens_l)
    pass_of = (C.c_int32 * max(1, n))()
    precise = (C.c_int32 * max(1, n))()
    rc = L.load().eg2_plan_passes(L.i32_array(lens_l), n, int(max_rows), int(precise_max), pass_of, precise)
    if rc < 0:
        raise L.Eg2Error(rc, "invalid pass-policy arguments")
    out = [([], bool(precise[p])) for p in range(rc)]
    for s in range(n):
        out[pass_of[s]][0].append(s)
    return out


class TextBackend:
    """GPU text backbone (``TextBackend::Gpu``, src/backend.rs:57-80)."""

    def __init__(self, dev: Device):
        self.dev = dev

    def embed_tokens(self, ids, out: np.ndarray | None = None) -> np.ndarray:
        """``embed_tokens[id] * sqrt(hidden)`` rows (src/text.rs:53-64)."""
        ids_a = np.ascontiguousarray(ids, dtype=np.uint32)
        if out is None:
            out = np.empty((len(ids_a), self.dev.hidden), dtype=np.float32)
        assert out.dtype == np.float32 and out.flags.c_contiguous and out.size == len(ids_a) * self.dev.hidden
        self.dev.check(self.dev._lib.eg2_embed_tokens(
            self.dev.handle, ids_a.ctypes.data_as(C.POINTER(C.c_uint32)), len(ids_a), out.ctypes.data_as(C.POINTER(C.c_float))))
        return out

    def forward_packed(self, embeds: np.ndarray, lens) -> np.ndarray:
        """Per-token states ``[rows, embedding_dim]`` of sequences packed back to back (src/backend.rs:73-79)."""
        lens_l = [int(x) for x in lens]
        if any(x <= 0 for x in lens_l):
            raise L.Eg2Error(-1, "empty token sequence")
        rows = sum(lens_l)
        embeds = np.ascontiguousarray(embeds, dtype=np.float32)
        if embeds.shape != (rows, self.dev.hidden):
            raise L.Eg2Error(-1, f"embeds shape {embeds.shape} does not match {rows} rows x {self.dev.hidden}")
        out = np.empty((rows, self.dev.embedding_dim), dtype=np.float32)
        if rows == 0:
            return out
        self.dev.check(self.dev._lib.eg2_forward_packed(
            self.dev.handle, embeds.ctypes.data, L.i32_array(lens_l), len(lens_l), out.ctypes.data))
        return out

    def forward_packed_device(self, embeds_ptr: int, lens, out_ptr: int, stream_ptr: int | None = None) -> None:
        """Device-pointer variant (e.g. ``torch.Tensor.data_ptr()``); lens stay on the host."""
        lens_l = [int(x) for x in lens]
        self.dev.check(self.dev._lib.eg2_forward_packed_device(
            self.dev.handle, C.c_void_p(embeds_ptr), L.i32_array(lens_l), len(lens_l), C.c_void_p(out_ptr),
            C.c_void_p(stream_ptr or 0)))

    def embed_ids(self, ids_list, dims=MATRYOSHKA_DIMS) -> dict[int, np.ndarray]:
        """Pooled, L2-normalised embeddings of token-id sequences in one packed pass, plus the
        Matryoshka cuts ``dims``: ``{embedding_dim: [n, 768], 512: [n, 512], ...}``."""
        seqs = [np.ascontiguousarray(x, dtype=np.uint32) for x in ids_list]
        lens = [len(s) for s in seqs]
        if any(x == 0 for x in lens):
            raise L.Eg2Error(-1, "empty token sequence")
        all_dims = [self.dev.embedding_dim] + [int(d) for d in dims]
        for d in all_dims:
            if d <= 0 or d > self.dev.embedding_dim:
                raise L.Eg2Error(-1, f"truncate_dim {d} out of range 1..={self.dev.embedding_dim}")
        ids = np.concatenate(seqs) if seqs else np.zeros(0, np.uint32)
        total = sum(all_dims)
        out = np.empty((len(seqs), total), dtype=np.float32)
        if seqs:
            self.dev.check(self.dev._lib.eg2_embed_packed(
                self.dev.handle, ids.ctypes.data, L.i32_array(lens), len(lens), L.i32_array(all_dims), len(all_dims),
                out.ctypes.data))
        res, off = {}, 0
        for d in all_dims:
            res[d] = out[:, off:off + d]
            off += d
        return res

    def embed_ids_device(self, ids_ptr: int, lens, dims, out_ptr: int, stream_ptr: int | None = None) -> None:
        lens_l = [int(x) for x in lens]
        d = [int(x) for x in dims]
        self.dev.check(self.dev._lib.eg2_embed_packed_device(
            self.dev.handle, C.c_void_p(ids_ptr), L.i32_array(lens_l), len(lens_l), L.i32_array(d), len(d),
            C.c_void_p(out_ptr), C.c_void_p(stream_ptr or 0)))


class VisionBackend:
    """GPU vision tower (``VisionBackend::Gpu``, src/backend.rs:82-96)."""

    def __init__(self, dev: Device):
        self.dev = dev

    def encode(self, patches: np.ndarray, positions: np.ndarray, grid_h: int, grid_w: int, pooled: bool = False):
        """Soft tokens ``[n / k^2, text_hidden]`` of one patched image (src/vision.rs:223-273);
        with ``pooled=True`` also the pooled tower states ``[n / k^2, vision_hidden]``."""
        patches = np.ascontiguousarray(patches, dtype=np.float32)
        pos = np.ascontiguousarray(positions, dtype=np.int32)
        n = grid_h * grid_w
        if patches.shape[0] != n or pos.shape != (n, 2):
            raise L.Eg2Error(-1, "malformed patches")
        vc = self.dev.cfg.vision
        if vc is None:
            raise L.Eg2Error(-1, "the checkpoint has no vision tower")
        k = vc.pooling_kernel_size
        n_out = (grid_h // k) * (grid_w // k)
        soft = np.empty((n_out, self.dev.hidden), dtype=np.float32)
        pooled_a = np.empty((n_out, vc.hidden_size), dtype=np.float32) if pooled else None
        self.dev.check(self.dev._lib.eg2_vision_encode(
            self.dev.handle, patches.ctypes.data, pos.ctypes.data_as(C.POINTER(C.c_int32)), grid_h, grid_w,
            pooled_a.ctypes.data if pooled else None, soft.ctypes.data))
        return (soft, pooled_a) if pooled else soft

    def encode_batch(self, patches: np.ndarray, positions: np.ndarray, grid_h: int, grid_w: int, pooled: bool = False,
                     out: np.ndarray | None = None):
        """Soft tokens ``[n_images, n / k^2, text_hidden]`` of several images of one patch grid in one
        device pass (``eg2_vision_encode_batch``); ``patches`` is ``[n_images, n, 3 p^2]``, the positions
        ``[n, 2]`` are shared. ``out`` (f32, C-contiguous, that shape) receives the soft tokens if given,
        e.g. a page-locked buffer."""
        patches = np.ascontiguousarray(patches, dtype=np.float32)
        pos = np.ascontiguousarray(positions, dtype=np.int32)
        n = grid_h * grid_w
        if patches.ndim != 3 or patches.shape[1] != n or pos.shape != (n, 2):
            raise L.Eg2Error(-1, "malformed patches")
        vc = self.dev.cfg.vision
        if vc is None:
            raise L.Eg2Error(-1, "the checkpoint has no vision tower")
        n_img = patches.shape[0]
        k = vc.pooling_kernel_size
        n_out = (grid_h // k) * (grid_w // k)
        soft = out if out is not None else np.empty((n_img, n_out, self.dev.hidden), dtype=np.float32)
        if soft.shape != (n_img, n_out, self.dev.hidden) or soft.dtype != np.float32 or not soft.flags.c_contiguous:
            raise L.Eg2Error(-1, "malformed output buffer")
        pooled_a = np.empty((n_img, n_out, vc.hidden_size), dtype=np.float32) if pooled else None
        self.dev.check(self.dev._lib.eg2_vision_encode_batch(
            self.dev.handle, patches.ctypes.data, pos.ctypes.data_as(C.POINTER(C.c_int32)), n_img, grid_h, grid_w,
            pooled_a.ctypes.data if pooled else None, soft.ctypes.data))
        return (soft, pooled_a) if pooled else soft


def embed_on_gpus(backends: list[TextBackend], ids_list, dims=MATRYOSHKA_DIMS):
    """Embed token-id sequences over several GPUs from one process: one :class:`TextBackend` (one
    device context) per GPU, each driven by its own host thread on its longest-first share of the
    documents (``shard.dispatch``). A GPU whose call fails with anything but an input error is dropped
    and its documents are re-queued on the others; a document with invalid input gets a
    ``shard.DocumentError`` in its slot. Returns ({dim: [n, dim] array}, report); rows of failed
    documents are NaN."""
    all_dims = [backends[0].dev.embedding_dim] + [int(d) for d in dims]
    total = sum(all_dims)

    def worker(tb):
        def embed(seqs):
            r = tb.embed_ids(seqs, dims)
            return np.concatenate([r[d] for d in all_dims], axis=1)
        return embed

    rows, report = shard.dispatch([worker(tb) for tb in backends], list(ids_list))
    flat = np.full((len(rows), total), np.nan, np.float32)
    for i, r in enumerate(rows):
        if not isinstance(r, shard.DocumentError):
            flat[i] = r
    out, off = {}, 0
    for d in all_dims:
        out[d] = flat[:, off:off + d]
        off += d
    return out, report
