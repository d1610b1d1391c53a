"""ctypes binding of ``_lib/libeg2_b200.so`` (the C ABI in include/eg2.h).

The library is the only compute path: if it is missing or fails to load, every call raises. There
is no CPU fallback in the product.
"""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_lib" / "libeg2_b200.so"
HEADER = HERE.parent / "include" / "eg2.h"

EG2_F32, EG2_TF32, EG2_BF16 = 0, 1, 2
PRECISIONS = {"f32": EG2_F32, "fp32": EG2_F32, "float32": EG2_F32, "tf32": EG2_TF32, "bf16": EG2_BF16}
ERRORS = {0: "ok", -1: "invalid argument", -2: "out of memory", -3: "CUDA error", -4: "device wait timed out", -5: "I/O error"}


class Eg2Error(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


_lib: C.CDLL | None = None
_P = C.c_void_p
_I32P = C.POINTER(C.c_int32)
_U32P = C.POINTER(C.c_uint32)
_FP = C.POINTER(C.c_float)


def exported_symbols() -> list[str]:
    """Function names declared in include/eg2.h."""
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"\b(eg2_[a-z_]+)\s*\(", text)


def load(build_if_missing: bool = True) -> C.CDLL:
    """Load the library (building it with nvcc first if it is absent and nvcc exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists() and build_if_missing:
        from . import build as _build  # noqa: WPS433 (local import: nvcc only needed here)

        _build.build()
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `python embeddinggemma2-rust_b200/build.py`")
    lib = C.CDLL(str(LIB_PATH))
    sig = {
        "eg2_open": (C.c_int, [C.c_int, C.c_int, C.c_char_p, C.POINTER(_P)]),
        "eg2_close": (None, [_P]),
        "eg2_last_error": (C.c_char_p, [_P]),
        "eg2_text_dims": (C.c_int, [_P, C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_int64), C.POINTER(C.c_int)]),
        "eg2_embed_tokens": (C.c_int, [_P, _U32P, C.c_int64, _FP]),
        "eg2_forward_packed": (C.c_int, [_P, _P, _I32P, C.c_int, _P]),
        "eg2_forward_packed_device": (C.c_int, [_P, _P, _I32P, C.c_int, _P, _P]),
        "eg2_embed_packed": (C.c_int, [_P, _P, _I32P, C.c_int, _I32P, C.c_int, _P]),
        "eg2_embed_packed_device": (C.c_int, [_P, _P, _I32P, C.c_int, _I32P, C.c_int, _P, _P]),
        "eg2_vision_encode": (C.c_int, [_P, _P, _I32P, C.c_int, C.c_int, _P, _P]),
        "eg2_vision_encode_batch": (C.c_int, [_P, _P, _I32P, C.c_int, C.c_int, C.c_int, _P, _P]),
        "eg2_set_stream": (C.c_int, [_P, _P]),
        "eg2_profile": (C.c_int, [_P, C.c_int]),
        "eg2_profile_read": (C.c_int, [_P, C.c_char_p, C.c_int]),
        "eg2_gemm": (C.c_int, [C.c_int, _P, C.c_int64, _P, C.c_int64, _P, C.c_int64, C.c_int, C.c_int, C.c_int, C.c_int, _P]),
        "eg2_attention": (C.c_int, [C.c_int, _P, _P, _P, _P, _I32P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _P]),
        "eg2_attention_noalloc": (C.c_int, [_P, _P, _P, _P, _I32P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _P]),
        "eg2_plan_passes": (C.c_int, [_I32P, C.c_int, C.c_int64, C.c_int, _I32P, _I32P]),
        "eg2_pass_policy": (C.c_int, [_P, C.POINTER(C.c_int64), C.POINTER(C.c_int)]),
        "eg2_launch_count": (C.c_longlong, []),
        "eg2_device_status": (C.c_int, []),
        "eg2_device_status_reset": (None, []),
        "eg2_wait_timeout_probe": (C.c_int, [C.c_int, C.c_uint, C.POINTER(C.c_int)]),
    }
    for name, (res, args) in sig.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    _lib = lib
    return lib


def check(rc: int, ctx=None) -> None:
    if rc != 0:
        msg = load().eg2_last_error(ctx)
        raise Eg2Error(rc, msg.decode() if msg else "")


def i32_array(values) -> C.Array:
    vals = [int(v) for v in values]
    return (C.c_int32 * max(1, len(vals)))(*vals)
