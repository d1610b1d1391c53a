"""The C-ABI library builds, loads and exports every function include/eg2.h declares (no GPU needed)."""
import ctypes

from conftest import pkg

L = pkg("lib")


def test_header_declares_the_boundary():
    names = set(L.exported_symbols())
    for n in ("eg2_open", "eg2_close", "eg2_last_error", "eg2_embed_tokens", "eg2_forward_packed",
              "eg2_embed_packed", "eg2_vision_encode", "eg2_gemm", "eg2_attention"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = L.load()
    for name in L.exported_symbols():
        assert hasattr(lib, name), name
        assert ctypes.cast(getattr(lib, name), ctypes.c_void_p).value


def test_open_rejects_bad_arguments_without_touching_a_gpu():
    lib = L.load()
    h = ctypes.c_void_p()
    assert lib.eg2_open(0, 7, b"/nonexistent", ctypes.byref(h)) == -1
    assert lib.eg2_last_error(None)
