"""CPU checks of the C-ABI library: it loads without a GPU and exports every
symbol declared in include/streamindex_b200.h (no compute calls)."""

import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "streamindex_b200.h")).read()
    return sorted(set(re.findall(r"SI_API\s+[\w\s\*]+?\b(si_\w+)\s*\(", src)))


def test_header_and_binding_agree():
    from streamindex_b200 import _lib

    assert _declared() == sorted(_lib.SIGNATURES), "ctypes signatures out of sync with the header"


def test_library_exports_every_symbol():
    from streamindex_b200 import _lib

    lib = _lib.load()
    for name in _declared():
        assert hasattr(lib, name), name
    assert lib.si_abi_version() == 1


def test_errors_are_reported_without_gpu():
    from streamindex_b200 import _lib

    lib = _lib.load()
    rc = lib.si_indexer_topk(None, None, None, 0, 0, 1, 8, 8, 48, 128, 4, 4, None, None, None, None, 0, None)
    assert rc == -1
    msg = lib.si_last_error().decode()
    assert "null" in msg or "H_I" in msg
    rc = lib.si_indexer_topk(None, None, None, 0, 0, 1, 8, 8, 64, 128, 0, 4, None, None, None, None, 0, None)
    assert rc == -1 and "top_k" in lib.si_last_error().decode()


def test_attention_argument_checks_without_gpu():
    """Shape limits of si_sparse_attn_fwd are checked before any device work:
    D must be a multiple of 8 up to 896 (Q lives in 14 TMEM atom slots) and Dv a
    multiple of 64 no larger than D."""
    import ctypes
    from streamindex_b200 import _lib

    lib = _lib.load()
    dummy = ctypes.c_void_p(256)  # never dereferenced: the checks fail first

    def call(D, Dv, H=64, K=8):
        return lib.si_sparse_attn_fwd(dummy, dummy, ctypes.cast(dummy, ctypes.POINTER(ctypes.c_float)),
                                      ctypes.cast(dummy, ctypes.POINTER(ctypes.c_int32)), 1, 4, H, D, 16, K, Dv,
                                      0.1, dummy, None, dummy, 256, None)

    assert call(960, 512) == -1 and "D must be" in lib.si_last_error().decode()
    assert call(900, 512) == -1 and "D must be" in lib.si_last_error().decode()
    assert call(576, 640) == -1 and "Dv" in lib.si_last_error().decode()
    assert call(576, 96) == -1 and "Dv" in lib.si_last_error().decode()
