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
