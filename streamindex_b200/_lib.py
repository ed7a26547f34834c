"""ctypes binding of the in-tree C-ABI library (``include/streamindex_b200.h``).

The library is the only compute path: if it is missing or fails to load,
every public op raises; there is no CPU or PyTorch fallback.
"""

from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

_lock = threading.Lock()
_lib = None

c_int, c_size_t, c_void_p, c_char_p, c_float = ctypes.c_int, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_float

# name -> (restype, argtypes); mirrors include/streamindex_b200.h
SIGNATURES = {
    "si_abi_version": (c_int, []),
    "si_last_error": (c_char_p, []),
    "si_read_status": (c_int, [c_void_p, ctypes.POINTER(c_int), c_void_p]),
    "si_selftest_wait_timeout": (c_int, [c_void_p, ctypes.c_ulonglong, c_void_p]),
    "si_indexer_topk_ws_bytes": (c_size_t, [c_int] * 6),
    "si_indexer_topk": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "si_indexer_topk_ex": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                   c_int, c_int, c_void_p, ctypes.c_longlong, ctypes.c_uint, c_void_p, c_void_p,
                                   c_void_p, c_size_t, c_void_p]),
    "si_indexer_topk_strided": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                        c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p,
                                        ctypes.c_longlong, ctypes.c_uint, c_void_p, c_void_p, c_void_p, c_size_t,
                                        c_void_p]),
    "si_sparse_attn_fwd_strided": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p,
                                           c_int, c_int, c_int, c_int, c_int, c_int, c_float, c_int, c_void_p,
                                           c_void_p, c_void_p, c_size_t, c_void_p]),
    "si_topk_row_sort": (c_int, [c_void_p, c_void_p, ctypes.c_longlong, c_int, c_void_p]),
    "si_indexer_topk_noalloc_max_ws_bytes": (c_size_t, []),
    "si_indexer_topk_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                        c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p]),
    "si_indexer_topk_noalloc_read_status": (c_int, [ctypes.POINTER(c_int), c_void_p]),
    "si_sparse_attn_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int,
                                   c_int, c_float, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "si_sparse_attn_fwd_kv2": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_int, c_int,
                                       c_int, c_int, c_int, c_int, c_float, c_void_p, c_void_p, c_void_p, c_size_t,
                                       c_void_p]),
    "si_csa_sparse_attn_fwd": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_int, c_int,
                                       ctypes.c_longlong, c_int, c_int, c_int, c_int, c_int, c_float, c_void_p,
                                       c_void_p, c_void_p, c_size_t, c_void_p]),
    "si_fp8_kv_row_bytes": (c_int, [c_int, c_int]),
    "si_kv_quant_fp8": (c_int, [c_void_p, ctypes.c_longlong, c_int, c_int, c_void_p, c_void_p]),
    "si_sparse_attn_fwd_fp8kv": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, c_void_p,
                                         c_int, c_int, c_int, c_int, c_int, c_int, c_float, c_void_p, c_void_p,
                                         c_void_p, c_size_t, c_void_p]),
    "si_sparse_attn_fwd_ex": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_int, c_int,
                                      c_int, c_int, c_int, c_int, c_float, c_int, c_void_p, c_void_p, c_void_p,
                                      c_size_t, c_void_p]),
    "si_sparse_attn_bwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                                   c_int, c_int, c_int, c_int, c_int, c_int, c_float, c_void_p, c_void_p, c_void_p,
                                   c_void_p]),
    "si_scores_topk_ws_bytes": (c_size_t, [c_int, c_int, c_int]),
    "si_scores_topk": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_size_t,
                               c_void_p]),
    "si_scores_topk_mask": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                    c_void_p, c_size_t, c_void_p]),
    "si_csa_build_idx": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "si_csa_build_idx_ex": (c_int, [c_void_p, c_int, c_int, ctypes.c_longlong, c_int, c_int, c_int, c_void_p,
                                    c_void_p]),
    "si_hca_build_idx": (c_int, [c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "si_token_compressor": (c_int, [c_void_p] * 6 + [c_int] * 6 + [c_void_p, c_void_p]),
    "si_mean_pool": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "si_indexer_score": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                 c_void_p, c_void_p, c_size_t, c_void_p]),
}


def lib_path() -> str:
    return _build.LIB


def load(build_if_missing: bool = True):
    """Load (building first if needed and allowed) and return the ctypes library."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = lib_path()
        if not os.path.exists(path):
            if not build_if_missing or os.environ.get("STREAMINDEX_NO_BUILD") == "1":
                raise RuntimeError(f"StreamIndex-B200 library not built: {path} (run python -m streamindex_b200.build)")
            _build.build()
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


class SIError(RuntimeError):
    pass


def check(rc: int):
    if rc != 0:
        raise SIError(load().si_last_error().decode(errors="replace"))


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def strides_arg(t, dims, align_elems: int = 8):
    """ctypes ``long long[len(dims)]`` of ``t``'s element strides over ``dims``
    when ``t`` can be read in place (last dim contiguous, those strides
    non-negative multiples of ``align_elems``, 16-byte aligned base), else None."""
    if t.stride(-1) != 1 or t.data_ptr() % 16:
        return None
    st = [t.stride(d) for d in dims]
    if any(x < 0 or x % align_elems for x in st):
        return None
    return (ctypes.c_longlong * len(st))(*st)


def stream_handle(device) -> int:
    import torch

    return torch.cuda.current_stream(device).cuda_stream


def read_status(ws, device) -> int:
    v = c_int(0)
    check(load().si_read_status(ws.data_ptr(), ctypes.byref(v), stream_handle(device)))
    return v.value


def maybe_check_status(ws, device, what: str):
    """With STREAMINDEX_CHECK=1, synchronise and raise if a kernel wait timed out."""
    if os.environ.get("STREAMINDEX_CHECK") == "1":
        st = read_status(ws, device)
        if st != 0:
            raise SIError(f"{what}: device status {st} (a bounded in-kernel wait timed out)")
