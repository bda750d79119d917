"""ctypes binding of the C ABI declared in include/vggt_sparse.h.

The shared library is built in-tree (``vggt_sparse.build``).  There is no
CPU or Python fallback: if the library is missing every operator raises
``ExtensionMissing``.
"""
import ctypes
import os

from .build import LIB_PATH

DTYPE_BF16, DTYPE_FP16 = 0, 1
SELECT_TOPK, SELECT_MASS = 0, 1
ATTN_AUTO, ATTN_MMA_SYNC, ATTN_TCGEN05 = 0, 1, 2
STATUS_BAD_INDEX, STATUS_BAD_COUNT, STATUS_TIMEOUT, STATUS_BAD_HEAD = 1, 2, 4, 8

# Every symbol the header declares, with its ctypes signature.
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
SIGNATURES = {
    "vggt_sparse_version": (_I, []),
    "vggt_sparse_last_error": (ctypes.c_char_p, []),
    "vggt_sparse_set_wait_limit_ns": (ctypes.c_uint64, [ctypes.c_uint64]),
    "vggt_sparse_set_wait_selftest": (_I, [_I]),
    "vggt_block_attention": (_I, [_P, _P, _P, _P, _P, _I, _I64, _I64, _I64, _I64, _I, _P, _P, _I,
                                  _P, _P, _I64, _I64, _I, _I, ctypes.c_float, _P, _P, _P, _I, _P]),
    "vggt_block_attention_ex": (_I, [_P, _P, _P, _P, _P, _I, _I64, _I64, _I64, _I64, _I, _P, _P,
                                     _I, _P, _P, _I64, _I64, _I, _I, ctypes.c_float, _P, _P, _P,
                                     _I, _P, _P, ctypes.c_size_t]),
    "vggt_block_attention_workspace_size": (ctypes.c_size_t, [_I64, _I64, _I64, _I, _I]),
    "vggt_token_sparse_attention": (_I, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I, _I,
                                         ctypes.c_float, _P, _P, _P]),
    "vggt_frame_qk_topk": (_I, [_P, _P, _P, _I64, _I64, _I64, _I64, _I, _I64, _I64, _P, _P]),
    "vggt_block_mask_assemble": (_I, [_P, _I64, _I64, _I64, _P, _P, _P, _P, _I64, _P, _P, _I64,
                                      _P, _P]),
    "vggt_history_update": (_I, [_P, _P, _I64, _I64, _I64, _P, _P, _P, _I64, _P]),
    "vggt_block_mask_estimate": (_I, [_P, _P, _I, _I64, _I64, _I64, _I, _P, _I64, _I, _I, _I, _I64,
                                      ctypes.c_double, ctypes.c_float, _P, _P, _P, _I64, _P, _P, _P,
                                      _P]),
    "vggt_block_select": (_I, [_P, _I64, _I64, _I, _I64, ctypes.c_double, _P, _I64, _P, _P]),
    "vggt_kv_push": (_I, [_P, _P, _P, _I, _I64, _I, _I, _P, _I, _I, _I64, _I, ctypes.c_uint32,
                          _I, _I, _P, _P]),
    "vggt_kv_push_flag_bytes": (_I64, [_I]),
    "vggt_qkv_workspace_size": (ctypes.c_size_t, [_I64, _I]),
    "vggt_qkv_project_pool": (_I, [_P, _P, _P, _I, _I64, _I, _I, _I, _P, _P, _P, _P,
                                   ctypes.c_float, _P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _P,
                                   _P, ctypes.c_size_t, _P, _P]),
    "vggt_block_select_pooled": (_I, [_P, _P, _I64, _P, _I64, _I64, _I64, _I, _I, _I64,
                                      ctypes.c_double, ctypes.c_float, _P, _I64, _P, _P, _P,
                                      _P]),
    "vggt_block_mask_estimate_noalloc": (_I, [_P, _P, _I, _I64, _I64, _I64, _I, _P, _I64, _I, _I,
                                              _I, _I64, ctypes.c_double, ctypes.c_float, _P, _I64,
                                              _P, _P, _P, _P]),
}


class ExtensionMissing(RuntimeError):
    """The compiled library is not present (build it; there is no fallback)."""


_LIB = None


def load(path=None):
    """Load (once) and return the ctypes handle of libvggt_sparse.so."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise ExtensionMissing(
            "libvggt_sparse.so not found at %s: build it with `python -m vggt_sparse.build` "
            "(no CPU fallback exists)" % p)
    lib = ctypes.CDLL(p)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _LIB = lib
    return lib


def last_error():
    return load().vggt_sparse_last_error().decode()


def set_wait_limit_ns(ns):
    """Limit (ns) of every pipeline wait in the tcgen05 attention kernels,
    process-wide, for launches enqueued afterwards; 0 restores the default
    (one second).  Returns the previous setting."""
    return int(load().vggt_sparse_set_wait_limit_ns(int(ns)))


def set_wait_selftest(enable):
    """While enabled, every tcgen05 attention launch waits on a barrier that
    nothing completes and takes the timeout path (tests of failure
    detection).  Returns the previous setting."""
    return int(load().vggt_sparse_set_wait_selftest(1 if enable else 0))


def check(rc):
    """Translate a C-ABI return code into a Python exception."""
    if rc == 0:
        return
    msg = last_error()
    if rc < 0:
        raise ValueError(msg)
    raise RuntimeError(msg or "CUDA error %d" % rc)
