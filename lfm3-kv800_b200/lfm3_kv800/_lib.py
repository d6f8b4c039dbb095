"""ctypes binding of libkv800_b200.so (the C ABI in include/kv800_b200.h).  No torch types cross the boundary: the
callers in kv800.py pass data pointers, sizes and the current CUDA stream handle.  A missing library raises
ImportError; nothing here falls back to another implementation."""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
# LFM3KV_LIB names another build of the same library (e.g. an instrumented or experimental build); the default is the
# in-tree build that build.py writes
LIB_PATH = os.environ.get("LFM3KV_LIB") or os.path.join(HERE, "_lib", "libkv800_b200.so")

OK, ERR_ARG, ERR_RANGE, ERR_CUDA, ERR_DEVICE = 0, 1, 2, 3, 4
_p, _i64, _int, _f = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float


class Paged(ctypes.Structure):
    """struct kv800_paged (include/kv800_b200.h)."""
    _fields_ = [("qpool", _p), ("qpool_bytes", _i64), ("boff", _p), ("boff_stride", _i64),
                ("epool", _p), ("epool_elems", _i64), ("eoff", _p), ("eoff_stride", _i64),
                ("ebs", _i64), ("e_hs", _i64), ("e_ts", _i64), ("e_v", _i64),
                ("sk", _p), ("sv", _p), ("sk_elems", _i64), ("sv_elems", _i64),
                ("skoff", _p), ("svoff", _p), ("N", _p), ("NQ", _p),
                ("nqmax", _i64), ("win", _i64), ("nsink", _i64)]


SIGNATURES = {
    "kv800_abi_version": (_int, []),
    "kv800_last_error": (ctypes.c_char_p, []),
    "kv800_constants": (_int, [_p, _p, _p, _p, _p]),
    "kv800_quantize_blocks": (_int, [_p, _p, _i64, _p, _p]),
    "kv800_dequantize_blocks": (_int, [_p, _i64, _p, _p, _p]),
    "kv800_fake_quant_k": (_int, [_p, _i64, _i64, _p, _p]),
    "kv800_fake_quant_v": (_int, [_p, _i64, _p, _p]),
    "kv800_write_slots": (_int, [_p, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, _i64, _p, _p]),
    "kv800_flush_step_workspace_size": (_i64, [_i64]),
    "kv800_flush_step": (_int, [_p, _i64, _i64, _i64, _i64, _i64, _p, _i64, _p, _i64, _i64, _i64, _p, _i64, _p, _p,
                                _i64, _i64, _p, _i64, _p, _p]),
    "kv800_write_sinks": (_int, [_p, _i64, _i64, _i64, _p, _i64, _p, _i64, _i64, _i64, _p, _i64, _p, _p, _p, _p, _p,
                                 _i64, _i64, _p, _p]),
    "kv800_decode_tables": (_int, [_p, _i64, _p, _i64, _i64, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _p,
                                   _p, _i64, _i64, _i64, _p, _p, _i64, _i64, _i64, _p, _p]),
    "kv800_prefill_kv": (_int, [_p, _i64, _i64, _i64, _p, _i64, _i64, _p, _p, _i64, _p, _i64, _i64, _i64, _i64, _i64,
                                _p, _i64, _i64, _i64, _p, _p, _i64, _p, _p, _i64, _p, _p, _p, _p]),
    "kv800_flush": (_int, [_p, _i64, _p, _i64, _i64, _i64, _i64, _i64, _p, _i64, _p, _i64, _p, _p, _i64, _i64, _p,
                           _p]),
    "kv800_write_exact": (_int, [_p, _i64, _p, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _i64, _i64, _p, _p]),
    "kv800_decode_workspace_size": (_i64, [_i64, _i64, _i64, _i64]),
    "kv800_decode": (_int, [ctypes.POINTER(Paged), _p, _p, _p, _i64, _i64, _i64, _p, _p, _i64, _p]),
    "kv800_decode_timed": (_int, [ctypes.POINTER(Paged), _p, _p, _p, _i64, _i64, _i64, _p, _p, _i64, _p,
                                  ctypes.POINTER(ctypes.c_float)]),
    "kv800_decode_noalloc": (_int, [ctypes.POINTER(Paged), _p, _p, _p, _i64, _i64, _i64, _p, _p]),
    "kv800_decode_noalloc_status": (_int, [_p, _p]),
    "kv800_qdecode": (_int, [_p, _p, _i64, _p, _i64, _p, _p, _p, _i64, _p, _p, _p, _i64, _i64, _i64, _i64, _f, _p,
                             _p]),
    "kv800_xdecode": (_int, [_p, ctypes.POINTER(Paged), _p, _p, _i64, _p, _p, _p, _i64, _i64, _f, _p, _p]),
    "kv800_combine": (_int, [_p, _p, _p, _i64, _i64, _p, _p]),
    "kv800_check_status": (_int, [_p, _p, _p]),
}

_LIB = None


def lib():
    """The loaded library (loaded once).  Raises ImportError when it has not been built."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"lfm3_kv800: CUDA library {LIB_PATH} is missing; build it with "
                              f"`python lfm3-kv800_b200/build.py` (nvcc 12.9, sm_100a)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        if L.kv800_abi_version() != 1:
            raise ImportError("lfm3_kv800: libkv800_b200.so ABI version mismatch")
        _LIB = L
    return _LIB


class KV800Error(RuntimeError):
    """A C-ABI call returned an error status."""

    def __init__(self, fn, code, msg):
        super().__init__(f"{fn} failed (status {code}): {msg}")
        self.code = code


def call(name, *args):
    L = lib()
    rc = getattr(L, name)(*args)
    if rc != OK:
        msg = (L.kv800_last_error() or b"").decode(errors="replace")
        if rc == ERR_ARG:
            raise ValueError(f"{name}: {msg}")
        raise KV800Error(name, rc, msg)
    return rc
