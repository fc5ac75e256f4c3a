"""ctypes binding of the C ABI declared in ``include/fa_b200.h``.

The shared library ``_lib/libfa_b200.so`` is built in-tree by ``build.py``.
There is no fallback: if the library is missing or fails to load, every call
raises ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import os
import threading

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libfa_b200.so")
_lock = threading.Lock()
_lib = None

FA_OK = 0
FA_ERR_UNSUPPORTED_HEAD_DIM = 1
FA_ERR_BAD_SHAPE = 2
FA_ERR_MISALIGNED = 3
FA_ERR_LAUNCH = 4
FA_ERR_TENSOR_MAP = 5
FA_ERR_DRIVER = 6
FA_ERR_DEVICE_TIMEOUT = 7
FA_ERR_NO_DEVICE = 8
FA_ERR_SCRATCH_LIMIT = 9
FA_ERR_OUT_OF_MEMORY = 10
FA_ERR_CUDA = 11

_p = ctypes.c_void_p
_i = ctypes.c_int
_f = ctypes.c_float
_s = ctypes.POINTER(ctypes.c_int64)

# name -> (restype, argtypes), in the order of include/fa_b200.h
SIGNATURES = {
    "fa_fwd": (_i, [_p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _s, _s, _s, _s, _f, _i, _i, _i, _p]),
    "fa_bwd_delta": (_i, [_p, _p, _p, _i, _i, _i, _i, _s, _s, _p]),
    "fa_bwd_dq": (_i, [_p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _i,
                       _s, _s, _s, _s, _s, _f, _i, _i, _i, _i, _p]),
    "fa_bwd_dkdv": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _i,
                         _s, _s, _s, _s, _s, _s, _f, _i, _i, _i, _i, _p]),
    "fa_merge_partial": (_i, [_p, _p, _p, _p, _i, _i, _i, _i, _p]),
    "fa_bwd_preprocess": (_i, [_p, _p, _p, _p, _i, _i, _i, _i, _s, _s, _p]),
    "fa_bwd_fused": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _i,
                          _s, _s, _s, _s, _s, _s, _f, _i, _i, _i, _i, _p]),
    "fa_bwd_dq_convert": (_i, [_p, _p, _i, _i, _i, _i, _s, _p]),
}
# the bf16 twins take the same arguments
SIGNATURES.update({name + "_bf16": SIGNATURES[name] for name in list(SIGNATURES)})
SIGNATURES.update({
    "fa_fwd_varlen": (_i, [_p] * 7 + [_i] * 8 + [_f, _i, _i, _p]),
    "fa_bwd_varlen": (_i, [_p] * 13 + [_i] * 8 + [_f, _i, _i, _i, _p]),
})
SIGNATURES["fa_fwd_paged"] = (_i, [_p] * 8 + [_i] * 10 + [_f, _i, _i, _p])
SIGNATURES["fa_fwd_paged_split"] = (_i, [_p] * 8 + [_i] * 10 + [_f, _i, _i, _p])
SIGNATURES["fa_combine_splits"] = (_i, [_p] * 4 + [_i] * 4 + [_p])
SIGNATURES.update({name + "_bf16": SIGNATURES[name]
                   for name in ("fa_fwd_varlen", "fa_bwd_varlen", "fa_fwd_paged", "fa_fwd_paged_split",
                                "fa_combine_splits")})
SIGNATURES.update({
    "fa_fwd_vdim": (_i, [_p] * 5 + [_i] * 7 + [_s] * 4 + [_f, _i, _p]),
    "fa_bwd_vdim": (_i, [_p] * 11 + [_i] * 7 + [_s] * 8 + [_f, _i, _i, _p]),
})
SIGNATURES.update({
    "fa_mask_pack": (_i, [_p, _i, _i, _i, _i, _s, _p, _p, _p]),
    "fa_fwd_masked": (_i, [_p] * 5 + [_i] * 7 + [_s] * 4 + [_p, _s, _f, _i, _p]),
    "fa_bwd_masked": (_i, [_p] * 11 + [_i] * 7 + [_s] * 8 + [_p, _s, _p, _s, _f, _i, _i, _p]),
})
_u64 = ctypes.c_uint64
SIGNATURES.update({
    "fa_fwd_dropout": (_i, [_p] * 5 + [_i] * 7 + [_s] * 4 + [_f, _u64, _f, _i, _p]),
    "fa_bwd_dropout": (_i, [_p] * 10 + [_i] * 7 + [_s] * 8 + [_f, _u64, _f, _i, _p]),
})
SIGNATURES.update({name + "_bf16": SIGNATURES[name]
                   for name in ("fa_fwd_vdim", "fa_bwd_vdim", "fa_fwd_masked", "fa_bwd_masked",
                                "fa_fwd_dropout", "fa_bwd_dropout")})
SIGNATURES.update({
    "fa_bwd_fused_noalloc": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _i,
                                  _s, _s, _s, _s, _s, _s, _s, _s, _f, _i, _p]),
    "fa_device_status": (_i, [_i]),
    "fa_status_string": (ctypes.c_char_p, [_i]),
    "fa_version": (_i, []),
})


def library_path() -> str:
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    """Load (once) and return the native library; raise if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH):
                raise RuntimeError(
                    "the B200 CUDA library is not built: expected " + _LIB_PATH
                    + " (run `python -m triton_flash_attention_b200.build`)")
            handle = ctypes.CDLL(_LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


_entries: dict = {}


def entry(name: str, dtype) -> ctypes._CFuncPtr:
    """The entry point ``name`` for operands of ``dtype`` (torch.float16 or
    torch.bfloat16): the fp16 symbol or its ``_bf16`` twin (looked up once)."""
    key = (name, dtype)
    fn = _entries.get(key)
    if fn is None:
        import torch

        fn = getattr(lib(), name + "_bf16" if dtype == torch.bfloat16 else name)
        _entries[key] = fn
    return fn


def status_string(code: int) -> str:
    return lib().fa_status_string(int(code)).decode()


def check(rc: int, what: str) -> None:
    if rc != FA_OK:
        raise RuntimeError(f"{what} failed: {status_string(rc)} (code {rc})")


_Strides3 = ctypes.c_int64 * 3
_strides_cache: dict = {}


def strides3(t) -> ctypes.Array:
    """(batch, head, seq) element strides of a 4-D (B, H, N, D) tensor, as a
    ctypes array shared by every call with the same strides (the library
    only reads it)."""
    s = t.stride()
    if s[3] != 1:
        raise ValueError("the head dimension must be contiguous (unit stride)")
    key = s[:3]
    arr = _strides_cache.get(key)
    if arr is None:
        if len(_strides_cache) > 1024:
            _strides_cache.clear()
        arr = _strides_cache[key] = _Strides3(*key)
    return arr


def device_status(reset: bool = False) -> int:
    """The device status word (0 = healthy); synchronises the device."""
    return int(lib().fa_device_status(1 if reset else 0))
