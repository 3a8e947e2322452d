"""ctypes binding of the sm_100a C ABI (``include/sparse_ai_b200.h``).

The shared library ``libsparse_ai_b200.so`` sits next to this file (built in-tree by
``sparse-ai_b200/build.py``).  There is no fallback: if the library is missing or fails to
load, every operator raises.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libsparse_ai_b200.so"

SA_OK, SA_EINVAL, SA_EUNSUPPORTED, SA_ELAUNCH, SA_EWORKSPACE = 0, -1, -2, -3, -4
SA_F32, SA_F16, SA_BF16, SA_I32, SA_I64 = 0, 1, 2, 3, 4

_FLOAT_CODES = {torch.float32: SA_F32, torch.float16: SA_F16, torch.bfloat16: SA_BF16}
_INT_CODES = {torch.int32: SA_I32, torch.int64: SA_I64}

_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_vp = ctypes.c_void_p
_f32 = ctypes.c_float
_p64 = ctypes.POINTER(ctypes.c_int64)

# name -> (restype, argtypes), in the order of include/sparse_ai_b200.h
_SIGNATURES = {
    "sa_last_error": (ctypes.c_char_p, []),
    "sa_abi_version": (_i32, []),
    "sa_read_device_status": (_i32, [_i32, ctypes.POINTER(ctypes.c_uint)]),
    "sa_release_thread_resources": (_i32, []),
    "sa_paged_kv_append": (_i32, [_i32, _i64, _i64, _i64, _i64, _i64, _vp, _p64, _vp, _p64, _vp,
                                   _p64, _i64, _vp, _vp, _p64, _vp, _p64, _vp, _i32, _p64, _i64,
                                   _i64, _vp, _i32, _p64, _vp]),
    "sa_ternary_quantize_pack": (_i32, [_i32, _i64, _i64, _vp, _i64, _vp, _vp, _vp]),
    "sa_ternary_dequantize": (_i32, [_i32, _i64, _i64, _vp, _vp, _vp, _i64, _vp]),
    "sa_build_block_lists_from_assignments": (_i32, [_vp, _i32, _p64, _i64, _i64, _i64, _i64,
                                                      _i64, _i64, _i64, _vp, _i64, _i32, _i32,
                                                      _i64, _vp, _vp, _i64, _vp, _vp]),
    "sa_build_block_lists": (_i32, [_vp, _i32, _p64, _i64, _i64, _i64, _i64, _vp, _i64, _i32,
                                    _i32, _i32, _i64, _vp, _i64, _vp, _vp]),
    "sa_build_transposed_block_lists": (_i32, [_vp, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _vp,
                                               _vp, _vp]),
    "sa_block_list_attention_fwd": (_i32, [_i32, _i64, _i64, _i64, _i64, _i64, _i64,
                                           _vp, _p64, _vp, _p64, _vp, _p64, _vp, _p64, _vp,
                                           _vp, _i64, _vp, _vp, _i32, _p64, _i32, _f32,
                                           _vp, _i64, _vp]),
    "sa_block_list_attention_fwd_workspace_bytes": (_i64, [_i64, _i64, _i64, _i64, _i64]),
    "sa_block_list_attention_bwd_workspace_bytes": (_i64, [_i64, _i64, _i64, _i64, _i64, _i64]),
    "sa_block_list_attention_bwd": (_i32, [_i32, _i64, _i64, _i64, _i64, _i64, _i64,
                                           _vp, _p64, _vp, _p64, _vp, _p64, _vp, _p64, _vp, _p64,
                                           _vp, _vp, _i64, _vp, _vp, _i32, _p64, _i32, _f32,
                                           _vp, _p64, _vp, _p64, _vp, _p64, _vp, _vp, _i64, _vp]),
    "sa_block_list_attention_bwd_phase": (_i32, [_i32, _i32, _i64, _i64, _i64, _i64, _i64, _i64,
                                                 _vp, _p64, _vp, _p64, _vp, _p64, _vp, _p64, _vp,
                                                 _p64, _vp, _vp, _i64, _vp, _vp, _i32, _p64, _i32,
                                                 _f32, _vp, _p64, _vp, _p64, _vp, _p64, _vp, _vp,
                                                 _i64, _vp]),
    "sa_ultrametric_decode_workspace_bytes": (_i64, [_i64, _i64, _i64, _i64, _i64]),
    "sa_ultrametric_decode": (_i32, [_i32, _i64, _i64, _i64, _i64, _i64, _i64,
                                     _vp, _p64, _vp, _p64, _vp, _p64, _vp, _p64, _i64, _vp,
                                     _vp, _i32, _p64, _vp, _i32, _p64, _i64, _i64, _i64, _i32,
                                     _vp, _p64, _vp, _i64, _vp]),
    "sa_ultrametric_decode_noalloc": (_i32, [_i32, _i64, _i64, _i64, _i64, _i64, _i64,
                                             _vp, _p64, _vp, _p64, _vp, _p64, _vp, _p64, _i64,
                                             _vp, _vp, _i32, _p64, _vp, _i32, _p64, _i64, _i64,
                                             _i64, _i32, _vp, _p64, _vp]),
    "sa_block_list_attention_fwd_accumulate": (_i32, [_i32, _i64, _i64, _i64, _i64, _i64, _i64,
                                                      _vp, _p64, _vp, _p64, _vp, _p64, _vp, _p64,
                                                      _vp, _vp, _i64, _vp, _i32, _f32, _vp, _i64,
                                                      _vp]),
    "sa_attention_lse_merge": (_i32, [_i32, _i64, _i64, _i64, _i64, _vp, _p64, _vp, _vp, _vp,
                                      _i32, _vp, _p64, _vp]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """Load (once) and return the library; raises RuntimeError when it is missing."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"the sm_100a library {LIB_PATH.name} is missing; build it with "
                f"`python sparse-ai_b200/build.py` (there is no CPU or Triton fallback)")
        handle = ctypes.CDLL(os.fspath(LIB_PATH))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def check(rc: int, what: str) -> None:
    if rc == SA_OK:
        return
    msg = lib().sa_last_error().decode(errors="replace")
    if rc == SA_EINVAL:
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what} failed ({rc}): {msg}")


def strides(t: torch.Tensor, ndim: int | None = None):
    st = t.stride()
    if ndim is not None and len(st) != ndim:
        raise ValueError(f"expected a {ndim}-d tensor, got shape {tuple(t.shape)}")
    return (ctypes.c_int64 * len(st))(*st)


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def float_code(dtype: torch.dtype) -> int:
    if dtype not in _FLOAT_CODES:
        raise ValueError(f"unsupported dtype {dtype}; expected float32, float16 or bfloat16")
    return _FLOAT_CODES[dtype]


def int_code(dtype: torch.dtype) -> int:
    if dtype not in _INT_CODES:
        raise ValueError(f"unsupported index dtype {dtype}; expected int32 or int64")
    return _INT_CODES[dtype]


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(name: str, *tensors) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(f"{name} runs only on CUDA (sm_100a) tensors; got a tensor on "
                               f"{t.device}. There is no CPU fallback.")


def read_device_status(reset: bool = True) -> int:
    v = ctypes.c_uint(0)
    check(lib().sa_read_device_status(int(reset), ctypes.byref(v)), "sa_read_device_status")
    return int(v.value)
