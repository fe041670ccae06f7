"""ctypes binding of libflashbfp.so (declarations in include/flashbfp.h).

The library is loaded on first use. If it has not been built the call raises: there is
no CPU fallback for any op.
"""
from __future__ import annotations

import ctypes
import os
import re

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libflashbfp.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "flashbfp.h")

F32, BF16, F16 = 0, 1, 2
DTYPE_CODE = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}

_c_i64 = ctypes.c_int64
_c_int = ctypes.c_int
_vp = ctypes.c_void_p

_PROTOS = {
    "fbfp_abi_version": (_c_int, []),
    "fbfp_status_string": (ctypes.c_char_p, [_c_int]),
    "fbfp_last_error": (ctypes.c_char_p, []),
    "fbfp_dequant": (_c_int, [_vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_int, _vp, _c_i64, _vp]),
    "fbfp_scatter_outliers": (_c_int, [_vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_int, _vp,
                                       _c_i64, _vp]),
    "fbfp_outlier_tiles_scratch_bytes": (_c_i64, [_c_i64, _c_i64]),
    "fbfp_outlier_tiles_index_words": (_c_i64, [_c_i64, _c_i64]),
    "fbfp_outlier_tiles_build": (_c_int, [_vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                                          _vp, _vp, _vp, _vp]),
    "fbfp_gemv_workspace_bytes": (_c_i64, [_c_i64, _c_i64]),
    "fbfp_gemv_check": (_c_int, [_vp, _vp]),
    "fbfp_gemv": (_c_int, [_vp, _c_int, _c_i64, _c_i64, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64,
                           _c_i64, _vp, _vp, _vp, _c_int, _vp, _c_int, _c_i64, _vp, _vp]),
    "fbfp_gemv_noalloc": (_c_int, [_vp, _c_int, _c_i64, _c_i64, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64,
                                   _c_i64, _vp, _vp, _vp, _c_int, _vp, _c_int, _c_i64, _vp]),
    "fbfp_gemv_resident": (_c_int, [_vp, _c_int, _c_i64, _c_i64, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64,
                                    _c_i64, _vp, _vp, _vp, _c_int, _vp, _c_int, _c_i64, _vp, _vp]),
    "fbfp_gemv_allreduce": (_c_int, [_vp, _c_int, _c_i64, _c_i64, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64,
                                     _c_i64, _vp, _vp, _vp, _c_int, _vp, _c_int, _c_i64, _vp, _vp, _c_int,
                                     _vp]),
    "fbfp_stream_fence": (_c_int, [_vp]),
    "fbfp_records_bytes": (_c_i64, [_c_i64, _c_i64, _c_i64]),
    "fbfp_records_scratch_bytes": (_c_i64, [_c_i64, _c_i64]),
    "fbfp_records_build": (_c_int, [_vp, _vp, _vp, _c_i64, _c_i64, _vp, _vp, _c_i64, _vp, _vp, _vp, _vp]),
    "fbfp_gemv_records": (_c_int, [_vp, _c_i64, _c_i64, _vp, _c_i64, _c_i64, _c_i64, _c_i64,
                                   _vp, _c_int, _vp, _c_int, _c_i64, _vp, _vp, _c_int, _vp]),
    "fbfp_embed": (_c_int, [_vp, _c_i64, _vp, _c_i64, _c_i64, ctypes.c_float, _vp, _vp, _vp]),
    "fbfp_rmsnorm": (_c_int, [_vp, _c_i64, _vp, ctypes.c_float, _c_i64, _vp, _vp]),
    "fbfp_post_residual_norm": (_c_int, [_vp, _c_i64, _vp, _vp, _vp, ctypes.c_float, _c_i64, _vp, _vp]),
    "fbfp_qk_rope_cache": (_c_int, [_vp, _c_i64, _c_i64, _c_i64, _c_i64, _vp, _vp, ctypes.c_float, _vp, _vp,
                                    _vp, _c_i64, _vp, _vp, _vp, _vp, _vp]),
    "fbfp_decode_attention": (_c_int, [_vp, _c_i64, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_i64, _vp, _c_i64,
                                       ctypes.c_float, _vp, _vp]),
    "fbfp_geglu": (_c_int, [_vp, _c_i64, _c_i64, _vp, _vp]),
    "fbfp_decode_attention_step_scratch_bytes": (_c_i64, [_c_i64, _c_i64, _c_i64, _c_i64]),
    "fbfp_decode_attention_step": (_c_int, [_vp, _c_i64, _c_i64, _c_i64, _c_i64, _vp, _vp, ctypes.c_float,
                                            _vp, _vp, _vp, _c_i64, _vp, _vp, _c_i64, _c_i64, ctypes.c_float,
                                            _vp, _vp, _vp, _vp]),
    "fbfp_advance_positions": (_c_int, [_vp, _c_i64, _vp]),
    "fbfp_advance_position": (_c_int, [_vp, _c_i64, _vp]),
    "fbfp_allreduce_ipc_handle_bytes": (_c_i64, []),
    "fbfp_allreduce_create": (_c_int, [_c_int, _c_int, _c_i64, _vp, _vp]),
    "fbfp_allreduce_open_peer": (_c_int, [_vp, _c_int, _vp]),
    "fbfp_allreduce_sum_f32": (_c_int, [_vp, _vp, _c_i64, _vp]),
    "fbfp_allreduce_set_timeout": (_c_int, [_vp, _c_i64]),
    "fbfp_allreduce_check": (_c_int, [_vp, _vp]),
    "fbfp_allreduce_destroy": (_c_int, [_vp]),
    "fbfp_gemm_prefill": (_c_int, [_vp, _c_int, _c_i64, _c_i64, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64,
                                   _c_i64, _vp, _vp, _vp, _c_int, _vp, _c_int, _c_i64, _vp, _vp]),
    "fbfp_gemm_expanded_scratch_bytes": (_c_i64, [_c_i64, _c_i64]),
    "fbfp_gemm_expanded": (_c_int, [_vp, _c_i64, _c_i64, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _vp, _vp,
                                    _vp, _c_i64, _vp, _vp, _c_i64, _vp, _vp, _c_int, _c_i64, _vp, _c_i64,
                                    _vp]),
    "fbfp_expand_x15": (_c_int, [_vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _vp, _vp, _vp, _c_i64, _vp, _vp,
                                 _c_i64, _vp, _c_i64, _vp]),
    "fbfp_compress_scratch_bytes": (_c_i64, [_c_i64, _c_i64, _c_i64, _c_i64]),
    "fbfp_compress_threshold": (_c_int, [_vp, _c_int, _c_i64, _c_i64, _c_i64, _vp, _vp, _vp]),
    "fbfp_compress_pack": (_c_int, [_vp, _c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _vp, _vp,
                                    _vp, _vp, _vp, _vp, _vp]),
    "fbfp_compress_outliers": (_c_int, [_vp, _c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _vp,
                                        _vp, _vp, _vp, _vp, _vp]),
}

_lib = None


class FlashBFPError(RuntimeError):
    pass


def lib() -> ctypes.CDLL:
    """The loaded library (loads it on first call; raises if it is not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FlashBFPError(
                f"{LIB_PATH} is missing: build it with `python -m flashbfp_b200.build` "
                "(FlashBFP-B200 has no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _PROTOS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def header_symbols() -> list[str]:
    """Entry points declared in include/flashbfp.h."""
    with open(HEADER) as f:
        text = f.read()
    return sorted(set(re.findall(r"\b(fbfp_[a-z0-9_]+)\s*\(", text)))


def check(status: int, what: str) -> None:
    if status == 0:
        return
    L = lib()
    msg = f"{what}: {L.fbfp_status_string(status).decode()}: {L.fbfp_last_error().decode()}"
    if status in (1, 4):
        raise ValueError(msg)
    if status == 2:
        raise NotImplementedError(msg)
    raise FlashBFPError(msg)


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_ptr(device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def require_cuda(t: torch.Tensor, what: str) -> None:
    if not (isinstance(t, torch.Tensor) and t.is_cuda):
        raise RuntimeError(f"{what} must be a CUDA tensor: FlashBFP-B200 runs only on the GPU "
                           "(no CPU fallback)")


def dtype_code(dt: torch.dtype, what: str) -> int:
    if dt not in DTYPE_CODE:
        raise NotImplementedError(f"{what}: unsupported dtype {dt}")
    return DTYPE_CODE[dt]
