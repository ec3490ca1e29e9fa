"""ctypes binding of libmarlin_q4.so (the C ABI in include/marlin_q4.h).

The library is built in-tree by marlin-mlx_b200/build.py.  There is no fallback: if the shared
library is missing, importing this module raises.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libmarlin_q4.so"

OK = 0
ERR_ARG, ERR_SHAPE, ERR_ALIGN, ERR_UNSUPPORTED, ERR_CUDA, ERR_WORKSPACE = -1, -2, -3, -4, -5, -6
BF16, F32 = 0, 1
PATH_I8MMA, PATH_BF16MMA = 0, 2
STEP_FUSED, STEP_LAYERS = 0, 1

# Every symbol include/marlin_q4.h declares, with its ctypes signature (restype, argtypes).
_vp, _i64, _i32, _f32, _sz, _u64 = (ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_float,
                                     ctypes.c_size_t, ctypes.c_uint64)


class Q4Tensor(ctypes.Structure):
    """marlin_q4_tensor"""
    _fields_ = [("weight", _vp), ("scales", _vp), ("biases", _vp), ("n", _i64), ("k", _i64),
                ("group_size", _i32), ("bits", _i32)]


class Q4Layer(ctypes.Structure):
    """marlin_q4_layer"""
    _fields_ = [("post_attn_norm", _vp), ("gate_proj", Q4Tensor), ("up_proj", Q4Tensor),
                ("down_proj", Q4Tensor)]


_PT, _PL = ctypes.POINTER(Q4Tensor), ctypes.POINTER(Q4Layer)

SIGNATURES = {
    "marlin_q4_version": (ctypes.c_char_p, []),
    "marlin_q4_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "marlin_q4_last_cuda_error": (ctypes.c_int, []),
    "marlin_q4_device_error": (ctypes.c_int, [ctypes.c_int]),
    "marlin_q4_set_pdl": (None, [ctypes.c_int]),
    "marlin_q4_set_wait_limit_cycles": (None, [_u64]),
    "marlin_q4_set_decode_path": (ctypes.c_int, [ctypes.c_int]),
    "marlin_q4_set_step_kernels": (ctypes.c_int, [ctypes.c_int]),
    "marlin_q4_decode_step_kernels": (ctypes.c_int, [_i64, _i64, _i64, _i32]),
    "marlin_q4_quantize": (ctypes.c_int, [_vp, _i64, _i64, _i32, _i32, _vp, _vp, _vp, _vp]),
    "marlin_q4_matmul": (ctypes.c_int, [_vp, _i32, _i64, _PT, _vp, _vp]),
    "marlin_q4_matmul_f32": (ctypes.c_int, [_vp, _i32, _i64, _PT, _vp, _vp]),
    "marlin_q4_cast_bf16": (ctypes.c_int, [_vp, _i64, _vp, _vp]),
    "marlin_q4_rms_norm": (ctypes.c_int, [_vp, _i32, _vp, _i64, _i64, _f32, _vp, _vp]),
    "marlin_q4_gate_up_swiglu": (ctypes.c_int, [_vp, _i32, _i64, _vp, _f32, _PT, _PT, _vp, _vp]),
    "marlin_q4_matmul_residual": (ctypes.c_int, [_vp, _i32, _i64, _PT, _vp, _i32, _vp, _vp]),
    "marlin_q4_mlp": (ctypes.c_int, [_vp, _i32, _i64, _PT, _PT, _PT, _vp, _vp, _sz, _vp]),
    "marlin_q4_mlp_workspace_size": (_sz, [_i64, _i64, _i32]),
    "marlin_q4_residual_add": (ctypes.c_int, [_vp, _i32, _vp, _i64, _vp, _vp]),
    "marlin_q4_lm_head_argmax": (ctypes.c_int, [_vp, _i32, _i64, _vp, _f32, _PT, _i64, _vp, _vp, _vp,
                                                _vp, _sz, _vp]),
    "marlin_q4_lm_head_workspace_size": (_sz, [_i64]),
    "marlin_q4_lm_head_argmax_static": (ctypes.c_int, [_vp, _i32, _i64, _vp, _f32, _PT, _i64, _vp, _vp, _vp,
                                                       _vp]),
    "marlin_q4_decode_keys": (ctypes.c_int, [_vp, _i64, _vp, _vp, _vp]),
    "marlin_q4_decode_step": (ctypes.c_int, [_vp, _i64, _i64, _i32, _PL, _vp, _f32, _PT, _vp, _vp, _vp,
                                             _vp, _sz, _vp]),
    "marlin_q4_decode_step_workspace_size": (_sz, [_i64, _i64, _i64]),
    "marlin_q4_tp_decode_step": (ctypes.c_int, [_vp, _i64, _i64, _i32, _vp, _vp, _f32, _vp, _i64, _vp, _vp, _vp, _i32,
                                                _i32, _vp, _vp, _sz, _vp]),
    "marlin_q4_tp_exchange_size": (_sz, [_i64, _i64, _i32]),
    "marlin_q4_device_alloc": (ctypes.c_int, [_sz, ctypes.POINTER(ctypes.c_void_p)]),
    "marlin_q4_device_free": (ctypes.c_int, [_vp]),
    "marlin_q4_ipc_get_handle": (ctypes.c_int, [_vp, _vp]),
    "marlin_q4_ipc_open_handle": (ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_void_p)]),
    "marlin_q4_ipc_close_handle": (ctypes.c_int, [_vp]),
    "marlin_q4_embed": (ctypes.c_int, [_vp, _i64, _PT, _vp, _vp]),
    "marlin_q4_synth_bf16": (ctypes.c_int, [_vp, _i64, _u64, _f32, _f32, _vp]),
}

_lib = None


def load(path: Path | None = None) -> ctypes.CDLL:
    """Load the product library (once).  Raises if it has not been built."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path or LIB_PATH)
    if not p.exists():
        raise ImportError(f"{p} is missing: build it with `python marlin-mlx_b200/build.py` "
                          "(there is no non-CUDA fallback)")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


class MarlinQ4Error(RuntimeError):
    def __init__(self, status: int, where: str):
        lib = load()
        msg = lib.marlin_q4_status_string(status).decode()
        if status == ERR_CUDA:
            msg += f" (cudaError {lib.marlin_q4_last_cuda_error()})"
        super().__init__(f"{where}: {msg} [{status}]")
        self.status = status


def check(status: int, where: str) -> None:
    if status != OK:
        raise MarlinQ4Error(status, where)
