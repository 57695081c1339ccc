"""ctypes binding of libfni8_b200.so (the C ABI declared in include/fni8_b200.h).

The library is loaded from this package's `_native/` directory, where
`fni8-serve_b200/build.py` writes it. There is no fallback: if the library is missing,
every op raises, so a silent CPU or eager-PyTorch path can never stand in for the
sm_100a kernels.
"""
from __future__ import annotations

import ctypes
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_native", "libfni8_b200.so")

# enum values of include/fni8_b200.h
OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_ALIGN, ERR_CUDA, ERR_WORKSPACE, ERR_DEVICE_TIMEOUT = range(7)
F16, BF16, F32, I32, I8 = range(5)
ACT_SILU, ACT_GELU_TANH = 0, 1
SCORE_SOFTMAX, SCORE_SIGMOID = 0, 1
PATH_AUTO, PATH_TILE, PATH_STREAM, PATH_FUSED, PATH_SPLITK = 0, 1, 2, 3, 4

_p = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_f = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/fni8_b200.h one to one
SIGNATURES: dict[str, tuple] = {
    "fni8_abi_version": (_i, []),
    "fni8_status_string": (ctypes.c_char_p, [_i]),
    "fni8_last_error_message": (ctypes.c_char_p, []),
    "fni8_device_status": (_i, [ctypes.POINTER(_i)]),
    "fni8_watchdog_selftest": (_i, [_i64, _i, _p]),
    "fni8_quantize_rows_i8": (_i, [_p, _i, _i64, _i64, _p, _p, _p]),
    "fni8_quantize_rows_i8_rows": (_i, [_p, _i, _i64, _i64, _p, _p, _p, _p]),
    "fni8_rmsnorm": (_i, [_p, _p, _p, _i, _i64, _i64, _f, _i, _p, _p, _p]),
    "fni8_rmsnorm_quant_i8": (_i, [_p, _p, _p, _i, _i64, _i64, _f, _i, _p, _p, _p, _p, _p]),
    "fni8_act_and_mul": (_i, [_p, _i, _i, _i64, _i64, _p, _p]),
    "fni8_act_and_mul_quant_i8": (_i, [_p, _i, _i, _i64, _i64, _p, _p, _p]),
    "fni8_act_and_mul_dual": (_i, [_p, _i, _i, _i64, _i64, _p, _p, _p, _p]),
    "fni8_act_and_mul_quant_i8_rows": (_i, [_p, _i, _i, _i64, _i64, _p, _p, _p, _p]),
    "fni8_gemm_w4a8": (_i, [_p, _p, _p, _p, _i64, _p, _p, _i, _i64, _i64, _i64, _p, _sz, _p]),
    "fni8_linear_w4a8": (_i, [_p, _i, _p, _p, _i64, _p, _p, _i64, _i64, _i64, _p, _p, _p, _sz, _p]),
    "fni8_gemm_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "fni8_workspace_init": (_i, [_p, _sz, _p]),
    "fni8_gemm_w8a8": (_i, [_p, _p, _p, _p, _p, _p, _p, _i, _i64, _i64, _i64, _p, _sz, _p]),
    "fni8_gemm_w8a8_ex": (_i, [_p, _p, _p, _p, _p, _p, _p, _i, _i64, _i64, _i64, _i, _p, _sz, _p]),
    "fni8_gemm_w8a8_i32": (_i, [_p, _p, _p, _i64, _i64, _i64, _i, _p, _sz, _p]),
    "fni8_gemm_w8a8_act": (_i, [_p, _p, _p, _p, _i, _p, _i, _i64, _i64, _i64, _p]),
    "fni8_grouped_gemm_w8a8_act": (_i, [_p, _p, _i64, _p, _p, _i64, _i64, _i64, _p, _p, _p, _i64, _i, _p, _i, _p]),
    "fni8_gemm_w8a8_peer_cols": (_i, [_p, _p, _p, _p, _p, _i, _i64, _i64, _i64, _p, _i, _i64, _i64, _p, _sz, _p, _sz,
                                      _p]),
    "fni8_gemm_w8a8_noalloc": (_i, [_p, _p, _p, _p, _p, _p, _p, _i, _i64, _i64, _i64, _p]),
    "fni8_linear_w8a8": (_i, [_p, _i, _p, _p, _p, _p, _i64, _i64, _i64, _p, _p, _p, _sz, _p]),
    "fni8_linear_w8a8_ex": (_i, [_p, _i, _p, _p, _p, _p, _i64, _i64, _i64, _p, _p, _i, _p, _sz, _p]),
    "fni8_moe_route": (_i, [_p, _i64, _i64, _i64, _i, _p, _i64, _i64, _i, _f, _i, _p, _p, _p]),
    "fni8_moe_plan_workspace_bytes": (_sz, [_i64, _i64]),
    "fni8_moe_plan": (_i, [_p, _i64, _i64, _p, _p, _p, _p, _p, _sz, _p]),
    "fni8_moe_gather_rows_i8": (_i, [_p, _p, _p, _i64, _i64, _i64, _p, _p, _p]),
    "fni8_moe_quantize_scatter_i8": (_i, [_p, _i, _i64, _i64, _p, _i64, _p, _p, _p]),
    "fni8_grouped_gemm_w8a8": (_i, [_p, _p, _i64, _p, _p, _i64, _i64, _i64, _p, _p, _p, _i64, _p, _i, _p]),
    "fni8_grouped_gemm_w8a8_scatter": (_i, [_p, _p, _i64, _p, _p, _i64, _i64, _i64, _p, _p, _p, _i64, _p, _p, _i64,
                                            _i64, _i, _p]),
    "fni8_moe_combine": (_i, [_p, _i, _p, _p, _i64, _i64, _i64, _p, _p]),
    "fni8_moe_experts_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _i64]),
    "fni8_moe_experts_w8a8": (_i, [_p, _i, _i64, _i64, _p, _p, _i64, _p, _p, _p, _p, _i64, _i64, _i, _p, _p, _sz,
                                   _p]),
    "fni8_ipc_alloc": (_i, [_sz, ctypes.POINTER(_p), _p]),
    "fni8_ipc_free": (_i, [_p]),
    "fni8_ipc_open": (_i, [_p, ctypes.POINTER(_p)]),
    "fni8_ipc_close": (_i, [_p]),
    "fni8_peer_barrier": (_i, [_p, _i64, _i64, _p, _p, _i64, _p, _i64, _p]),
    "fni8_moe_map_ids": (_i, [_p, _i64, _p, _i64, _p, _p]),
    "fni8_ep_placement": (_i, [_p, _i64, _i64, _i64, _p, _p, _p, _p, _p]),
    "fni8_ep_dispatch_i8": (_i, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _i64, _i64, _p]),
    "fni8_ep_return": (_i, [_p, _i, _p, _i64, _p, _i64, _i64, _p, _i64, _p]),
}


class Fni8Error(RuntimeError):
    """A libfni8_b200 entry point returned a non-zero status."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


_LIB: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """Load (once) and return the native library; raises if it has not been built."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build the sm_100a kernels with `python fni8-serve_b200/build.py` "
                "(fni8-serve_b200 has no CPU or eager fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def check(status: int, what: str) -> None:
    if status != OK:
        L = lib()
        msg = L.fni8_last_error_message().decode(errors="replace")
        kind = L.fni8_status_string(status).decode()
        raise Fni8Error(status, f"{what}: {kind}: {msg}")


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)
