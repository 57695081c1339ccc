"""ctypes view of the plain-C oracle (oracle/w8a8_ref.c) — TEST INFRASTRUCTURE ONLY.

Only tests/ use it: a second, independent restatement of the W8A8 integer path that the
torch oracle (w8a8_oracle.py) and the sm_100a kernels are checked against. `load()`
builds it with oracle/Makefile when the library is missing or older than its source.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "w8a8_ref.c")
LIB = os.path.join(HERE, "_build", "libw8a8_ref.so")
F16, BF16 = 0, 1
_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


def load():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(SRC):
            build()
        lib = ctypes.CDLL(LIB)
        i64, vp, i32 = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int
        lib.fni8o_to_f32.argtypes = [vp, i32, i64, vp]
        lib.fni8o_from_f32.argtypes = [vp, i32, i64, vp]
        lib.fni8o_quantize_weight_rows.argtypes = [vp, i64, i64, vp, vp]
        lib.fni8o_quantize_rows.argtypes = [vp, i32, i64, i64, vp, vp]
        lib.fni8o_gemm_i32.argtypes = [vp, vp, i64, i64, i64, vp]
        lib.fni8o_gemm_i32.restype = i32
        lib.fni8o_dequant.argtypes = [vp, vp, vp, vp, vp, i32, i64, i64, vp]
        lib.fni8o_linear_w8a8.argtypes = [vp, i32, i64, i64, vp, vp, i64, vp, vp, vp, vp, vp]
        lib.fni8o_linear_w8a8.restype = i32
        lib.fni8o_unpack_i4.argtypes = [vp, i64, i64, vp]
        lib.fni8o_dequant_weight_i4.argtypes = [vp, vp, i64, i64, i64, vp, vp]
        lib.fni8o_linear_w4a8.argtypes = [vp, i32, i64, i64, vp, vp, i64, i64, vp, vp, vp, vp, vp]
        lib.fni8o_moe_plan.argtypes = [vp, i64, ctypes.c_int32, vp, vp, vp, vp, vp]
        lib.fni8o_moe_plan.restype = i64
        lib.fni8o_moe_combine.argtypes = [vp, i32, vp, vp, i64, i64, i64, vp]
        _lib = lib
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def _half_bits(t: torch.Tensor) -> tuple[np.ndarray, int]:
    if t.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError(f"fp16 or bf16 expected, got {t.dtype}")
    return np.ascontiguousarray(t.contiguous().view(torch.int16).numpy()), (F16 if t.dtype == torch.float16 else BF16)


def _from_bits(b: np.ndarray, dtype: int) -> torch.Tensor:
    return torch.from_numpy(b).view(torch.float16 if dtype == F16 else torch.bfloat16)


def to_f32(t: torch.Tensor) -> torch.Tensor:
    b, dt = _half_bits(t)
    out = np.empty(b.shape, np.float32)
    load().fni8o_to_f32(_p(b), dt, b.size, _p(out))
    return torch.from_numpy(out)


def from_f32(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    x = np.ascontiguousarray(t.float().numpy())
    dt = F16 if dtype == torch.float16 else BF16
    out = np.empty(x.shape, np.int16)
    load().fni8o_from_f32(_p(x), dt, x.size, _p(out))
    return _from_bits(out, dt)


def quantize_weight_rowwise(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    x = np.ascontiguousarray(w.float().numpy())
    N, K = x.shape
    q, s = np.empty((N, K), np.int8), np.empty(N, np.float32)
    load().fni8o_quantize_weight_rows(_p(x), N, K, _p(q), _p(s))
    return torch.from_numpy(q), torch.from_numpy(s)


def quantize_rows(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    b, dt = _half_bits(x)
    M, K = b.shape
    q, s = np.empty((M, K), np.int8), np.empty(M, np.float32)
    load().fni8o_quantize_rows(_p(b), dt, M, K, _p(q), _p(s))
    return torch.from_numpy(q), torch.from_numpy(s)


def gemm_i32(a: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    an, wn = np.ascontiguousarray(a.numpy()), np.ascontiguousarray(w.numpy())
    (M, K), N = an.shape, wn.shape[0]
    acc = np.empty((M, N), np.int32)
    if load().fni8o_gemm_i32(_p(an), _p(wn), M, N, K, _p(acc)):
        raise OverflowError("int32 accumulator range exceeded")
    return torch.from_numpy(acc)


def dequant(acc: torch.Tensor, a_scale: torch.Tensor, w_scale: torch.Tensor, bias: torch.Tensor | None = None,
            residual: torch.Tensor | None = None, out_dtype: torch.dtype = torch.float16) -> torch.Tensor:
    accn = np.ascontiguousarray(acc.numpy())
    M, N = accn.shape
    asn = np.ascontiguousarray(a_scale.float().numpy())
    wsn = np.ascontiguousarray(w_scale.float().numpy())
    bn = _half_bits(bias.to(out_dtype))[0] if bias is not None else None
    rn = _half_bits(residual.to(out_dtype))[0] if residual is not None else None
    dt = F16 if out_dtype == torch.float16 else BF16
    out = np.empty((M, N), np.int16)
    load().fni8o_dequant(_p(accn), _p(asn), _p(wsn), _p(bn), _p(rn), dt, M, N, _p(out))
    return _from_bits(out, dt)


def linear_w8a8(x: torch.Tensor, wq: torch.Tensor, ws: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    K = x.shape[-1]
    b, dt = _half_bits(x.reshape(-1, K))
    M = b.shape[0]
    wn, wsn = np.ascontiguousarray(wq.numpy()), np.ascontiguousarray(ws.float().numpy())
    N = wn.shape[0]
    bn = _half_bits(bias.to(x.dtype))[0] if bias is not None else None
    q, s = np.empty((M, K), np.int8), np.empty(M, np.float32)
    acc, out = np.empty((M, N), np.int32), np.empty((M, N), np.int16)
    if load().fni8o_linear_w8a8(_p(b), dt, M, K, _p(wn), _p(wsn), N, _p(bn), _p(q), _p(s), _p(acc), _p(out)):
        raise OverflowError("int32 accumulator range exceeded")
    return _from_bits(out, dt).reshape(*x.shape[:-1], N)


def unpack_i4(packed: torch.Tensor) -> torch.Tensor:
    p = np.ascontiguousarray(packed.numpy())
    N, K = p.shape[0], 2 * p.shape[1]
    codes = np.empty((N, K), np.int8)
    load().fni8o_unpack_i4(_p(p), N, K, _p(codes))
    return torch.from_numpy(codes)


def dequant_weight_i4_fallback(packed: torch.Tensor, scale: torch.Tensor, group_size: int) -> torch.Tensor:
    p = np.ascontiguousarray(packed.numpy())
    sc = np.ascontiguousarray(scale.float().numpy())
    N, K = p.shape[0], 2 * p.shape[1]
    codes, out = np.empty((N, K), np.int8), np.empty((N, K), np.int16)
    load().fni8o_dequant_weight_i4(_p(p), _p(sc), N, K, group_size, _p(codes), _p(out))
    return _from_bits(out, F16)


def linear_w4a8(x: torch.Tensor, packed: torch.Tensor, scale: torch.Tensor, group_size: int,
                bias: torch.Tensor | None = None) -> torch.Tensor:
    K = x.shape[-1]
    b, dt = _half_bits(x.reshape(-1, K))
    M = b.shape[0]
    p = np.ascontiguousarray(packed.numpy())
    sc = np.ascontiguousarray(scale.float().numpy())
    N = p.shape[0]
    if 2 * p.shape[1] != K or K % group_size:
        raise ValueError("packed weight does not match K / group_size")
    bn = _half_bits(bias.to(x.dtype))[0] if bias is not None else None
    q, s = np.empty((M, K), np.int8), np.empty(M, np.float32)
    codes, out = np.empty((N, K), np.int8), np.empty((M, N), np.int16)
    load().fni8o_linear_w4a8(_p(b), dt, M, K, _p(p), _p(sc), N, group_size, _p(bn), _p(q), _p(s), _p(codes), _p(out))
    return _from_bits(out, dt).reshape(*x.shape[:-1], N)


def moe_plan(topi: torch.Tensor, E: int):
    """(counts [E], offsets [E+1], row_of_slot [T*k], slot_of_row [rows]) as int64 tensors."""
    ti = np.ascontiguousarray(topi.reshape(-1).to(torch.int32).numpy())
    n = ti.size
    counts, offsets = np.empty(E, np.int32), np.empty(E + 1, np.int32)
    ros, sor, cur = np.empty(n, np.int32), np.empty(max(n, 1), np.int32), np.empty(E, np.int32)
    rows = load().fni8o_moe_plan(_p(ti), n, E, _p(counts), _p(offsets), _p(ros), _p(sor), _p(cur))
    return (torch.from_numpy(counts).long(), torch.from_numpy(offsets).long(), torch.from_numpy(ros).long(),
            torch.from_numpy(sor[:rows].copy()).long())


def moe_combine(y: torch.Tensor, row_of_slot: torch.Tensor, topw: torch.Tensor) -> torch.Tensor:
    b, dt = _half_bits(y)
    T, k = topw.shape
    H = b.shape[1]
    ros = np.ascontiguousarray(row_of_slot.reshape(-1).to(torch.int32).numpy())
    tw = np.ascontiguousarray(topw.float().numpy())
    out = np.empty((T, H), np.int16)
    load().fni8o_moe_combine(_p(b), dt, _p(ros), _p(tw), T, k, H, _p(out))
    return _from_bits(out, dt)
