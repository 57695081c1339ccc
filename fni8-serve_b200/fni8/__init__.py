"""fni8 — B200-native (sm_100a) drop-in for the `fni8` kernel package fni8-serve imports.

fni8-serve's layers import exactly these names (fni8serve/layers/linear.py:19-25,
norm.py:16, activation.py:10, models/weights.py:14-15):

    fni8.QTensor, fni8.linear, fni8.rmsnorm, fni8.act_and_mul,
    fni8.quant.core.quantize_int8_rowwise

Put the directory that contains this package first on sys.path and LinearW8A8,
RMSNorm, SiluAndMul/GeluAndMul and GatedMLP run unchanged on hand-written tcgen05 /
TMA kernels through the C ABI of include/fni8_b200.h. `fni8.moe.SparseMoE` replaces
the per-expert Python loop with grouped GEMMs, `fni8.parallel` adds the
expert-parallel and column-parallel multi-GPU forms, and `fni8.format` (FQReader,
FQWriter, save_fni8; fni8serve/loader.py:16, convert.py:320) reads and writes the
`.fni8` weight container.

Importing the package does not load the native library; the first op does, and it
raises if the library has not been built (there is no fallback path).
"""
from . import format, mlp, quant  # noqa: F401
from ._native import Fni8Error
from .format import FQReader, FQWriter, save_fni8
from .ops import (act_and_mul, act_and_mul_quant, device_status, gemm_i32, linear, linear_act_q, linear_q,
                  quantize_rows, rmsnorm, rmsnorm_quant)
from .qtensor import QTensor

__all__ = [
    "QTensor", "linear", "rmsnorm", "act_and_mul", "quant",
    "rmsnorm_quant", "act_and_mul_quant", "linear_q", "linear_act_q", "quantize_rows", "gemm_i32", "device_status",
    "Fni8Error", "FQReader", "FQWriter", "save_fni8", "format",
]
__version__ = "0.1.0"
