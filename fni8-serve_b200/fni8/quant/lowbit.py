"""`fni8.quant.lowbit.quantize_lowbit`: symmetric per-group low-bit weights.

Called by fni8-serve's converter for 4-bit checkpoints (fni8serve/convert.py:24,69-79:
`codes, scale = quantize_lowbit(w, 4, dim=-1, group_size=g)`, codes [O, I] and scale
[O, I // g], which it packs two per byte into a `per_group_i4` QTensor with codebook
"int4"). The original lives in the absent `fni8` package; this restates the scheme the
W4A8 kernel and its tests assume: per group of `group_size` consecutive elements along
`dim`, scale = absmax / (2^(bits-1) - 1) (at least 1e-8), codes = round_half_even(w /
scale) clamped to [-2^(bits-1), 2^(bits-1) - 1]; fp32 arithmetic. The reference's own
reconstruction (fni8serve/layers/linear.py:33-45) is code * scale per group, which these
codes satisfy. The NF4 codebook is not provided: fni8-serve then leaves NF4_CODEBOOK unset
(linear.py:22-25) and the W4A8 kernel takes the int4 codebook only.
"""
from __future__ import annotations

import torch


def quantize_lowbit(w: torch.Tensor, bits: int, dim: int = -1, group_size: int = 128):
    if not 2 <= bits <= 8:
        raise ValueError(f"quantize_lowbit: bits must be in [2, 8] (got {bits})")
    if group_size <= 0:
        raise ValueError("quantize_lowbit: group_size must be positive")
    wf = w.float().movedim(dim, -1)
    n = wf.shape[-1]
    if n % group_size:
        raise ValueError(f"quantize_lowbit: {n} elements along dim do not split into groups of {group_size}")
    qmax = (1 << (bits - 1)) - 1
    g = wf.reshape(*wf.shape[:-1], n // group_size, group_size)
    scale = (g.abs().amax(-1) / float(qmax)).clamp_min(1e-8)
    codes = torch.round(g / scale.unsqueeze(-1)).clamp_(-(qmax + 1), qmax).to(torch.int8)
    codes = codes.reshape(*wf.shape).movedim(-1, dim)
    return codes, scale.movedim(-1, dim) if dim not in (-1, w.dim() - 1) else scale
