"""`fni8.quant.lowbit.quantize_lowbit`: symmetric per-group low-bit weights.

Called by fni8-serve's converter for 4-bit checkpoints (fni8serve/convert.py:24,69-79:
`codes, scale = quantize_lowbit(w, 4, dim=-1, group_size=g)`, codes [O, I] and scale
[O, I // g], which it packs two per byte into a `per_group_i4` QTensor with codebook
"int4"). The original lives in the absent `fni8` package; this restates the scheme the
W4A8 kernel and its tests assume: per group of `group_size` consecutive elements along
`dim`, scale = absmax / (2^(bits-1) - 1) (at least 1e-8), codes = round_half_even(w /
scale) clamped to [-2^(bits-1), 2^(bits-1) - 1]; fp32 arithmetic. The reference's own
reconstruction (fni8serve/layers/linear.py:33-45) is code * scale per group, which these
codes satisfy.

`NF4_CODEBOOK`: the 16 levels of 4-bit NormalFloat, which fni8-serve looks up by code for
`per_group_i4` weights with codebook "nf4" (its fp16 fallback, layers/linear.py:22-25,37-39)
and for NF4 LoRA adapters (training/qlora.py:9-11,31,54). The W4A8 kernel takes the int4
codebook only; NF4 stays on fni8-serve's fallback, which only needs the table.
"""
from __future__ import annotations

from statistics import NormalDist

import torch


def _normal_float_levels(bits: int = 4) -> list[float]:
    """NormalFloat levels (Dettmers et al., QLoRA, 2023): quantiles of N(0, 1) scaled to
    [-1, 1], built asymmetrically so that 0 is a level and all 2^bits codes are used:
    2^(bits-1) positive levels at the probabilities evenly spaced from `offset` down to
    (excluding) 1/2, 2^(bits-1) - 1 negative levels likewise, and zero. `offset` is the
    mean of 1 - 1/(2(2^bits - 1)) and 1 - 1/(2 * 2^bits), which keeps the outermost
    quantile finite. Levels ascending, float64."""
    n = 1 << bits
    offset = 0.5 * ((1 - 1 / (2 * (n - 1))) + (1 - 1 / (2 * n)))
    ppf = NormalDist().inv_cdf

    def side(count: int) -> list[float]:
        step = (offset - 0.5) / count
        return [ppf(offset - i * step) for i in range(count)]

    levels = side(n // 2) + [0.0] + [-v for v in side(n // 2 - 1)]
    top = max(levels)
    return sorted(v / top for v in levels)


NF4_CODEBOOK: list[float] = _normal_float_levels(4)


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
