"""`fni8.quant.core.quantize_int8_rowwise`: per-output-row symmetric int8 weights.

Called at load time by fni8serve/models/weights.py:24 (`to_qtensor`) and
fni8serve/convert.py:65. The arithmetic restates the reference tests' own fixture
(tests/test_layers.py:29-33): scale = absmax(row).clamp_min(1e-6) / 127,
q = round_half_even(w / scale) clamped to [-127, 127]; computed in fp32 here.
Returns (q int8 [O, I], scale fp32 [O, 1]) — the call sites squeeze the last dim.
This is load-time preprocessing on whatever device `w` lives on, not a hot-path op.
"""
from __future__ import annotations

import torch


def quantize_int8_rowwise(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    if w.dim() != 2:
        raise ValueError("quantize_int8_rowwise expects a 2-D weight [out, in]")
    wf = w.float()
    s = wf.abs().amax(dim=-1, keepdim=True).clamp_min(1e-6) / 127.0
    q = torch.round(wf / s).clamp_(-127, 127).to(torch.int8)
    return q, s
