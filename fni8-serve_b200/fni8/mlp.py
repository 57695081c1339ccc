"""Drop-in for fni8serve.layers.mlp.GatedMLP: down(act_and_mul(gate_up(x))).

Same constructor as the reference (fni8serve/layers/mlp.py:22-40): merged gate_up and
down QTensors, `act`, optional biases. The reference composes three calls
(LinearW8A8 -> SiluAndMul/GeluAndMul -> LinearW8A8), which materialises the [M, 2I]
gate_up output in fp16 and reads it back. Here, at prefill sizes, the gate_up GEMM
applies act(gate) * up in its epilogue (fni8.linear_act_q), so only the [M, I] product is
written; it is quantised per token and fed to the down projection. Results are identical
bit for bit to the composed fni8 calls. Decode-sized batches (where the split-K kernels
stream the weights) and layers the fused GEMM does not cover (biases, I not a multiple of
128, 4-bit weights) take the composed path.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from .ops import act_and_mul, linear, linear_act_q, linear_q, quantize_rows
from .qtensor import QTensor

_ACTS = {"silu": "silu", "gelu_tanh": "gelu_tanh", "gelu_pytorch_tanh": "gelu_tanh"}
# token count from which the fused tile GEMM is used (below it the split-K decode kernels win)
FUSED_MIN_TOKENS = 257


class GatedMLP(nn.Module):
    def __init__(self, gate_up: QTensor, down: QTensor, *, act: str = "silu", bias_gate_up=None, bias_down=None):
        super().__init__()
        if act not in _ACTS:
            raise ValueError(f"GatedMLP: unsupported activation {act!r}")
        self.gate_up = gate_up
        self.down = down
        self.act = _ACTS[act]
        self.bias_gate_up = bias_gate_up
        self.bias_down = bias_down
        self.hidden_size = down.data.shape[0]
        self.intermediate_size = gate_up.data.shape[0] // 2

    def _fusable(self, M: int) -> bool:
        return (M >= FUSED_MIN_TOKENS and self.bias_gate_up is None and self.gate_up.scheme == "per_row_i8"
                and self.down.scheme == "per_row_i8" and self.intermediate_size % 128 == 0)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        K = x.shape[-1]
        M = x.numel() // K
        if not self._fusable(M):
            return linear(act_and_mul(linear(x, self.gate_up, bias=self.bias_gate_up), self.act), self.down,
                          bias=self.bias_down)
        q, s = quantize_rows(x)
        p = linear_act_q(q, s, self.gate_up, self.act, out_dtype=x.dtype)
        hq, hs = quantize_rows(p)
        return linear_q(hq, hs, self.down, bias=self.bias_down, out_dtype=x.dtype)
