"""Grouped W8A8 expert GEMMs behind fni8-serve's SparseMoE.

The reference runs the routed experts as a Python loop over E experts, each doing
`mask.any()` / `nonzero()` (host syncs), a gather, a GatedMLP on the dp4a GEMM and an
`index_add_` (fni8serve/models/moe.py:97-105). Here the same computation is one device
pipeline without host synchronisation (capturable in a CUDA graph):

    route    softmax/sigmoid + (group-limited) top-k + renorm      moe.py:65-95
    quant    per-token int8 of the hidden states, once per token
    plan     stable grouping of (token, slot) pairs by expert
    gather   int8 rows into expert order
    GEMM     grouped tcgen05 gate_up over all experts in one persistent launch
    act      SiLU(gate) * up -> per-token int8
    GEMM     grouped tcgen05 down
    combine  out[t] = sum_j w[t, j] * y[row(t, j)]                moe.py:97,105

`SparseMoE` below takes the reference module's constructor arguments unchanged
(moe.py:25-60), so `fni8serve.models.moe.SparseMoE = fni8.moe.SparseMoE` (or the
one-line import swap in that file) moves every MoE family onto the grouped kernels.
"""
from __future__ import annotations

import ctypes

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _native as nat
from .ops import _ACT, _DT, _need_cuda, _stream, _vp, act_and_mul, linear
from .qtensor import QTensor


def route(logits: torch.Tensor, top_k: int, *, scoring: str = "softmax", sel_bias: torch.Tensor | None = None,
          num_expert_groups: int | None = None, topk_group: int | None = None, norm_topk_prob: bool = True,
          scaling: float = 1.0, weight_dtype: torch.dtype = torch.float16) -> tuple[torch.Tensor, torch.Tensor]:
    """Router logits [T, E] (fp32) -> (topi int32 [T, k], topw fp32 [T, k]).

    topw holds the values the reference multiplies with after `.to(x.dtype)`
    (moe.py:95): they are rounded to `weight_dtype` (pass torch.float32 to keep fp32).
    """
    _need_cuda(logits, "moe.route")
    lg = logits.float().contiguous()
    T, E = lg.shape
    if scoring not in ("softmax", "sigmoid"):
        raise ValueError(f"unknown scoring_func {scoring!r}")
    sc = nat.SCORE_SOFTMAX if scoring == "softmax" else nat.SCORE_SIGMOID
    bias = sel_bias.float().contiguous() if (sel_bias is not None and scoring == "sigmoid") else None
    ng = int(num_expert_groups) if (num_expert_groups is not None and topk_group is not None) else 0
    tg = int(topk_group) if ng else 0
    wd = {torch.float16: nat.F16, torch.bfloat16: nat.BF16, torch.float32: nat.F32}[weight_dtype]
    topi = torch.empty((T, top_k), dtype=torch.int32, device=lg.device)
    topw = torch.empty((T, top_k), dtype=torch.float32, device=lg.device)
    nat.call("fni8_moe_route", _vp(lg), T, E, top_k, sc, _vp(bias), ng, tg, int(norm_topk_prob),
             ctypes.c_float(scaling), wd, _vp(topi), _vp(topw), _stream(lg.device))
    return topi, topw


def plan(topi: torch.Tensor, num_experts: int):
    """Stable expert grouping: (counts[E], offsets[E+1], row_of_slot[T*k], slot_of_row[T*k])."""
    _need_cuda(topi, "moe.plan")
    ti = topi.to(torch.int32).contiguous().reshape(-1)
    n = ti.numel()
    dev = ti.device
    counts = torch.empty(num_experts, dtype=torch.int32, device=dev)
    offsets = torch.empty(num_experts + 1, dtype=torch.int32, device=dev)
    ros = torch.empty(n, dtype=torch.int32, device=dev)
    sor = torch.full((n,), -1, dtype=torch.int32, device=dev)
    wsb = nat.lib().fni8_moe_plan_workspace_bytes(n, num_experts)
    ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=dev)
    nat.call("fni8_moe_plan", _vp(ti), n, num_experts, _vp(counts), _vp(offsets), _vp(ros), _vp(sor), _vp(ws),
             wsb, _stream(dev))
    return counts, offsets, ros, sor


def grouped_gemm(a: torch.Tensor, a_scale: torch.Tensor, w: torch.Tensor, w_scale: torch.Tensor,
                 seg_expert: torch.Tensor, seg_off: torch.Tensor, seg_cnt: torch.Tensor,
                 out_dtype: torch.dtype = torch.float16) -> torch.Tensor:
    """out[R, N] where rows [off[s], off[s]+cnt[s]) use expert seg_expert[s] of w[E, N, K].

    Rows outside every segment are left unwritten. out_dtype torch.int32 returns the raw
    accumulators.
    """
    _need_cuda(a, "moe.grouped_gemm")
    R, K = a.shape
    E, N, K2 = w.shape
    if K2 != K:
        raise ValueError("grouped_gemm: K mismatch")
    odt = {torch.float16: nat.F16, torch.bfloat16: nat.BF16, torch.int32: nat.I32}[out_dtype]
    out = torch.empty((R, N), dtype=out_dtype, device=a.device)
    S = seg_expert.numel()
    nat.call("fni8_grouped_gemm_w8a8", _vp(a.contiguous()), _vp(a_scale.float().contiguous()), R, _vp(w.contiguous()),
             _vp(w_scale.float().contiguous()), E, N, K, _vp(seg_expert.int().contiguous()),
             _vp(seg_off.int().contiguous()), _vp(seg_cnt.int().contiguous()), S, _vp(out), odt, _stream(a.device))
    return out


def quantize_scatter(x: torch.Tensor, row_of_slot: torch.Tensor, top_k: int, rows: int):
    """Per-token int8 quantisation of x[T, H] written straight to the expert-grouped rows of
    the plan: returns (q [rows, H] int8, scale [rows] fp32) with row row_of_slot[t*k + j]
    holding token t's codes (the quantise + gather of the expert loop in one pass)."""
    _need_cuda(x, "moe.quantize_scatter")
    x2 = x.contiguous()
    T, H = x2.shape
    q = torch.empty((rows, H), dtype=torch.int8, device=x.device)
    s = torch.empty((rows,), dtype=torch.float32, device=x.device)
    nat.call("fni8_moe_quantize_scatter_i8", _vp(x2), _DT[x.dtype], T, H, _vp(row_of_slot.int().contiguous()), top_k,
             _vp(q), _vp(s), _stream(x.device))
    return q, s


def grouped_gemm_act(a: torch.Tensor, a_scale: torch.Tensor, w_gu: torch.Tensor, s_gu: torch.Tensor,
                     seg_expert: torch.Tensor, seg_off: torch.Tensor, seg_cnt: torch.Tensor, act: str = "silu",
                     out_dtype: torch.dtype = torch.float16) -> torch.Tensor:
    """The grouped gate_up projection with act_and_mul in its epilogue: out[R, I] where rows
    [off[s], off[s]+cnt[s]) hold act(gate) * up of expert seg_expert[s] of w_gu [E, 2I, K].
    Equal bit for bit to act_and_mul(grouped_gemm(...)). Rows outside every segment are
    left unwritten."""
    _need_cuda(a, "moe.grouped_gemm_act")
    R, K = a.shape
    E, two_i, K2 = w_gu.shape
    if K2 != K:
        raise ValueError("grouped_gemm_act: K mismatch")
    I = two_i // 2
    out = torch.empty((R, I), dtype=out_dtype, device=a.device)
    S = seg_expert.numel()
    nat.call("fni8_grouped_gemm_w8a8_act", _vp(a.contiguous()), _vp(a_scale.float().contiguous()), R,
             _vp(w_gu.contiguous()), _vp(s_gu.float().contiguous()), E, I, K, _vp(seg_expert.int().contiguous()),
             _vp(seg_off.int().contiguous()), _vp(seg_cnt.int().contiguous()), S, _ACT[act], _vp(out), _DT[out_dtype],
             _stream(a.device))
    return out


def combine(y: torch.Tensor, row_of_slot: torch.Tensor, topw: torch.Tensor) -> torch.Tensor:
    """out[t] = sum_j topw[t, j] * y[row_of_slot[t*k + j]] (fp32 accumulation, one rounding)."""
    _need_cuda(y, "moe.combine")
    T, k = topw.shape
    H = y.shape[-1]
    out = torch.empty((T, H), dtype=y.dtype, device=y.device)
    nat.call("fni8_moe_combine", _vp(y.contiguous()), _DT[y.dtype], _vp(row_of_slot.int().contiguous()),
             _vp(topw.float().contiguous()), T, k, H, _vp(out), _stream(y.device))
    return out


class ExpertStack:
    """All experts' int8 weights stacked for the grouped GEMM: gate_up [E, 2I, H],
    down [E, H, I] with per-row fp32 scales [E, 2I] / [E, H]."""

    def __init__(self, w_gu: torch.Tensor, s_gu: torch.Tensor, w_dn: torch.Tensor, s_dn: torch.Tensor):
        self.w_gu, self.s_gu, self.w_dn, self.s_dn = (t.contiguous() for t in (w_gu, s_gu, w_dn, s_dn))
        self.num_experts, two_i, self.hidden = self.w_gu.shape
        self.intermediate = two_i // 2

    @classmethod
    def from_qtensors(cls, experts: list[tuple[QTensor, QTensor]]) -> "ExpertStack":
        for gu, dn in experts:
            if gu.scheme != "per_row_i8" or dn.scheme != "per_row_i8":
                raise NotImplementedError("grouped expert GEMM takes per_row_i8 experts")
        return cls(torch.stack([gu.data for gu, _ in experts]), torch.stack([gu.scale for gu, _ in experts]),
                   torch.stack([dn.data for _, dn in experts]), torch.stack([dn.scale for _, dn in experts]))

    def to(self, device) -> "ExpertStack":
        return ExpertStack(self.w_gu.to(device), self.s_gu.to(device), self.w_dn.to(device), self.s_dn.to(device))


def experts(x: torch.Tensor, topi: torch.Tensor, topw: torch.Tensor, stack: ExpertStack,
            act: str = "silu") -> torch.Tensor:
    """Routed-expert output for x[T, H] given the routing (one native call)."""
    _need_cuda(x, "moe.experts")
    if act not in _ACT:
        raise ValueError(f"unsupported activation {act!r}")
    x2 = x.contiguous()
    T, H = x2.shape
    k = topi.shape[1]
    E, I = stack.num_experts, stack.intermediate
    wsb = nat.lib().fni8_moe_experts_workspace_bytes(T, H, k, E, I)
    ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=x.device)
    out = torch.empty_like(x2)
    nat.call("fni8_moe_experts_w8a8", _vp(x2), _DT[x.dtype], T, H, _vp(topi.int().contiguous()),
             _vp(topw.float().contiguous()), k, _vp(stack.w_gu), _vp(stack.s_gu), _vp(stack.w_dn), _vp(stack.s_dn),
             E, I, _ACT[act], _vp(out), _vp(ws), wsb, _stream(x.device))
    return out


class SparseMoE(nn.Module):
    """Drop-in for fni8serve.models.moe.SparseMoE (same constructor, same routing)."""

    def __init__(self, *, gate: torch.Tensor, experts: list[tuple[QTensor, QTensor]], top_k: int,
                 norm_topk_prob: bool = True, act: str = "silu", shared_expert: tuple[QTensor, QTensor] | None = None,
                 shared_expert_gate: torch.Tensor | None = None, scoring_func: str = "softmax",
                 e_score_correction_bias: torch.Tensor | None = None, routed_scaling_factor: float = 1.0,
                 num_expert_groups: int | None = None, topk_group: int | None = None):
        super().__init__()
        self.gate = nn.Parameter(gate, requires_grad=False)
        self.top_k = top_k
        self.norm_topk_prob = norm_topk_prob
        self.scoring_func = scoring_func
        self.routed_scaling_factor = routed_scaling_factor
        self.num_expert_groups = num_expert_groups
        self.topk_group = topk_group
        self.act = "gelu_tanh" if act in ("gelu_pytorch_tanh", "gelu_tanh") else act
        self.register_buffer("e_score_bias", e_score_correction_bias.float()
                             if e_score_correction_bias is not None else None, persistent=False)
        self.stack = ExpertStack.from_qtensors(experts)
        self.shared = shared_expert
        self.shared_gate = nn.Parameter(shared_expert_gate, requires_grad=False) \
            if shared_expert_gate is not None else None

    def _apply(self, fn, recurse=True):  # move the stacked experts with .cuda()/.to()
        super()._apply(fn, recurse)
        dev = self.gate.device
        self.stack = self.stack.to(dev)
        if self.shared is not None:
            self.shared = (self.shared[0].to(dev), self.shared[1].to(dev))
        return self

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, S, H = x.shape
        xf = x.reshape(-1, H)
        router_logits = F.linear(xf.float(), self.gate.float())  # moe.py:65, same op
        topi, topw = route(router_logits, self.top_k, scoring=self.scoring_func, sel_bias=self.e_score_bias,
                           num_expert_groups=self.num_expert_groups, topk_group=self.topk_group,
                           norm_topk_prob=self.norm_topk_prob, scaling=self.routed_scaling_factor,
                           weight_dtype=x.dtype)
        out = experts(xf, topi, topw, self.stack, self.act)
        if self.shared is not None:
            gu, dn = self.shared
            shared_out = linear(act_and_mul(linear(xf, gu), self.act), dn)
            if self.shared_gate is not None:
                g = torch.sigmoid(F.linear(xf.float(), self.shared_gate.float())).to(x.dtype)
                shared_out = shared_out * g
            out = out + shared_out
        return out.reshape(B, S, H)
