"""Multi-GPU forms of the W8A8 path: expert parallelism for the MoE block and column
(output-channel) sharding for dense layers. One process per GPU, NCCL over NVLink /
NVSwitch through torch.distributed.

The reference has neither: its MoE runs every expert locally (fni8serve/models/moe.py:99-105)
and its config forbids tensor parallelism on its PCIe fleet (fni8serve/config.py:40-45).
Both are new capabilities sized for an 8 x B200 NVSwitch box.

Expert parallel (rank r owns experts [r*E/P, (r+1)*E/P)):
    quantise own tokens -> group (token, slot) pairs by expert (= by owner rank)
    -> all_to_all of per-expert counts -> all_to_all of int8 rows + fp32 scales
    -> grouped GEMMs over (source rank, local expert) segments
    -> all_to_all of fp16 expert outputs back -> weighted combine.
Activations cross NVLink as int8 (half the bytes of fp16). The split sizes are the only
values that visit the host (one small copy per layer, needed by all_to_all_single).

Column parallel: rank r holds rows [r*N/P, (r+1)*N/P) of W and its scales, computes
y[:, slice] with the local GEMM and all_gathers the slices. Large batches go in row chunks
whose all_gathers run asynchronously, so chunk c's exchange over NVLink overlaps the GEMM
of chunk c+1; rows are independent, so the result is the same bit for bit.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _native as nat
from .moe import ExpertStack, combine, grouped_gemm, plan
from .ops import _need_cuda, _stream, _vp, act_and_mul_quant, linear, quantize_rows
from .qtensor import QTensor


def gather_rows(q: torch.Tensor, scale: torch.Tensor, slot_of_row: torch.Tensor, rows: int, top_k: int):
    """q_out[r] = q[slot_of_row[r] // top_k] for r < rows (int8 rows + fp32 scales)."""
    _need_cuda(q, "parallel.gather_rows")
    K = q.shape[1]
    qo = torch.empty((rows, K), dtype=torch.int8, device=q.device)
    so = torch.empty((rows,), dtype=torch.float32, device=q.device)
    nat.call("fni8_moe_gather_rows_i8", _vp(q), _vp(scale), _vp(slot_of_row), rows, K, top_k, _vp(qo), _vp(so),
             _stream(q.device))
    return qo, so


def expert_shard(num_experts: int, world: int, rank: int) -> tuple[int, int]:
    if num_experts % world:
        raise ValueError(f"{num_experts} experts do not split over {world} ranks")
    per = num_experts // world
    return rank * per, (rank + 1) * per


def exchange_plan(counts: torch.Tensor, world: int, group=None):
    """Per-expert counts of this rank -> (recv_counts [P, E/P] device, send_splits, recv_splits).

    recv_counts[s, e] is how many rows source rank s sends for local expert e. This is the
    single host synchronisation of an expert-parallel layer.
    """
    E = counts.numel()
    recv = torch.empty_like(counts)
    dist.all_to_all_single(recv, counts, group=group)
    both = torch.cat([counts.view(world, E // world).sum(1), recv.view(world, E // world).sum(1)]).cpu()
    send_splits = both[:world].tolist()
    recv_splits = both[world:].tolist()
    return recv.view(world, E // world), send_splits, recv_splits


def segments_from_counts(recv_counts: torch.Tensor):
    """(source rank, local expert) segments in arrival order: expert ids, offsets, counts."""
    P, El = recv_counts.shape
    cnt = recv_counts.reshape(-1).to(torch.int32)
    off = torch.zeros_like(cnt)
    off[1:] = torch.cumsum(cnt, 0)[:-1].to(torch.int32)
    exp = torch.arange(El, dtype=torch.int32, device=cnt.device).repeat(P)
    return exp, off, cnt


class KernelOps:
    """The device kernels one expert-parallel layer uses (the C ABI through fni8)."""

    quantize_rows = staticmethod(quantize_rows)
    plan = staticmethod(plan)
    gather_rows = staticmethod(gather_rows)
    grouped_gemm = staticmethod(grouped_gemm)
    act_and_mul_quant = staticmethod(act_and_mul_quant)
    combine = staticmethod(combine)


class ExpertParallelMoE:
    """Routed-expert block with experts sharded over the ranks of `group`.

    `ops` supplies the compute steps (default: the sm_100a kernels); the exchange logic
    around them is what this class owns."""

    def __init__(self, local: ExpertStack, num_experts: int, group=None, act: str = "silu", ops=KernelOps):
        self.local = local
        self.E = num_experts
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.act = act
        self.ops = ops
        lo, hi = expert_shard(num_experts, self.world, self.rank)
        if local.num_experts != hi - lo:
            raise ValueError("local expert stack does not match this rank's shard")

    def __call__(self, x: torch.Tensor, topi: torch.Tensor, topw: torch.Tensor) -> torch.Tensor:
        T, H = x.shape
        k = topi.shape[1]
        ops = self.ops
        xq, xs = ops.quantize_rows(x)
        counts, offsets, ros, sor = ops.plan(topi, self.E)
        recv_counts, send_splits, recv_splits = exchange_plan(counts, self.world, self.group)
        n_send, n_recv = sum(send_splits), sum(recv_splits)
        aq, as_ = ops.gather_rows(xq, xs, sor, n_send, k)
        rq = torch.empty((n_recv, H), dtype=torch.int8, device=x.device)
        rs = torch.empty((n_recv,), dtype=torch.float32, device=x.device)
        dist.all_to_all_single(rq, aq, recv_splits, send_splits, group=self.group)
        dist.all_to_all_single(rs, as_, recv_splits, send_splits, group=self.group)
        exp, off, cnt = segments_from_counts(recv_counts)
        L = self.local
        h = ops.grouped_gemm(rq, rs, L.w_gu, L.s_gu, exp, off, cnt, out_dtype=x.dtype)
        hq, hs = ops.act_and_mul_quant(h, self.act)
        y = ops.grouped_gemm(hq, hs, L.w_dn, L.s_dn, exp, off, cnt, out_dtype=x.dtype)
        back = torch.empty((n_send, H), dtype=x.dtype, device=x.device)
        dist.all_to_all_single(back, y, send_splits, recv_splits, group=self.group)
        return ops.combine(back, ros, topw)


def shard_rows(qt: QTensor, world: int, rank: int) -> QTensor:
    """Rows [r*N/P, (r+1)*N/P) of a per_row_i8 weight (output-channel shard)."""
    N = qt.data.shape[0]
    if N % world:
        raise ValueError(f"N={N} does not split over {world} ranks")
    lo, hi = rank * N // world, (rank + 1) * N // world
    return QTensor(qt.data[lo:hi].contiguous(), qt.scale[lo:hi].contiguous(), scheme=qt.scheme)


class ColumnParallelLinearW8A8:
    """y = x W^T with W's output channels sharded over the ranks of `group`."""

    def __init__(self, shard: QTensor, group=None, matmul=linear, chunk_rows: int = 1024):
        self.shard = shard
        self.group = group
        self.world = dist.get_world_size(group)
        self.matmul = matmul  # fni8.linear (the sm_100a kernels) unless a test swaps it
        # batches of at least 2 x chunk_rows rows are computed and exchanged in chunks
        self.chunk_rows = chunk_rows

    def __call__(self, x: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
        K = x.shape[-1]
        x2 = x.reshape(-1, K)
        M = x2.shape[0]
        n = self.shard.data.shape[0]
        if self.world == 1:
            return self.matmul(x2, self.shard, bias).reshape(*x.shape[:-1], n)
        step = self.chunk_rows if M >= 2 * self.chunk_rows else max(M, 1)
        pending = []
        for r0 in range(0, M, step):
            r1 = min(M, r0 + step)
            y = self.matmul(x2[r0:r1], self.shard, bias).contiguous()
            parts = torch.empty((self.world * (r1 - r0), n), dtype=y.dtype, device=y.device)
            work = dist.all_gather_into_tensor(parts, y, group=self.group, async_op=True)
            pending.append((r0, r1, y, parts, work))
        out = torch.empty((M, self.world * n), dtype=pending[0][2].dtype if pending else x.dtype, device=x.device)
        for r0, r1, y, parts, work in pending:
            work.wait()  # the current stream waits for this chunk's exchange
            out[r0:r1].view(r1 - r0, self.world, n).copy_(parts.view(self.world, r1 - r0, n).permute(1, 0, 2))
        return out.reshape(*x.shape[:-1], self.world * n)
