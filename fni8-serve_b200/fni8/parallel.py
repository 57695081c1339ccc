"""Multi-GPU forms of the W8A8 path: expert parallelism for the MoE block and column
(output-channel) sharding for dense layers. One process per GPU, NCCL over NVLink /
NVSwitch through torch.distributed.

The reference has neither: its MoE runs every expert locally (fni8serve/models/moe.py:99-105)
and its config forbids tensor parallelism on its PCIe fleet (fni8serve/config.py:40-45).
Both are new capabilities sized for an 8 x B200 NVSwitch box.

Expert parallel (rank r owns E/P experts: [r*E/P, (r+1)*E/P), or those a load-balanced
placement gives it, balanced_placement), two transports:
  p2p (CUDA tensors, one node): quantise own tokens -> group (token, slot) pairs by expert
    -> per-expert counts all-gathered through peer memory -> placement computed on the
    device -> int8 rows + scales stored straight into the owners' receive buffers (CUDA
    IPC peer memory over NVLink) -> grouped GEMMs, one segment per local expert, the down
    projection's epilogue storing each expert output straight back into its source's
    buffer, at the row's index in the source's expert-sorted order -> weighted combine. Each exchange ends in a barrier kernel over
    peer memory (PeerSync) on the same stream, so a rank reads its buffers only after every
    rank's stores are done. Nothing visits the host: the layer replays from a CUDA graph.
  nccl (any backend, gloo included): the same steps with all_to_all_single; the split
    sizes visit the host (one small copy per layer).
Activations cross NVLink as int8 (half the bytes of fp16).

Column parallel: rank r holds rows [r*N/P, (r+1)*N/P) of W and its scales and computes
y[:, slice]; every rank needs all of y. Two transports:
  p2p (CUDA, one node): the GEMM stores its slice straight into every rank's output buffer
    (CUDA IPC peer memory over NVLink): at prefill sizes from the tile GEMM's epilogue, so
    each tile crosses NVLink while later tiles compute; at decode sizes by a copy kernel
    after the split-K GEMM. A barrier kernel over peer memory then orders the ranks.
  nccl (any backend): the local GEMM and all_gather_into_tensor, in row chunks whose
    exchanges run asynchronously.
Rows and columns are independent, so every form gives the single-GPU result bit for bit.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _native as nat
from .moe import ExpertStack, combine, grouped_gemm, grouped_gemm_act, plan
from .ops import (_ACT, _DT, _need_cuda, _stream, _vp, act_and_mul_quant, linear, linear_q_peer_cols,
                  quantize_rows)
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


def balanced_placement(load, world: int) -> torch.Tensor:
    """Expert placement for expert parallelism from per-expert loads (rows routed to each
    expert, e.g. counted over recent batches on all ranks): every rank owns E/P experts and
    the ranks' total loads are as even as a greedy longest-load-first assignment makes them
    (the heaviest remaining expert goes to the least-loaded rank with room; ties by id, so
    every rank computes the same placement). Returns place [E] int64: expert e runs on rank
    place[e] // (E/P) as its local expert place[e] % (E/P). With skewed routing the
    contiguous placement (place[e] = e) leaves one rank with several of the heaviest experts,
    and every rank waits for it."""
    c = [float(v) for v in torch.as_tensor(load).reshape(-1).tolist()]
    E = len(c)
    if E % world:
        raise ValueError(f"{E} experts do not split over {world} ranks")
    per = E // world
    total = [0.0] * world
    used = [0] * world
    place = [0] * E
    for e in sorted(range(E), key=lambda i: (-c[i], i)):
        r = min((r for r in range(world) if used[r] < per), key=lambda r: (total[r], r))
        place[e] = r * per + used[r]
        used[r] += 1
        total[r] += c[e]
    return torch.tensor(place, dtype=torch.int64)


def experts_of_rank(place: torch.Tensor, world: int, rank: int) -> list[int]:
    """The expert ids rank `rank` holds under `place` (balanced_placement), in local order:
    its local expert stack is these experts' weights, stacked in this order."""
    p = [int(v) for v in place.tolist()]
    per = len(p) // world
    ids = [-1] * per
    for e, v in enumerate(p):
        if v // per == rank:
            ids[v % per] = e
    if min(ids) < 0:
        raise ValueError("placement does not give every rank E/P experts")
    return ids


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


def p2p_placement(cnt_all: torch.Tensor, rank: int, world: int):
    """Placement of a peer-memory exchange from cnt_all[s, e] (rows source rank s sends to
    global expert e; experts [d*El, (d+1)*El) live on rank d). Rank d's receive buffer holds
    its local experts one after another, each expert's rows ordered by source rank.
    Returns (dst_base [world, El]: where this rank's rows of (d, local expert) start in d's
    buffer; seg_off [El], seg_cnt [El]: this rank's received segments; n_recv [1])."""
    P, E = cnt_all.shape
    El = E // world
    c = cnt_all.view(P, world, El).to(torch.int32)  # [source, owner, local expert]
    tot = c.sum(0, dtype=torch.int32)  # [owner, local expert]
    base = torch.cumsum(tot, 1, dtype=torch.int32) - tot  # exclusive over local experts
    before = torch.cumsum(c, 0, dtype=torch.int32) - c  # exclusive over sources
    dst_base = (base + before[rank]).contiguous()
    return dst_base, base[rank].contiguous(), tot[rank].contiguous(), tot[rank].sum(dtype=torch.int32).reshape(1)


def ep_placement(cnt_all: torch.Tensor, rank: int, world: int):
    """p2p_placement on the device in one kernel (C: fni8_ep_placement); same outputs, int32."""
    P, E = cnt_all.shape
    c = cnt_all.to(torch.int32).contiguous()
    El = E // world
    dst_base = torch.empty((world, El), dtype=torch.int32, device=c.device)
    seg_off = torch.empty(El, dtype=torch.int32, device=c.device)
    seg_cnt = torch.empty(El, dtype=torch.int32, device=c.device)
    n_recv = torch.empty(1, dtype=torch.int32, device=c.device)
    nat.call("fni8_ep_placement", _vp(c), world, rank, E, _vp(dst_base), _vp(seg_off), _vp(seg_cnt), _vp(n_recv),
             _stream(c.device))
    return dst_base, seg_off, seg_cnt, n_recv


def _cuda_view(ptr: int, nbytes: int, device: torch.device) -> torch.Tensor:
    """uint8 tensor over device memory this module owns (no copy, no ownership)."""

    class _Mem:
        __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3,
                                    "strides": None}

    return torch.as_tensor(_Mem(), device=device)


class PeerBuffer:
    """One zeroed CUDA IPC allocation of `nbytes` on every rank of `group`, mapped into every
    rank: bases[r] is rank r's allocation as this process addresses it (bases[rank] is this
    rank's own, also viewed as the uint8 tensor `mem`)."""

    def __init__(self, nbytes: int, device: torch.device, group=None):
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        if self.world > 8:
            raise ValueError("peer memory spans at most 8 ranks")
        ptr = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        nat.call("fni8_ipc_alloc", nbytes, ctypes.byref(ptr), ctypes.cast(handle, ctypes.c_void_p))
        self._own = ptr.value
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        self._opened = []
        bases = []
        try:
            for r, h in enumerate(handles):
                if r == self.rank:
                    bases.append(self._own)
                    continue
                p = ctypes.c_void_p()
                hb = ctypes.create_string_buffer(h, 64)
                nat.call("fni8_ipc_open", ctypes.cast(hb, ctypes.c_void_p), ctypes.byref(p))
                self._opened.append(p.value)
                bases.append(p.value)
        except BaseException:
            # unmap what this rank mapped and free its own buffer before reporting the error
            for p in self._opened:
                nat.lib().fni8_ipc_close(ctypes.c_void_p(p))
            nat.lib().fni8_ipc_free(ctypes.c_void_p(self._own))
            self._opened, self._own = [], None
            raise
        self.bases = bases
        self.nbytes = nbytes
        self.mem = _cuda_view(self._own, nbytes, device)

    def pointers(self, offset: int = 0):
        """Every rank's base + offset, as the ctypes pointer array the kernels take."""
        return (ctypes.c_void_p * self.world)(*[b + offset for b in self.bases])

    def close(self, group=None):
        """Unmap the peers' allocations and free this rank's (every rank calls it; after a
        barrier, so no rank still stores into them)."""
        if self._own is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=group)
        for p in self._opened:
            nat.call("fni8_ipc_close", p)
        self._opened = []
        dist.barrier(group=group)
        self.mem = None
        nat.call("fni8_ipc_free", self._own)
        self._own = None


class PeerSync:
    """Barrier of the ranks over peer memory, on the current stream (C: fni8_peer_barrier):
    the flag words live in a PeerBuffer region of `world` uint32 (zeroed at allocation), the
    epoch counter in this rank's memory. A call passes once every rank has made the same
    call, and then sees every store into its memory that the ranks' earlier kernels issued;
    given src (n int32 on this rank) and dst_offset (the PeerBuffer offset of a [world, n]
    int32 region) it also all-gathers src. Waits are bounded (1 s; fni8.device_status
    reports a rank that never arrived). Every rank calls the same barriers in the same
    order."""

    def __init__(self, buf: PeerBuffer, offset: int, device: torch.device):
        self.world, self.rank = buf.world, buf.rank
        self._buf = buf
        self._flags = buf.pointers(offset)
        self._flags_p = ctypes.cast(self._flags, ctypes.c_void_p)
        self._epoch = torch.zeros(1, dtype=torch.int32, device=device)
        self._dst = {}

    def __call__(self, src: torch.Tensor | None = None, dst_offset: int | None = None):
        n = 0 if src is None else src.numel()
        dst = None
        if n:
            if dst_offset not in self._dst:
                a = self._buf.pointers(dst_offset)
                self._dst[dst_offset] = (a, ctypes.cast(a, ctypes.c_void_p))
            dst = self._dst[dst_offset][1]
        nat.call("fni8_peer_barrier", self._flags_p, self.world, self.rank, _vp(self._epoch),
                 _vp(src) if n else None, n, dst, 1000000, _stream(self._epoch.device))


class PeerExchange:
    """Receive and back buffers of one rank in one PeerBuffer, mapped into every peer of
    `group`: rows [cap] of int8 [H] + fp32 scale + int32 tag received from any rank, and back
    rows [max_tokens * top_k] of `dtype` [H] returned in this rank's expert-sorted row order,
    plus the
    per-expert counts of every rank [world, num_experts] and the flag words of the layer's
    barrier (`sync`). cap = world * max_tokens * top_k covers any routing."""

    def __init__(self, max_tokens: int, top_k: int, hidden: int, dtype: torch.dtype, device: torch.device,
                 group=None, num_experts: int = 0):
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        if self.world > 8:
            raise ValueError("the peer-memory exchange spans at most 8 ranks")
        self.max_tokens, self.top_k, self.hidden, self.dtype = max_tokens, top_k, hidden, dtype
        self.cap = self.world * max_tokens * top_k
        self.back_rows = max_tokens * top_k
        esz = torch.tensor([], dtype=dtype).element_size()
        parts = [("q", self.cap * hidden), ("s", self.cap * 4), ("tag", self.cap * 4),
                 ("back", self.back_rows * hidden * esz), ("cnt", self.world * max(num_experts, 1) * 4),
                 ("flags", self.world * 4)]
        self.off, total = {}, 0
        for name, nbytes in parts:
            self.off[name] = total
            total += (nbytes + 255) // 256 * 256
        self.nbytes = total
        self.buf = PeerBuffer(total, device, group)
        self._arrays = {name: self.buf.pointers(self.off[name]) for name, _ in parts}
        self.peer = {name: ctypes.cast(a, ctypes.c_void_p) for name, a in self._arrays.items()}
        mem = self.buf.mem
        self.rq = mem[self.off["q"]:self.off["q"] + self.cap * hidden].view(self.cap, hidden).view(torch.int8)
        self.rs = mem[self.off["s"]:self.off["s"] + self.cap * 4].view(torch.float32)
        self.tag = mem[self.off["tag"]:self.off["tag"] + self.cap * 4].view(torch.int32)
        self.back = mem[self.off["back"]:self.off["back"] + self.back_rows * hidden * esz].view(dtype).view(
            self.back_rows, hidden)
        self.num_experts = num_experts
        self.cnt = mem[self.off["cnt"]:self.off["cnt"] + self.world * max(num_experts, 1) * 4].view(torch.int32)
        self.sync = PeerSync(self.buf, self.off["flags"], device)

    def fits(self, T: int, top_k: int, hidden: int, dtype: torch.dtype) -> bool:
        return T <= self.max_tokens and top_k == self.top_k and hidden == self.hidden and dtype == self.dtype

    def close(self, group=None):
        """Unmap the peers' buffers and free this rank's (every rank calls it)."""
        self.rq = self.rs = self.tag = self.back = self.cnt = self.sync = None
        self.buf.close(group)


def ep_dispatch(xq, xs, slot_of_row, offsets, E, rank, top_k, dst_base, xchg: PeerExchange, max_rows):
    nat.call("fni8_ep_dispatch_i8", _vp(xq), _vp(xs), _vp(slot_of_row), _vp(offsets), E, xchg.world, rank, top_k,
             xchg.hidden, _vp(dst_base), xchg.peer["q"], xchg.peer["s"], xchg.peer["tag"], xchg.cap, max_rows,
             _stream(xq.device))


def ep_return(y, n_recv, xchg: PeerExchange):
    nat.call("fni8_ep_return", _vp(y), _DT[y.dtype], _vp(n_recv), xchg.cap, _vp(xchg.tag), xchg.hidden, xchg.world,
             xchg.peer["back"], xchg.back_rows, _stream(y.device))


def grouped_gemm_scatter(a, a_scale, w, w_scale, seg_expert, seg_off, seg_cnt, row_tag, peers, world, peer_rows,
                         out_dtype=torch.float16):
    """Grouped W8A8 GEMM whose output row r lands in row (row_tag[r] & 0xFFFFFF) of
    buffer peers[row_tag[r] >> 24] (a ctypes array of `world` device pointers to
    [peer_rows, N] buffers of out_dtype): the expert-parallel return fused into the down
    projection's epilogue (C: fni8_grouped_gemm_w8a8_scatter)."""
    _need_cuda(a, "grouped_gemm_scatter")
    R, K = a.shape
    E, N, _ = w.shape
    nat.call("fni8_grouped_gemm_w8a8_scatter", _vp(a), _vp(a_scale), R, _vp(w), _vp(w_scale), E, N, K, _vp(seg_expert),
             _vp(seg_off), _vp(seg_cnt), seg_expert.numel(), _vp(row_tag), peers, world, peer_rows, _DT[out_dtype],
             _stream(a.device))


def quantize_rows_dev(x: torch.Tensor, rows_dev: torch.Tensor):
    """fni8 quantize_rows over the first rows_dev[0] rows of x (the rest left as is)."""
    M, K = x.shape
    q = torch.empty((M, K), dtype=torch.int8, device=x.device)
    s = torch.empty((M,), dtype=torch.float32, device=x.device)
    nat.call("fni8_quantize_rows_i8_rows", _vp(x), _DT[x.dtype], M, K, _vp(rows_dev), _vp(q), _vp(s),
             _stream(x.device))
    return q, s


def act_and_mul_quant_rows(h: torch.Tensor, rows_dev: torch.Tensor, act: str = "silu"):
    """fni8 act_and_mul_quant over the first rows_dev[0] rows of h (the rest left as is)."""
    I = h.shape[-1] // 2
    M = h.shape[0]
    q = torch.empty((M, I), dtype=torch.int8, device=h.device)
    s = torch.empty((M,), dtype=torch.float32, device=h.device)
    nat.call("fni8_act_and_mul_quant_i8_rows", _vp(h), _DT[h.dtype], _ACT[act], M, I, _vp(rows_dev), _vp(q), _vp(s),
             _stream(h.device))
    return q, s


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

    def __init__(self, local: ExpertStack, num_experts: int, group=None, act: str = "silu", ops=KernelOps,
                 transport: str = "auto", max_tokens: int | None = None, fuse_return: bool = True,
                 placement: torch.Tensor | None = None):
        """transport: "p2p" (peer-memory exchange, CUDA, at most 8 ranks on one node),
        "nccl" (all_to_all_single, any backend) or "auto" (p2p for the NCCL backend with the
        sm_100a kernels, nccl otherwise). max_tokens: the most tokens one rank passes per
        call (p2p buffers are sized for it; default: the first call's, as a maximum over the
        ranks). fuse_return (p2p): the down projection's epilogue stores each expert output
        straight into its source's slot over NVLink (fni8_grouped_gemm_w8a8_scatter), so the
        return overlaps the GEMM; False runs the GEMM and then the return kernel. placement:
        which rank holds which expert (balanced_placement; `local` then holds
        experts_of_rank(placement, world, rank) in that order); default: rank r holds experts
        [r*E/P, (r+1)*E/P). Every rank passes the same placement."""
        self.fuse_return = fuse_return
        if placement is not None:
            placement = torch.as_tensor(placement, dtype=torch.int64).reshape(-1)
            if placement.numel() != num_experts or not torch.equal(placement.sort().values,
                                                                   torch.arange(num_experts)):
                raise ValueError("placement must be a permutation of the expert ids")
        self.placement = placement
        self._place_dev = None
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
        if transport == "auto":
            transport = "p2p" if (ops is KernelOps and dist.get_backend(group) == "nccl" and self.world <= 8) else "nccl"
        if transport not in ("p2p", "nccl"):
            raise ValueError(f"unknown transport {transport!r}")
        self.transport = transport
        self.max_tokens = max_tokens
        self.xchg: PeerExchange | None = None

    def close(self):
        """Release the peer-memory buffers (every rank calls it)."""
        if self.xchg is not None:
            self.xchg.close(self.group)
            self.xchg = None

    def _placed(self, topi: torch.Tensor) -> torch.Tensor:
        """Expert ids -> placement slots (rank * E/P + local index); ids outside [0, E) stay
        as they are (the plan drops them)."""
        if self.placement is None:
            return topi
        if self._place_dev is None or self._place_dev.device != topi.device:
            self._place_dev = self.placement.to(device=topi.device, dtype=torch.int32)
        if topi.is_cuda and topi.dtype == torch.int32:  # one kernel (C: fni8_moe_map_ids)
            t = topi.contiguous()
            out = torch.empty_like(t)
            nat.call("fni8_moe_map_ids", _vp(t), t.numel(), _vp(self._place_dev), self.E, _vp(out),
                     _stream(t.device))
            return out
        ok = (topi >= 0) & (topi < self.E)
        return torch.where(ok, self._place_dev.to(topi.dtype)[topi.clamp(0, self.E - 1).long()], topi)

    def __call__(self, x: torch.Tensor, topi: torch.Tensor, topw: torch.Tensor) -> torch.Tensor:
        topi = self._placed(topi)
        if self.transport == "p2p":
            return self._p2p(x, topi, topw)
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

    def _p2p(self, x: torch.Tensor, topi: torch.Tensor, topw: torch.Tensor) -> torch.Tensor:
        _need_cuda(x, "ExpertParallelMoE")
        T, H = x.shape
        k = topi.shape[1]
        P, E, El = self.world, self.E, self.E // self.world
        if self.xchg is None:
            mt = self.max_tokens
            if mt is None:
                m = torch.tensor([T], dtype=torch.int64, device=x.device)
                dist.all_reduce(m, op=dist.ReduceOp.MAX, group=self.group)
                mt = int(m.item())
            self.xchg = PeerExchange(mt, k, H, x.dtype, x.device, self.group, num_experts=E)
            self._iota = torch.arange(El, dtype=torch.int32, device=x.device)
        X = self.xchg
        if not X.fits(T, k, H, x.dtype):
            raise ValueError(f"ExpertParallelMoE: {T} tokens x top-{k} x {H} {x.dtype} exceeds the exchange buffers "
                             f"({X.max_tokens} x top-{X.top_k} x {X.hidden} {X.dtype}); pass max_tokens")
        xq, xs = quantize_rows(x)
        counts, offsets, ros, sor = plan(topi, E)
        X.sync(counts.to(torch.int32).contiguous(), X.off["cnt"])  # every rank's counts, all-gathered
        dst_base, seg_off, seg_cnt, n_recv = ep_placement(X.cnt.view(P, E), self.rank, P)
        ep_dispatch(xq, xs, sor, offsets, E, self.rank, k, dst_base, X, T * k)
        X.sync()  # every rank's rows have landed
        L = self.local
        if L.intermediate % 128 == 0:  # gate_up with act_and_mul in its epilogue
            p = grouped_gemm_act(X.rq, X.rs, L.w_gu, L.s_gu, self._iota, seg_off, seg_cnt, act=self.act,
                                 out_dtype=x.dtype)
            hq, hs = quantize_rows_dev(p, n_recv)
        else:
            h = grouped_gemm(X.rq, X.rs, L.w_gu, L.s_gu, self._iota, seg_off, seg_cnt, out_dtype=x.dtype)
            hq, hs = act_and_mul_quant_rows(h, n_recv, self.act)
        if self.fuse_return:  # each output row goes straight to its source's slot
            grouped_gemm_scatter(hq, hs, L.w_dn, L.s_dn, self._iota, seg_off, seg_cnt, X.tag, X.peer["back"],
                                 X.world, X.back_rows, out_dtype=x.dtype)
        else:
            y = grouped_gemm(hq, hs, L.w_dn, L.s_dn, self._iota, seg_off, seg_cnt, out_dtype=x.dtype)
            ep_return(y, n_recv, X)
        X.sync()  # every output is back at its source
        return combine(X.back[: T * k], ros, topw)  # back rows in this rank's sorted order


def shard_rows(qt: QTensor, world: int, rank: int) -> QTensor:
    """Rows [r*N/P, (r+1)*N/P) of a per_row_i8 weight (output-channel shard)."""
    N = qt.data.shape[0]
    if N % world:
        raise ValueError(f"N={N} does not split over {world} ranks")
    lo, hi = rank * N // world, (rank + 1) * N // world
    return QTensor(qt.data[lo:hi].contiguous(), qt.scale[lo:hi].contiguous(), scheme=qt.scheme)


class ColumnParallelLinearW8A8:
    """y = x W^T with W's output channels sharded over the ranks of `group`.

    transport "p2p" (the sm_100a kernels, NCCL group of at most 8 ranks on one node): the
    GEMM stores this rank's columns straight into every rank's output buffer over NVLink
    (fni8.ops.linear_q_peer_cols), then a barrier kernel over peer memory (PeerSync) on the
    same stream orders the ranks; no host synchronisation, so a decode runner can capture it. The
    output buffers are the layer's own: `ring` buffers of [max_rows, world * n] in CUDA IPC
    memory (max_rows default: the first call's rows, as a maximum over the ranks), used in
    turn. A call returns a view of its buffer, valid until `ring` more calls of this layer
    (copy=True returns a tensor of its own). close() releases them (every rank, before
    destroy_process_group).
    transport "nccl" (any backend): the local GEMM (`matmul`) and all_gather_into_tensor;
    batches of at least 2 * chunk_rows rows go in row chunks whose exchanges run
    asynchronously.
    "auto": p2p for the NCCL backend with the sm_100a kernels and per_row_i8 shards, else nccl.
    """

    def __init__(self, shard: QTensor, group=None, matmul=linear, chunk_rows: int = 1024, transport: str = "auto",
                 max_rows: int | None = None, ring: int = 2):
        self.shard = shard
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.matmul = matmul  # fni8.linear (the sm_100a kernels) unless a test swaps it
        self.chunk_rows = chunk_rows
        if transport == "auto":
            transport = ("p2p" if (matmul is linear and 1 < self.world <= 8 and shard.scheme == "per_row_i8" and
                                   shard.data.is_cuda and dist.get_backend(group) == "nccl") else "nccl")
        if transport not in ("p2p", "nccl"):
            raise ValueError(f"unknown transport {transport!r}")
        if transport == "p2p" and shard.data.shape[0] % 64:
            raise ValueError(f"p2p column all-gather takes shards of a multiple of 64 columns "
                             f"(got {shard.data.shape[0]})")
        if ring < 1:
            raise ValueError("ring must be at least 1")
        self.transport = transport
        self.max_rows = max_rows
        self.ring = ring
        self.buf: PeerBuffer | None = None

    def close(self):
        """Release the p2p output buffers (every rank calls it)."""
        if self.buf is not None:
            self.buf.close(self.group)
            self.buf = None

    def __call__(self, x: torch.Tensor, bias: torch.Tensor | None = None, copy: bool = False) -> torch.Tensor:
        K = x.shape[-1]
        x2 = x.reshape(-1, K)
        M = x2.shape[0]
        n = self.shard.data.shape[0]
        if self.world == 1:
            return self.matmul(x2, self.shard, bias).reshape(*x.shape[:-1], n)
        if self.transport == "p2p":
            y = self._p2p(x2, bias)
            return (y.clone() if copy else y).reshape(*x.shape[:-1], self.world * n)
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

    def _p2p(self, x2: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
        _need_cuda(x2, "ColumnParallelLinearW8A8")
        M, K = x2.shape
        n = self.shard.data.shape[0]
        Nt = self.world * n
        if self.buf is None:
            rows = self.max_rows
            if rows is None:
                m = torch.tensor([M], dtype=torch.int64, device=x2.device)
                dist.all_reduce(m, op=dist.ReduceOp.MAX, group=self.group)
                rows = int(m.item())
            self._rows = max(rows, 1)
            self._slot = (self._rows * Nt * 2 + 255) // 256 * 256  # 16-bit outputs
            self.buf = PeerBuffer(self.ring * self._slot + 256, x2.device, self.group)  # + barrier flags
            self._arrays = [self.buf.pointers(i * self._slot) for i in range(self.ring)]
            self._ptrs = [ctypes.cast(a, ctypes.c_void_p) for a in self._arrays]
            self._sync = PeerSync(self.buf, self.ring * self._slot, x2.device)
            self._next = 0
        if M > self._rows:
            raise ValueError(f"ColumnParallelLinearW8A8: {M} rows exceed the output buffers ({self._rows}); "
                             "pass max_rows")
        i = self._next
        self._next = (i + 1) % self.ring
        q, s = quantize_rows(x2)
        linear_q_peer_cols(q, s, self.shard, self._ptrs[i], self.world, Nt, self.rank * n, bias=bias,
                           out_dtype=x2.dtype)
        self._sync()  # every rank's columns have landed
        return self.buf.mem[i * self._slot:i * self._slot + M * Nt * 2].view(x2.dtype).view(M, Nt)
