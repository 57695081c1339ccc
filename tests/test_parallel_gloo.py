"""Multi-process logic of the multi-GPU forms, on CPU gloo ranks (world_size 2, and 3 for
the peer-exchange failure path).

The expert-parallel layer (fni8/parallel.py) owns the exchange: per-expert counts,
split sizes, int8 row dispatch, (source rank, local expert) segments and the combine
return trip. Here its compute steps are the CPU oracle's, so two gloo ranks must
reproduce the single-process oracle MoE bit for bit; the column-parallel linear must
reassemble the unsharded output exactly; a peer-memory exchange whose set-up fails must
release what it mapped and allocated. No GPU is involved.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class OracleOps:
    """The compute steps of ExpertParallelMoE, restated on CPU with the oracle."""

    @staticmethod
    def quantize_rows(x):
        from oracle import w8a8_oracle as O

        return O.quantize_rows(x)

    @staticmethod
    def plan(topi, E):
        from oracle import w8a8_oracle as O

        c, o, r, s = O.moe_plan(topi, E)
        return c.int(), o.int(), r.int(), s.int()

    @staticmethod
    def gather_rows(q, s, slot_of_row, rows, k):
        t = slot_of_row[:rows].long() // k
        return q[t], s[t]

    @staticmethod
    def grouped_gemm(a, a_scale, w, w_scale, exp, off, cnt, out_dtype=torch.float16):
        from oracle import w8a8_oracle as O

        out = torch.zeros((a.shape[0], w.shape[1]), dtype=out_dtype)
        for e, o, c in zip(exp.tolist(), off.tolist(), cnt.tolist()):
            if c:
                out[o:o + c] = O.dequant(O.int_mm_fast(a[o:o + c], w[e]), a_scale[o:o + c], w_scale[e],
                                         out_dtype=out_dtype)
        return out

    @staticmethod
    def act_and_mul_quant(h, act):
        from oracle import w8a8_oracle as O

        return O.quantize_rows(O.act_and_mul(h, act))

    @staticmethod
    def combine(y, row_of_slot, topw):
        T, k = topw.shape
        acc = torch.zeros((T, y.shape[1]), dtype=torch.float32)
        for j in range(k):
            r = row_of_slot.view(T, k)[:, j].long()
            acc = acc + topw[:, j:j + 1].float() * y[r].float()
        return acc.to(y.dtype)


def _weights(E, H, I):
    from oracle import w8a8_oracle as O

    g = torch.Generator().manual_seed(5)
    gu = [O.quantize_weight_rowwise(0.05 * torch.randn(2 * I, H, generator=g)) for _ in range(E)]
    dn = [O.quantize_weight_rowwise(0.05 * torch.randn(H, I, generator=g)) for _ in range(E)]
    return (torch.stack([q for q, _ in gu]), torch.stack([s for _, s in gu]),
            torch.stack([q for q, _ in dn]), torch.stack([s for _, s in dn]))


def _ep_worker(rank, world, port, errq):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from fni8.moe import ExpertStack
        from fni8.parallel import ExpertParallelMoE, balanced_placement, expert_shard, experts_of_rank
        from oracle import w8a8_oracle as O

        E, k, H, I, T = 8, 2, 64, 32, 24 + 8 * rank  # ragged: ranks hold different token counts
        w_gu, s_gu, w_dn, s_dn = _weights(E, H, I)
        lo, hi = expert_shard(E, world, rank)
        ep = ExpertParallelMoE(ExpertStack(w_gu[lo:hi], s_gu[lo:hi], w_dn[lo:hi], s_dn[lo:hi]), E, ops=OracleOps)
        g = torch.Generator().manual_seed(100 + rank)
        x = torch.randn(T, H, generator=g).half()
        bias = torch.zeros(E)
        bias[0] = 3.0  # skew: expert 0 (rank 0) is popular
        topi, topw = O.moe_route(torch.randn(T, E, generator=g) + bias, k)
        got = ep(x, topi.int(), topw.float())
        ref = O.moe_experts_w8a8(x, topi, topw.float(), w_gu, s_gu, w_dn, s_dn, exact=False)
        assert torch.equal(got, ref), (got.float() - ref.float()).abs().max()
        # load-balanced placement from the routed load of all ranks: the popular expert 0
        # and its neighbours no longer share a rank; same result bit for bit
        load = torch.bincount(topi.reshape(-1), minlength=E)
        dist.all_reduce(load)
        place = balanced_placement(load, world)
        assert place.sort().values.tolist() == list(range(E))
        ids = experts_of_rank(place, world, rank)
        epb = ExpertParallelMoE(ExpertStack(w_gu[ids], s_gu[ids], w_dn[ids], s_dn[ids]), E, ops=OracleOps,
                                placement=place)
        assert torch.equal(epb(x, topi.int(), topw.float()), ref)
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report to the parent, which fails the test
        errq.put(f"rank {rank}: {e!r}")
        raise


def _cp_worker(rank, world, port, errq):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from fni8 import QTensor
        from fni8.parallel import ColumnParallelLinearW8A8, shard_rows
        from oracle import w8a8_oracle as O

        M, K, N = 7, 64, 96
        g = torch.Generator().manual_seed(3)
        wq, ws = O.quantize_weight_rowwise(0.02 * torch.randn(N, K, generator=g))
        x = torch.randn(M, K, generator=g).half()
        full = QTensor(wq, ws)

        def mm(x2, qt, bias):
            return O.linear_w8a8(x2, qt.data, qt.scale, bias=bias, exact=False)

        cp = ColumnParallelLinearW8A8(shard_rows(full, world, rank), matmul=mm)
        got = cp(x)
        assert torch.equal(got, O.linear_w8a8(x, wq, ws, exact=False))
        # row chunks with asynchronous exchanges (7 rows in chunks of 3): same result
        cpc = ColumnParallelLinearW8A8(shard_rows(full, world, rank), matmul=mm, chunk_rows=3)
        assert torch.equal(cpc(x), O.linear_w8a8(x, wq, ws, exact=False))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        errq.put(f"rank {rank}: {e!r}")
        raise


def _ipc_fail_worker(rank, world, port, errq):
    """PeerExchange set-up where mapping a peer's buffer fails: the rank unmaps the peer it
    already mapped, frees its own buffer and raises (native calls faked on the host)."""
    try:
        import ctypes

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from fni8 import _native as nat
        from fni8.parallel import PeerExchange

        own, log, opens = 0x10000 * (rank + 1), [], [0]

        def fake_call(name, *args):
            if name == "fni8_ipc_alloc":
                args[1]._obj.value = own
                ctypes.memmove(args[2].value, b"handle-of-%d" % rank, 11)
            elif name == "fni8_ipc_open":
                opens[0] += 1
                if opens[0] == 2:
                    raise nat.Fni8Error(nat.ERR_CUDA, "fni8_ipc_open: peer mapping refused")
                args[1]._obj.value = 0x900000 + opens[0]
            else:
                raise AssertionError(f"unexpected native call {name}")

        class FakeLib:
            def fni8_ipc_close(self, p):
                log.append(("close", p.value))
                return 0

            def fni8_ipc_free(self, p):
                log.append(("free", p.value))
                return 0

        nat.call, nat.lib = fake_call, (lambda: FakeLib())
        try:
            PeerExchange(4, 2, 16, torch.float16, torch.device("cpu"))
            raise AssertionError("PeerExchange did not raise")
        except nat.Fni8Error:
            pass
        assert log == [("close", 0x900001), ("free", own)], log
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        errq.put(f"rank {rank}: {e!r}")
        raise


def _spawn(worker, world):
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    for p in procs:
        if p.is_alive():
            p.kill()
            errs.append("rank timed out")
    assert not errs and all(p.exitcode == 0 for p in procs), errs


def test_balanced_placement():
    """Greedy longest-load-first placement: E/P experts per rank, every expert placed once,
    the heaviest experts on different ranks, loads within one expert of even."""
    from fni8.parallel import balanced_placement, experts_of_rank

    load = torch.tensor([100, 90, 80, 5, 5, 5, 5, 5, 1, 1, 1, 1, 0, 0, 0, 0])
    for P in (1, 2, 4, 8):
        place = balanced_placement(load, P)
        per = 16 // P
        ranks = [experts_of_rank(place, P, r) for r in range(P)]
        assert sorted(e for ids in ranks for e in ids) == list(range(16))
        tot = [int(load[ids].sum()) for ids in ranks]
        assert max(tot) - min(tot) <= int(load.max()), (P, tot)
        if P >= 3:
            assert len({int(place[e]) // per for e in (0, 1, 2)}) == 3
    with pytest.raises(ValueError):
        balanced_placement(load, 3)


def test_peer_exchange_cleans_up_a_failed_mapping():
    _spawn(_ipc_fail_worker, 3)


@pytest.mark.parametrize("worker", [_ep_worker, _cp_worker], ids=["expert_parallel", "column_parallel"])
def test_two_gloo_ranks(worker):
    _spawn(worker, 2)


def test_exchange_helpers_single_rank():
    from fni8.parallel import expert_shard, segments_from_counts

    assert expert_shard(128, 8, 3) == (48, 64)
    with pytest.raises(ValueError):
        expert_shard(10, 4, 0)
    exp, off, cnt = segments_from_counts(torch.tensor([[2, 0, 5], [1, 3, 0]]))
    assert exp.tolist() == [0, 1, 2, 0, 1, 2] and off.tolist() == [0, 2, 2, 7, 8, 11] and cnt.tolist() == [2, 0, 5, 1, 3, 0]


def test_p2p_placement_matches_a_sequential_layout():
    """The device-side placement of the peer-memory exchange (parallel.p2p_placement) against
    a plain walk over (owner, local expert, source) in buffer order."""
    from fni8.parallel import p2p_placement

    g = torch.Generator().manual_seed(11)
    for world, E in ((2, 8), (4, 16), (8, 128)):
        El = E // world
        cnt = torch.randint(0, 40, (world, E), generator=g, dtype=torch.int32)
        cnt[0, :El] = 0  # empty experts
        # reference: rank d's buffer lists its local experts in order, each by source rank
        start = {}
        for d in range(world):
            pos = 0
            for el in range(El):
                for s_ in range(world):
                    start[(s_, d, el)] = pos
                    pos += int(cnt[s_, d * El + el])
        for rank in range(world):
            dst_base, seg_off, seg_cnt, n_recv = p2p_placement(cnt, rank, world)
            for d in range(world):
                for el in range(El):
                    assert int(dst_base[d, el]) == start[(rank, d, el)]
            for el in range(El):
                assert int(seg_off[el]) == start[(0, rank, el)]
                assert int(seg_cnt[el]) == int(cnt[:, rank * El + el].sum())
            assert int(n_recv[0]) == int(cnt[:, rank * El:(rank + 1) * El].sum())
