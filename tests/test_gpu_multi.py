"""The multi-GPU forms on 2 GPUs over NCCL (skipped with fewer than 2 GPUs).

The expert-parallel MoE layer and the column-parallel linear run the sm_100a kernels
on each rank and exchange over NCCL; each rank checks its result against the
single-GPU kernels on the unsharded weights, bit for bit (every row's int32 sums and
its dequant epilogue do not depend on how the rows or columns were grouped).
"""
import ctypes
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))


def _ep_worker(rank, world, port, errq):
    try:
        _init(rank, world, port)
        import fni8.moe as moe
        from fni8 import QTensor
        from fni8.moe import ExpertStack
        from fni8.parallel import ExpertParallelMoE, balanced_placement, expert_shard, experts_of_rank
        from fni8.quant.core import quantize_int8_rowwise

        dev = torch.device("cuda", rank)
        E, k, H, I = 16, 4, 512, 256
        T = 300 + 77 * rank  # ragged: the ranks hold different token counts
        g = torch.Generator(device=dev).manual_seed(5)
        gu = [quantize_int8_rowwise(0.05 * torch.randn(2 * I, H, generator=g, device=dev)) for _ in range(E)]
        dn = [quantize_int8_rowwise(0.05 * torch.randn(H, I, generator=g, device=dev)) for _ in range(E)]
        w_gu = torch.stack([q for q, _ in gu])
        s_gu = torch.stack([s.view(-1) for _, s in gu])
        w_dn = torch.stack([q for q, _ in dn])
        s_dn = torch.stack([s.view(-1) for _, s in dn])
        lo, hi = expert_shard(E, world, rank)
        local = ExpertStack(w_gu[lo:hi].contiguous(), s_gu[lo:hi].contiguous(), w_dn[lo:hi].contiguous(),
                            s_dn[lo:hi].contiguous())
        full = ExpertStack(w_gu, s_gu, w_dn, s_dn)
        gx = torch.Generator(device=dev).manual_seed(100 + rank)
        x = torch.randn(T, H, generator=gx, device=dev).half()
        bias = torch.zeros(E, device=dev)
        bias[0] = 3.0  # skew: expert 0 (rank 0) is popular
        topi, topw = moe.route(torch.randn(T, E, generator=gx, device=dev) + bias, k)
        ref = moe.experts(x, topi, topw, full)
        # peer-memory exchange (the default on NCCL) and the all_to_all exchange
        # load-balanced placement: rank r holds the experts balanced_placement gives it
        load = torch.bincount(topi.reshape(-1).long(), minlength=E)
        dist.all_reduce(load)
        place = balanced_placement(load.cpu(), world)
        ids = experts_of_rank(place, world, rank)
        placed = ExpertStack(w_gu[ids].contiguous(), s_gu[ids].contiguous(), w_dn[ids].contiguous(),
                             s_dn[ids].contiguous())
        epb = ExpertParallelMoE(placed, E, placement=place)
        got = epb(x, topi, topw)
        torch.cuda.synchronize()
        assert torch.equal(got, ref), ("placed", (got.float() - ref.float()).abs().max().item())
        epb.close()
        # bf16 activations through the same exchange (fused return of bf16 rows)
        xb = x.to(torch.bfloat16)
        epf = ExpertParallelMoE(placed, E, placement=place)
        got = epf(xb, topi, topw)
        refb = moe.experts(xb, topi, topw, full)
        torch.cuda.synchronize()
        assert got.dtype == torch.bfloat16 and torch.equal(got, refb), ("bf16", (got.float() - refb.float()).abs().max().item())
        epf.close()
        for transport, fuse in (("p2p", True), ("p2p", False), ("nccl", False)):
            ep = ExpertParallelMoE(local, E, transport=transport, fuse_return=fuse)
            assert ep.transport == transport
            got = ep(x, topi, topw)
            torch.cuda.synchronize()
            assert torch.equal(got, ref), (transport, fuse, (got.float() - ref.float()).abs().max().item())
            # a rank with no tokens still takes every collective step
            got0 = ep(x[:0], topi[:0], topw[:0]) if rank == 1 else ep(x, topi, topw)
            assert got0.shape[0] == (0 if rank == 1 else T)
            if transport == "p2p":
                # nothing visits the host: the layer replays from a CUDA graph
                st = torch.cuda.Stream()
                st.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(st):
                    ep(x, topi, topw)
                torch.cuda.current_stream().wait_stream(st)
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    out = ep(x, topi, topw)
                graph.replay()
                torch.cuda.synchronize()
                assert torch.equal(out, ref), ("graph", (out.float() - ref.float()).abs().max().item())
                del graph, out
                code = ctypes.c_int(0)
                from fni8 import _native as nat
                nat.call("fni8_device_status", ctypes.byref(code))  # no capacity overflow recorded
                ep.close()
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report to the parent, which fails the test
        errq.put(f"rank {rank}: {e!r}")
        raise


def _cp_worker(rank, world, port, errq):
    try:
        _init(rank, world, port)
        import fni8
        from fni8 import QTensor
        from fni8.parallel import ColumnParallelLinearW8A8, shard_rows
        from fni8.quant.core import quantize_int8_rowwise

        dev = torch.device("cuda", rank)
        K, N = 1024, 2048
        g = torch.Generator(device=dev).manual_seed(3)
        q, s = quantize_int8_rowwise(0.02 * torch.randn(N, K, generator=g, device=dev))
        full = QTensor(q, s.view(-1))
        shard = shard_rows(full, world, rank)
        cp = ColumnParallelLinearW8A8(shard, max_rows=300)  # p2p: all-gather from the GEMM over NVLink
        assert cp.transport == "p2p"
        cpn = ColumnParallelLinearW8A8(shard, transport="nccl")
        cpc = ColumnParallelLinearW8A8(shard, transport="nccl", chunk_rows=128)  # 300 rows: 3 chunks
        outs = []
        bias = (0.1 * torch.randn(N, generator=g, device=dev)).half()
        bshard = bias.view(world, N // world)[rank].contiguous()
        for M in (1, 16, 300):  # split-K + copy kernel, and the tile GEMM with the stores in its epilogue
            x = torch.randn(M, K, generator=g, device=dev).half()
            ref = fni8.linear(x, full)
            for layer in (cp, cpn, cpc):
                got = layer(x)
                assert torch.equal(got, ref), (M, layer.transport, (got.float() - ref.float()).abs().max().item())
            outs.append((cp(x, copy=True), ref))
            got = cp(x, bias=bshard)  # each rank's bias slice, applied in its epilogue
            assert torch.equal(got, fni8.linear(x, full, bias)), ("bias", M)
        for got, ref in outs:  # copies stay valid after later calls reuse the ring
            assert torch.equal(got, ref)
        # no host synchronisation: the p2p layer replays from a CUDA graph
        x = torch.randn(300, K, generator=g, device=dev).half()
        ref = fni8.linear(x, full)
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            cp(x)
        torch.cuda.current_stream().wait_stream(st)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = cp(x)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
        del graph, out
        cp.close()
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        errq.put(f"rank {rank}: {e!r}")
        raise


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("worker", [_ep_worker, _cp_worker], ids=["expert_parallel", "column_parallel"])
def test_two_nccl_ranks(worker):
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=worker, args=(r, 2, port, errq)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    for p in procs:
        if p.is_alive():
            p.kill()
            errs.append("rank timed out")
    assert not errs and all(p.exitcode == 0 for p in procs), errs
