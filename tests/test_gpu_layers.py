"""fni8-serve's layer contracts on the sm_100a path: the fused RMSNorm -> int8 hand-off,
CUDA-graph capture of the decode-path ops, and the grouped MoE pipeline against the
oracle and against the reference SparseMoE's own outputs (tests/golden/moe_*.npz)."""
import pytest
import torch
import torch.nn.functional as F

from oracle import w8a8_oracle as O

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a B200")]

DEV = "cuda"


def gen(seed):
    return torch.Generator().manual_seed(seed)


def qweight(N, K, seed):
    return O.quantize_weight_rowwise(0.02 * torch.randn(N, K, generator=gen(seed)))


def test_norm_to_linear_sidecar_is_invisible():
    """fni8.rmsnorm leaves int8 rows on its output; fni8.linear consumes them instead of
    re-quantising. Results must equal the unfused chain exactly, and the side-car must be
    ignored once the tensor is modified in place."""
    import fni8

    M, K, N = 64, 4096, 1024
    g = gen(1)
    x = torch.randn(M, K, generator=g).half().to(DEV)
    r = torch.randn(M, K, generator=g).half().to(DEV)
    w = (1 + 0.1 * torch.randn(K, generator=g)).half().to(DEV)
    wq, ws = qweight(N, K, 2)
    qt = fni8.QTensor(wq.to(DEV), ws.to(DEV))
    h, _ = fni8.rmsnorm(x, w, 1e-6, residual=r)
    assert getattr(h, "_fni8_q", None) is not None
    fused = fni8.linear(h, qt)
    plain = fni8.linear(h.clone(), qt)  # clone drops the side-car
    assert torch.equal(fused, plain)
    h.mul_(2)  # bumps the version counter: side-car must not be used
    assert torch.equal(fni8.linear(h, qt), fni8.linear(h.clone(), qt))


@pytest.mark.parametrize("shape", [(2, 33, 4096), (48, 4096)])
@pytest.mark.parametrize("act", ["silu", "gelu_tanh"])
def test_act_to_down_sidecar_is_invisible(shape, act):
    """fni8.act_and_mul writes the product and its int8 rows in one pass; the down
    projection consumes the rows. The product equals the unfused kernel's, the down
    output equals the unfused chain's exactly (3-D inputs keep their leading dims), and a
    modified product is re-quantised."""
    import fni8
    from fni8 import ops

    *lead, two_i = shape
    I, N = two_i // 2, 640
    x = torch.randn(*lead, two_i, generator=gen(3)).half().to(DEV)
    wq, ws = qweight(N, I, 4)
    qt = fni8.QTensor(wq.to(DEV), ws.to(DEV))
    h = fni8.act_and_mul(x, act)
    assert getattr(h, "_fni8_q", None) is not None
    ops.FUSE_ACT_QUANT = False
    try:
        h_plain = fni8.act_and_mul(x, act)
    finally:
        ops.FUSE_ACT_QUANT = True
    assert getattr(h_plain, "_fni8_q", None) is None
    assert torch.equal(h, h_plain)
    fused = fni8.linear(h, qt)
    assert fused.shape == (*lead, N)
    assert torch.equal(fused, fni8.linear(h_plain, qt))
    h.add_(1)
    assert torch.equal(fni8.linear(h, qt), fni8.linear(h.clone(), qt))


def test_norm_to_linear_sidecar_keeps_leading_dims():
    import fni8

    B, S, K, N = 2, 17, 1024, 384
    x = torch.randn(B, S, K, generator=gen(5)).half().to(DEV)
    w = torch.ones(K, dtype=torch.float16, device=DEV)
    wq, ws = qweight(N, K, 6)
    qt = fni8.QTensor(wq.to(DEV), ws.to(DEV))
    h = fni8.rmsnorm(x, w, 1e-6)
    y = fni8.linear(h, qt)
    assert y.shape == (B, S, N) and torch.equal(y, fni8.linear(h.clone(), qt))


def test_decode_ops_capture_in_cuda_graph():
    """The reference engine captures decode in a CUDA graph (engine/cuda_graph.py); the
    ops must be capturable (no host sync, no allocation outside the caching allocator)."""
    import fni8

    K, N = 4096, 6144
    wq, ws = qweight(N, K, 3)
    qt = fni8.QTensor(wq.to(DEV), ws.to(DEV))
    w = torch.ones(K, dtype=torch.float16, device=DEV)
    static_x = torch.randn(8, K, generator=gen(4)).half().to(DEV)
    fni8.linear(fni8.rmsnorm(static_x, w, 1e-6), qt)  # warm-up: workspace allocated outside capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        static_y = fni8.linear(fni8.act_and_mul(torch.cat([static_x, static_x], -1)), qt)
    for seed in (5, 6):
        static_x.copy_(torch.randn(8, K, generator=gen(seed)).half())
        graph.replay()
        torch.cuda.synchronize()
        ref = fni8.linear(fni8.act_and_mul(torch.cat([static_x, static_x], -1)), qt)
        assert torch.equal(static_y, ref)


# ------------------------------------------------------------------ MoE
def _experts(E, H, I, seed):
    g = gen(seed)
    w_gu = torch.stack([qweight(2 * I, H, 100 * seed + e)[0] for e in range(E)])
    s_gu = torch.stack([qweight(2 * I, H, 100 * seed + e)[1] for e in range(E)])
    w_dn = torch.stack([qweight(H, I, 100 * seed + 50 + e)[0] for e in range(E)])
    s_dn = torch.stack([qweight(H, I, 100 * seed + 50 + e)[1] for e in range(E)])
    del g
    return w_gu, s_gu, w_dn, s_dn


@pytest.mark.parametrize("scoring", ["softmax", "sigmoid"])
def test_route_matches_oracle(scoring):
    import fni8.moe as M

    T, E, k = 300, 128, 8
    logits = torch.randn(T, E, generator=gen(7))
    kw, okw = {}, {}
    if scoring == "sigmoid":
        b = 0.1 * torch.randn(E, generator=gen(8))
        kw = dict(sel_bias=b.to(DEV), num_expert_groups=8, topk_group=4)
        okw = dict(sel_bias=b, n_groups=8, topk_group=4)
    topi, topw = M.route(logits.to(DEV), k, scoring=scoring, **kw)
    ti, tw = O.moe_route(logits, k, scoring=scoring, **okw)
    assert torch.equal(topi.cpu().long(), ti)
    torch.testing.assert_close(topw.cpu(), tw.float(), rtol=2e-3, atol=1e-6)


def test_plan_matches_oracle():
    import fni8.moe as M

    T, k, E = 4096, 8, 128
    topi = torch.randint(0, E, (T, k), generator=gen(9), dtype=torch.int32)
    topi[3, 2] = E + 4  # out-of-range id: dropped
    counts, offsets, ros, sor = M.plan(topi.to(DEV), E)
    c, o, r, s = O.moe_plan(topi, E)
    assert torch.equal(counts.cpu().long(), c) and torch.equal(offsets.cpu().long(), o)
    assert torch.equal(ros.cpu().long(), r) and torch.equal(sor.cpu()[: int(o[-1])].long(), s)


def test_grouped_gemm_int32_exact():
    import fni8.moe as M

    E, N, K = 12, 768, 512
    cnt = torch.tensor([0, 1, 130, 127, 128, 5, 0, 300, 17, 256, 3, 64], dtype=torch.int32)
    off = torch.zeros(E, dtype=torch.int32)
    off[1:] = torch.cumsum(cnt, 0)[:-1]
    R = int(cnt.sum())
    a = torch.randint(-127, 128, (R, K), generator=gen(10), dtype=torch.int8)
    w = torch.randint(-127, 128, (E, N, K), generator=gen(11), dtype=torch.int8)
    perm = torch.randperm(E, generator=gen(12)).int()  # segment s uses expert perm[s]
    got = M.grouped_gemm(a.to(DEV), torch.ones(R, device=DEV), w.to(DEV), torch.ones(E, N, device=DEV),
                         perm.to(DEV), off.to(DEV), cnt.to(DEV), out_dtype=torch.int32).cpu()
    for s in range(E):
        o, c = int(off[s]), int(cnt[s])
        if c:
            assert torch.equal(got[o:o + c], O.int_mm_fast(a[o:o + c], w[int(perm[s])])), s


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_ep_placement_kernel_matches_restatement(world):
    """The exchange placement kernel (fni8_ep_placement) equals parallel.p2p_placement, the
    torch restatement the CPU tests pin, for every rank; the expert-id map kernel
    (fni8_moe_map_ids) equals indexing, ids outside [0, E) passing through."""
    import ctypes

    from fni8 import _native as nat
    from fni8.parallel import ep_placement, p2p_placement

    E = 128
    cnt = torch.randint(0, 300, (world, E), generator=gen(40), dtype=torch.int32)
    cnt[0, 5] = 0
    for rank in range(world):
        want = p2p_placement(cnt, rank, world)
        got = ep_placement(cnt.to(DEV), rank, world)
        for w, g in zip(want, got):
            assert torch.equal(w.reshape(-1).int(), g.cpu().reshape(-1)), rank
    ids = torch.randint(-2, E + 3, (4096, 8), generator=gen(41), dtype=torch.int32)
    perm = torch.randperm(E, generator=gen(42)).int()
    ids_d, perm_d = ids.to(DEV), perm.to(DEV)
    out = torch.empty_like(ids_d)
    nat.call("fni8_moe_map_ids", ctypes.c_void_p(ids_d.data_ptr()), ids.numel(), ctypes.c_void_p(perm_d.data_ptr()),
             E, ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    ok = (ids >= 0) & (ids < E)
    assert torch.equal(out.cpu(), torch.where(ok, perm[ids.clamp(0, E - 1).long()], ids))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_grouped_gemm_row_scatter(dtype):
    """The scatter epilogue (expert-parallel return fused into the down projection): every
    output row lands in row (tag & 0xFFFFFF) of buffer tag >> 24 and equals the plain grouped
    GEMM's row bit for bit; no other row of the buffers is written. Two local buffers stand
    in for two ranks' back buffers; segments of 0, 1 and ragged row counts."""
    import ctypes

    import fni8.moe as M
    from fni8.parallel import grouped_gemm_scatter

    E, N, K = 6, 2048, 768
    cnt = torch.tensor([40, 0, 130, 1, 300, 57], dtype=torch.int32)
    off = torch.zeros(E, dtype=torch.int32)
    off[1:] = torch.cumsum(cnt, 0)[:-1]
    R = int(cnt.sum())
    a = torch.randint(-127, 128, (R, K), generator=gen(20), dtype=torch.int8).to(DEV)
    a_s = (torch.rand(R, generator=gen(21)) * 1e-2).to(DEV)
    w = torch.randint(-127, 128, (E, N, K), generator=gen(22), dtype=torch.int8).to(DEV)
    w_s = (torch.rand(E, N, generator=gen(23)) * 1e-2).to(DEV)
    seg = torch.arange(E, dtype=torch.int32).to(DEV)
    ref = M.grouped_gemm(a, a_s, w, w_s, seg, off.to(DEV), cnt.to(DEV), out_dtype=dtype)
    rows = 400  # per buffer
    dest = torch.randint(0, 2, (R,), generator=gen(24))
    slot = torch.empty(R, dtype=torch.int64)
    for b in range(2):  # distinct slots within each buffer
        idx = (dest == b).nonzero().flatten()
        slot[idx] = torch.randperm(rows, generator=gen(25 + b))[: idx.numel()]
    tag = ((dest << 24) | slot).to(torch.int32).to(DEV)
    bufs = [torch.full((rows, N), -7.0, dtype=dtype, device=DEV) for _ in range(2)]
    peers = (ctypes.c_void_p * 2)(*[b.data_ptr() for b in bufs])
    grouped_gemm_scatter(a, a_s, w, w_s, seg, off.to(DEV), cnt.to(DEV), tag, ctypes.cast(peers, ctypes.c_void_p), 2,
                         rows, out_dtype=dtype)
    torch.cuda.synchronize()
    got_all = torch.stack([bufs[int(dest[r])][int(slot[r])] for r in range(R)])
    assert torch.equal(got_all, ref)
    for b in range(2):
        unused = torch.ones(rows, dtype=torch.bool)
        unused[slot[dest == b]] = False
        assert bool((bufs[b][unused.to(DEV)] == -7.0).all())


@pytest.mark.parametrize("M,P", [(1, 3), (40, 3), (256, 3), (300, 3), (1000, 3), (1000, 6), (4100, 8)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_linear_peer_cols_all_gather(M, P, dtype):
    """The column all-gather GEMM (fni8_gemm_w8a8_peer_cols): a shard's outputs land at its
    column offset in every destination buffer, bit-exact against the plain GEMM, and nothing
    outside those columns and rows is written. Three local buffers stand in for three ranks'
    output buffers (six and eight for the narrower tile bands used beyond four ranks); the
    sizes cover the split-K + copy path (M <= 256) and the tile GEMM with the stores in its
    epilogue (CTA pairs from 256 rows, a partial last tile at 300/1000/4100)."""
    import ctypes

    import fni8
    from fni8 import QTensor
    from fni8.ops import linear_q_peer_cols

    K, n, rank = 1024, 768, 1
    Nt, rows = P * n, M + 5
    x = (torch.randn(M, K, generator=gen(30)) * 2).to(dtype).to(DEV)
    w = torch.randint(-127, 128, (n, K), generator=gen(31), dtype=torch.int8).to(DEV)
    ws = (torch.rand(n, generator=gen(32)) * 1e-3).to(DEV)
    bias = (torch.randn(n, generator=gen(33)) * 0.1).to(dtype).to(DEV)
    shard = QTensor(w, ws)
    q, s = fni8.quantize_rows(x)
    ref = fni8.linear_q(q, s, shard, bias=bias, out_dtype=dtype)
    sentinel = torch.tensor(-7.0, dtype=dtype)
    bufs = [torch.full((rows, Nt), -7.0, dtype=dtype, device=DEV) for _ in range(P)]
    peers = (ctypes.c_void_p * P)(*[b.data_ptr() for b in bufs])
    linear_q_peer_cols(q, s, shard, ctypes.cast(peers, ctypes.c_void_p), P, Nt, rank * n, bias=bias, out_dtype=dtype)
    torch.cuda.synchronize()
    for b in bufs:
        got = b.cpu()
        assert torch.equal(got[:M, rank * n:(rank + 1) * n], ref.cpu())
        untouched = torch.ones(rows, Nt, dtype=torch.bool)
        untouched[:M, rank * n:(rank + 1) * n] = False
        assert bool((got[untouched] == sentinel).all())


def test_linear_peer_cols_rejects_bad_layouts():
    """Host-side checks of the all-gather GEMM: columns past ld, misaligned column offset,
    a shard width that is not a multiple of 64."""
    import ctypes

    import fni8
    from fni8 import QTensor
    from fni8.ops import linear_q_peer_cols

    K, n = 256, 64
    q, s = fni8.quantize_rows(torch.randn(4, K, device=DEV).half())
    buf = torch.zeros(4, 4 * n, dtype=torch.float16, device=DEV)
    peers = ctypes.cast((ctypes.c_void_p * 1)(buf.data_ptr()), ctypes.c_void_p)
    shard = QTensor(torch.zeros(n, K, dtype=torch.int8, device=DEV), torch.ones(n, device=DEV))
    with pytest.raises(fni8.Fni8Error):
        linear_q_peer_cols(q, s, shard, peers, 1, 4 * n, 3 * n + 8)  # past ld
    with pytest.raises(fni8.Fni8Error):
        linear_q_peer_cols(q, s, shard, peers, 1, 4 * n, 4)  # not a 16-byte column offset
    odd = QTensor(torch.zeros(48, K, dtype=torch.int8, device=DEV), torch.ones(48, device=DEV))
    with pytest.raises(fni8.Fni8Error):
        linear_q_peer_cols(q, s, odd, peers, 1, 4 * n, 0)


@pytest.mark.parametrize("scoring", ["softmax", "sigmoid"])
def test_sparse_moe_dropin_matches_reference_golden(golden, scoring):
    import fni8
    import fni8.moe as M

    g = golden(f"moe_{scoring}")
    E, k = int(g["E"]), int(g["k"])
    experts = [(fni8.QTensor(torch.from_numpy(g["w_gu"][e]), torch.from_numpy(g["s_gu"][e])),
                fni8.QTensor(torch.from_numpy(g["w_dn"][e]), torch.from_numpy(g["s_dn"][e]))) for e in range(E)]
    kw = {}
    if scoring == "sigmoid":
        kw = dict(scoring_func="sigmoid", e_score_correction_bias=torch.from_numpy(g["bias"]), num_expert_groups=2,
                  topk_group=1)
    moe = M.SparseMoE(gate=torch.from_numpy(g["gate"]), experts=experts, top_k=k, **kw).to(DEV)
    x = torch.from_numpy(g["x"]).to(DEV)
    y = moe(x).cpu()
    ref = torch.from_numpy(g["y"])
    cos = F.cosine_similarity(y.flatten().float(), ref.flatten().float(), dim=0).item()
    assert y.shape == ref.shape and cos >= 0.99, cos


def test_sparse_moe_shared_expert_matches_reference_golden(golden):
    """The drop-in SparseMoE with a gated shared expert and routed_scaling_factor
    (fni8serve/models/moe.py:95,107-112) against the reference block's output, and the
    oracle's routed + shared restatement (tests/golden/moe_shared.npz)."""
    import fni8
    import fni8.moe as M

    g = golden("moe_shared")
    E, k = int(g["E"]), int(g["k"])
    T = lambda a: torch.from_numpy(a)  # noqa: E731
    experts = [(fni8.QTensor(T(g["w_gu"][e]), T(g["s_gu"][e])), fni8.QTensor(T(g["w_dn"][e]), T(g["s_dn"][e])))
               for e in range(E)]
    shared = (fni8.QTensor(T(g["sh_gu_q"]), T(g["sh_gu_s"])), fni8.QTensor(T(g["sh_dn_q"]), T(g["sh_dn_s"])))
    moe = M.SparseMoE(gate=T(g["gate"]), experts=experts, top_k=k, shared_expert=shared,
                      shared_expert_gate=T(g["sgate"]), routed_scaling_factor=float(g["scaling"])).to(DEV)
    x = T(g["x"]).to(DEV)
    y = moe(x).cpu()
    ref = T(g["y"])
    cos = F.cosine_similarity(y.flatten().float(), ref.flatten().float(), dim=0).item()
    assert y.shape == ref.shape and cos >= 0.99, cos


def test_fni8_container_loads_to_the_gpu(tmp_path):
    """A .fni8 checkpoint (fni8.format) loads straight into the layout the kernels read:
    the linear on the loaded weight equals the linear on the original, bit for bit."""
    import fni8
    from fni8 import FQReader, save_fni8
    from fni8.quant.core import quantize_int8_rowwise

    N, K = 384, 512
    q, sc = quantize_int8_rowwise(0.02 * torch.randn(N, K, generator=gen(40)))
    qt = fni8.QTensor(q, sc.view(-1).float())
    path = str(tmp_path / "m.fni8")
    save_fni8(path, {"mlp.up.weight": qt}, meta={"arch": "qwen3"})
    with FQReader(path) as r:
        w = r.load_many(["mlp.up.weight"], "cuda")["mlp.up.weight"]
    assert w.data.is_cuda and w.scheme == "per_row_i8"
    x = torch.randn(8, K, generator=gen(41)).half().to(DEV)
    assert torch.equal(fni8.linear(x, w), fni8.linear(x, qt.cuda()))
