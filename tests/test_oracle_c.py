"""The plain-C restatement of the integer path (oracle/w8a8_ref.c) against the reference's
own fixtures and against the torch oracle, bit for bit (CPU only).

Two independent statements of the same arithmetic: the torch oracle (which the GPU parity
tests compare the kernels with) and a scalar C loop nest with the IEEE conversions and
the fp32 operation order written out. Where they agree on every input below, the oracle's
result does not depend on how torch evaluates it.
"""
import numpy as np
import pytest
import torch

from oracle import c_oracle as C
from oracle import w8a8_oracle as O


def t(a):
    return torch.from_numpy(np.ascontiguousarray(a))


def gen(seed):
    return torch.Generator().manual_seed(seed)


def activations(M, K, seed, dtype):
    """N(0,1) tokens with a few outlier channels x20, a zero row and an extreme row."""
    g = gen(seed)
    x = torch.randn(M, K, generator=g)
    ch = torch.randperm(K, generator=g)[: max(1, K // 1000)]
    x[:, ch] *= 20
    if M > 2:
        x[1] = 0
        x[2, 0] = 60000.0 if dtype == torch.float16 else 3e38
    return x.to(dtype)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_conversions_are_ieee(dtype):
    """Every fp16/bf16 bit pattern widens exactly as torch widens it, and fp32 values around
    every rounding boundary (ties, subnormals, overflow) narrow as torch narrows them."""
    bits = torch.arange(-32768, 32768, dtype=torch.int32).to(torch.int16).view(dtype)
    ref = bits.float()
    got = C.to_f32(bits)
    fin = torch.isfinite(ref)
    assert torch.equal(got[fin], ref[fin]) and torch.isnan(got[~fin]).eq(torch.isnan(ref[~fin])).all()
    g = gen(3)
    f = torch.cat([ref[fin], (ref[fin] * (1 + 2.0 ** -12)), torch.randn(200000, generator=g) * 1e4,
                   torch.randn(200000, generator=g) * 1e-6, torch.tensor([65519.99, 65520.0, 65536.0, -65520.0,
                                                                          2.0 ** -25, 3 * 2.0 ** -26, 1e-30, 0.0, -0.0])])
    assert torch.equal(C.from_f32(f, dtype).view(torch.int16), f.to(dtype).view(torch.int16))


def test_weight_quant_matches_reference_fixture(golden):
    """fni8-serve tests/test_smoke.py:14-18 (fp32 per-row absmax/127): codes and scales
    exactly as the reference computed them."""
    g = golden("i8_fixture")
    q, s = C.quantize_weight_rowwise(t(g["smoke_w"]))
    assert torch.equal(q, t(g["smoke_q"])) and torch.equal(s, t(g["smoke_s"]))
    qo, so = O.quantize_weight_rowwise(t(g["smoke_w"]))
    assert torch.equal(q, qo) and torch.equal(s, so)


@pytest.mark.parametrize("tag", ["smoke", "cfg0"])
def test_linear_on_reference_fixtures(golden, tag):
    """The reference fixtures' inputs (tests/golden/linear.npz): the C and torch oracles give
    identical int8 rows, scales, int32 sums and outputs, with and without bias."""
    g = golden("linear")
    x, wq, ws, bias = t(g[f"{tag}_x"]), t(g[f"{tag}_wq"]), t(g[f"{tag}_ws"]), t(g[f"{tag}_bias"])
    q, s = C.quantize_rows(x)
    qo, so = O.quantize_rows(x)
    assert torch.equal(q, qo) and torch.equal(s, so)
    assert torch.equal(C.gemm_i32(q, wq), O.int_mm_exact(qo, wq))
    for b in (None, bias):
        assert torch.equal(C.linear_w8a8(x, wq, ws, bias=b), O.linear_w8a8(x, wq, ws, bias=b))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M,K,N", [(1, 16, 8), (7, 40, 24), (33, 1024, 96), (5, 4096, 64)])
def test_linear_matches_torch_oracle(M, K, N, dtype):
    x = activations(M, K, M * 7 + K, dtype)
    wq, ws = O.quantize_weight_rowwise(0.02 * torch.randn(N, K, generator=gen(N)))
    bias = (0.1 * torch.randn(N, generator=gen(5))).to(dtype)
    res = torch.randn(M, N, generator=gen(6)).to(dtype)
    q, s = C.quantize_rows(x)
    qo, so = O.quantize_rows(x)
    assert torch.equal(q, qo) and torch.equal(s, so)
    if M > 2:
        assert s[1] == 0 and not q[1].any()  # a zero row: scale 0, codes 0
    acc = C.gemm_i32(q, wq)
    assert torch.equal(acc, O.int_mm_exact(q, wq))
    for b, r in ((None, None), (bias, None), (bias, res)):
        assert torch.equal(C.dequant(acc, s, ws, b, r, dtype), O.dequant(acc, s, ws, b, r, dtype))
    assert torch.equal(C.linear_w8a8(x, wq, ws, bias=bias), O.linear_w8a8(x, wq, ws, bias=bias))


def test_gemm_extremes_and_overflow():
    """Full-range codes at K = 131072 stay inside int32 (127 * 127 * K < 2^31); one more
    step outside it is reported, not wrapped silently."""
    K = 131072
    a = torch.full((2, K), 127, dtype=torch.int8)
    a[1] = -127
    w = torch.full((3, K), 127, dtype=torch.int8)
    w[2] = -127
    acc = C.gemm_i32(a, w)
    assert acc[0, 0] == 127 * 127 * K and acc[1, 0] == -127 * 127 * K and acc[1, 2] == 127 * 127 * K
    assert torch.equal(acc, O.int_mm_exact(a, w))
    with pytest.raises(OverflowError):
        C.gemm_i32(torch.full((1, 2 * K), 127, dtype=torch.int8), torch.full((1, 2 * K), 127, dtype=torch.int8))


def test_w4a8_on_reference_fixture(golden):
    """per_group_i4 / int4: the C unpack and fp16 fallback weight equal the reference's own
    reconstruction (fni8serve/layers/linear.py:33-45, tests/golden/linear_i4.npz) bit for
    bit, and the C and torch W4A8 linears agree bit for bit (same group order)."""
    g = golden("linear_i4")
    packed, scale, gs = t(g["packed"]), t(g["scale"]), int(g["group_size"])
    assert torch.equal(C.unpack_i4(packed), O.unpack_i4(packed))
    assert torch.equal(C.dequant_weight_i4_fallback(packed, scale, gs), t(g["w_ref"]))
    x, bias = t(g["x"]), t(g["bias"])
    for b in (None, bias):
        assert torch.equal(C.linear_w4a8(x, packed, scale, gs, bias=b), O.linear_w4a8(x, packed, scale, gs, bias=b))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_w4a8_matches_torch_oracle(dtype):
    N, K, gs = 48, 512, 128
    x = activations(9, K, 17, dtype)
    packed, scale = O.quantize_weight_i4(0.05 * torch.randn(N, K, generator=gen(18)), gs)
    codes = torch.randint(-8, 8, (N, K), generator=gen(19), dtype=torch.int8)  # every code, both nibbles
    for p in (packed, O.pack_i4(codes)):
        assert torch.equal(C.unpack_i4(p), O.unpack_i4(p))
        assert torch.equal(C.linear_w4a8(x, p, scale, gs), O.linear_w4a8(x, p, scale, gs))
    assert torch.equal(C.unpack_i4(O.pack_i4(codes)), codes)


@pytest.mark.parametrize("T,k,E", [(1, 1, 4), (37, 2, 8), (256, 8, 128), (5, 4, 3)])
def test_moe_plan_matches_torch_oracle(T, k, E):
    """Stable grouping of (token, slot) pairs by expert (index work: exact), including
    expert ids outside [0, E) (not grouped, row -1) and experts nobody chose."""
    g = gen(T * 31 + E)
    topi = torch.randint(-1, E + 1, (T, k), generator=g)
    topi[0, 0] = E - 1
    for got, ref in zip(C.moe_plan(topi, E), O.moe_plan(topi, E)):
        assert torch.equal(got, ref.long())


@pytest.mark.parametrize("scoring", ["softmax", "sigmoid"])
def test_moe_plan_on_reference_routing(golden, scoring):
    """The reference's own expert choices (tests/golden/moe_*.npz) grouped by both oracles."""
    g = golden(f"moe_{scoring}")
    topi, E = t(g["topi"]), int(g["E"])
    for got, ref in zip(C.moe_plan(topi, E), O.moe_plan(topi, E)):
        assert torch.equal(got, ref.long())


def test_moe_block_from_c_pieces_matches_torch_oracle(golden):
    """The routed-expert block assembled from the C pieces (row quantisation, plan, exact
    int32 GEMMs and dequant per expert, weighted combine) equals the torch oracle's
    moe_experts_w8a8 bit for bit on the reference fixture's routing; SiLU·mul (a libm
    transcendental) is the torch oracle's in both."""
    g = golden("moe_softmax")
    x, topi = t(g["x"]), t(g["topi"])
    H = x.shape[-1]
    xf = x.reshape(-1, H)
    k, E = topi.shape[-1], int(g["E"])
    w_gu, s_gu, w_dn, s_dn = t(g["w_gu"]), t(g["s_gu"]), t(g["w_dn"]), t(g["s_dn"])
    topw = torch.rand(topi.shape, generator=gen(9))
    counts, offsets, ros, sor = C.moe_plan(topi, E)
    xq, xs = C.quantize_rows(xf)
    tok = sor // k
    y = torch.empty(sor.numel(), H, dtype=x.dtype)
    for e in range(E):
        r0, r1 = int(offsets[e]), int(offsets[e + 1])
        if r0 == r1:
            continue
        rows = tok[r0:r1]
        h = C.dequant(C.gemm_i32(xq[rows], w_gu[e]), xs[rows], s_gu[e], out_dtype=x.dtype)
        hq, hs = C.quantize_rows(O.act_and_mul(h))
        y[r0:r1] = C.dequant(C.gemm_i32(hq, w_dn[e]), hs, s_dn[e], out_dtype=x.dtype)
    got = C.moe_combine(y, ros.view(topi.shape), topw)
    assert torch.equal(got, O.moe_experts_w8a8(xf, topi, topw, w_gu, s_gu, w_dn, s_dn))
