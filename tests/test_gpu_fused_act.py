"""gate_up GEMM with act_and_mul in its epilogue (fni8serve/layers/mlp.py:39-40).

The fused tile kernel dequantises the gate and up accumulators exactly as the plain
epilogue stores them and forms act(gate) * up exactly as the act_and_mul kernels do, so
its [M, I] product must equal fni8_gemm_w8a8 -> fni8_act_and_mul bit for bit (dense and
grouped, fp16 and bf16, SiLU and tanh-GELU, ragged row counts). Against the CPU oracle the
product is held to the act_and_mul rule (one ulp: CUDA expf/tanhf vs torch), and the down
projection of the drop-in GatedMLP is bit-exact given the GPU's product.
"""
import pytest
import torch

from oracle import w8a8_oracle as O

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a B200")]

DEV = "cuda"


def gen(seed):
    return torch.Generator().manual_seed(seed)


def qweight(N, K, seed, scale=0.02):
    return O.quantize_weight_rowwise(scale * torch.randn(N, K, generator=gen(seed)))


def ulp_close(a, b, ulps=1, dtype=torch.float16):
    a, b = a.float().cpu(), b.float().cpu()
    eps = 2.0 ** -10 if dtype == torch.float16 else 2.0 ** -7
    ulp = torch.maximum(b.abs(), torch.full_like(b, 6.1e-5)) * eps
    return bool(((a - b).abs() <= ulps * ulp * 1.01).all())


@pytest.mark.parametrize("M,I,K", [(1, 128, 256), (200, 768, 2048), (256, 1408, 1024), (777, 384, 512),
                                   (2048, 12288, 4096)])
@pytest.mark.parametrize("act", ["silu", "gelu_tanh"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_dense_gate_up_act_equals_unfused(M, I, K, act, dtype):
    import fni8

    if I == 12288 and (act != "silu" or dtype != torch.float16):
        pytest.skip("the Qwen3-8B shape runs once")
    wq, ws = qweight(2 * I, K, I + K, scale=0.2)
    qt = fni8.QTensor(wq.to(DEV), ws.to(DEV))
    g = gen(M + I)
    a = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8)
    s = torch.rand(M, generator=g) * 0.02 + 1e-3
    got = fni8.linear_act_q(a.to(DEV), s.to(DEV), qt, act, out_dtype=dtype)
    h = fni8.linear_q(a.to(DEV), s.to(DEV), qt, out_dtype=dtype)
    ref = fni8.act_and_mul(h, act)
    assert torch.equal(got, ref)
    h_cpu = O.dequant(O.int_mm_fast(a, wq), s, ws, out_dtype=dtype)
    assert torch.equal(h.cpu(), h_cpu)
    assert ulp_close(got, O.act_and_mul(h_cpu, act), dtype=dtype) if act == "silu" else \
        torch.allclose(got.float().cpu(), O.act_and_mul(h_cpu, act).float(), rtol=2e-3, atol=2e-4)
    assert fni8.device_status() == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_grouped_gate_up_act_equals_unfused(dtype):
    import fni8
    import fni8.moe as M

    E, I, K = 12, 768, 512
    cnt = torch.tensor([0, 1, 130, 127, 128, 5, 0, 300, 17, 256, 3, 64], dtype=torch.int32)
    off = torch.zeros(E, dtype=torch.int32)
    off[1:] = torch.cumsum(cnt, 0)[:-1]
    R = int(cnt.sum())
    a = torch.randint(-127, 128, (R, K), generator=gen(10), dtype=torch.int8)
    s = torch.rand(R, generator=gen(13)) * 0.02 + 1e-3
    w = torch.stack([qweight(2 * I, K, 50 + e, scale=0.2)[0] for e in range(E)])
    sw = torch.stack([qweight(2 * I, K, 50 + e, scale=0.2)[1] for e in range(E)])
    perm = torch.randperm(E, generator=gen(12)).int()  # segment s uses expert perm[s]
    args = (a.to(DEV), s.to(DEV), w.to(DEV), sw.to(DEV), perm.to(DEV), off.to(DEV), cnt.to(DEV))
    got = M.grouped_gemm_act(*args, act="silu", out_dtype=dtype)
    h = M.grouped_gemm(*args, out_dtype=dtype)
    ref = fni8.act_and_mul(h, "silu")
    for sg in range(E):
        o, c = int(off[sg]), int(cnt[sg])
        if c:
            assert torch.equal(got[o:o + c], ref[o:o + c]), sg
    assert fni8.device_status() == 0


@pytest.mark.parametrize("M", [8, 300, 1024])
def test_gated_mlp_dropin(M):
    """fni8.mlp.GatedMLP (the constructor of fni8serve/layers/mlp.py:22-36): the fused path
    (M >= 257) equals the composed fni8 calls bit for bit, and its down projection equals
    the oracle's given the GPU's product."""
    import fni8
    from fni8.mlp import GatedMLP

    H, I = 1024, 768
    gu_q, gu_s = qweight(2 * I, H, 1)
    dn_q, dn_s = qweight(H, I, 2)
    mlp = GatedMLP(fni8.QTensor(gu_q.to(DEV), gu_s.to(DEV)), fni8.QTensor(dn_q.to(DEV), dn_s.to(DEV)), act="silu")
    x = torch.randn(M, H, generator=gen(M)).half()
    y = mlp(x.to(DEV))
    composed = fni8.linear(fni8.act_and_mul(fni8.linear(x.to(DEV), mlp.gate_up)), mlp.down)
    assert torch.equal(y, composed)
    q, s = fni8.quantize_rows(x.to(DEV))
    prod = fni8.linear_act_q(q, s, mlp.gate_up).cpu()
    hq, hs = O.quantize_rows(prod)
    assert torch.equal(y.cpu(), O.dequant(O.int_mm_fast(hq, dn_q), hs, dn_s))
    assert fni8.device_status() == 0


def test_act_gemm_rejects_unsupported_shapes():
    import fni8
    from fni8 import Fni8Error

    qt = fni8.QTensor(torch.zeros(2 * 96, 64, dtype=torch.int8, device=DEV), torch.ones(2 * 96, device=DEV))
    with pytest.raises(Fni8Error, match="multiple of 128"):
        fni8.linear_act_q(torch.zeros(4, 64, dtype=torch.int8, device=DEV), torch.ones(4, device=DEV), qt)


@pytest.mark.parametrize("T,k,H", [(4096, 8, 2048), (37, 4, 512), (5, 2, 4096)])
def test_quantize_scatter_equals_quantize_then_gather(T, k, H):
    """fni8_moe_quantize_scatter_i8 (quantise each token once, write its codes to the
    expert-grouped rows of its slots) equals quantize_rows followed by the row gather, and
    the oracle; slots the plan dropped (expert id out of range) get no row."""
    import fni8
    import fni8.moe as M
    from fni8.parallel import gather_rows

    E = 16
    x = torch.randn(T, H, generator=gen(T)).half()
    topi = torch.randint(0, E, (T, k), generator=gen(T + 1), dtype=torch.int32)
    topi[0, 0] = E + 3  # dropped by the plan
    counts, offsets, ros, sor = M.plan(topi.to(DEV), E)
    n = int(offsets[-1].item())
    got_q, got_s = M.quantize_scatter(x.to(DEV), ros, k, n)
    xq, xs = fni8.quantize_rows(x.to(DEV))
    ref_q, ref_s = gather_rows(xq, xs, sor, n, k)
    assert torch.equal(got_q, ref_q) and torch.equal(got_s, ref_s)
    oq, os_ = O.quantize_rows(x)
    tok = sor[:n].long().cpu() // k
    assert torch.equal(got_q.cpu(), oq[tok]) and torch.equal(got_s.cpu(), os_[tok])


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_silu_over_every_16bit_value(dtype):
    """act(g) for every finite 16-bit g (up = 1): within one ulp of torch's silu on CPU, and
    equal on at least 99.9 % of the values (the fp32 quotient is formed with a refined
    reciprocal; only values within ~2 fp32 ulps of a 16-bit rounding boundary may round the
    other way)."""
    import fni8

    bits = torch.arange(-32768, 32768, dtype=torch.int32).to(torch.int16)
    g = bits.view(dtype)
    g = g[torch.isfinite(g.float())]
    x = torch.cat([g[:, None], torch.ones_like(g)[:, None]], dim=1)  # [n, 2]: gate | up
    got = fni8.act_and_mul(x.to(DEV), "silu").cpu().flatten()
    ref = torch.nn.functional.silu(g.float()).to(dtype)
    eps = 2.0 ** -10 if dtype == torch.float16 else 2.0 ** -7
    tiny = 6.1e-5 if dtype == torch.float16 else 1.2e-38
    ulp = torch.maximum(ref.float().abs(), torch.full_like(ref.float(), tiny)) * eps
    assert bool(((got.float() - ref.float()).abs() <= ulp * 1.01).all())
    assert (got == ref).float().mean() > 0.999
