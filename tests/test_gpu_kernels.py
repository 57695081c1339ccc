"""Parity of the sm_100a kernels with the CPU oracle, through the C ABI.

Integer and index results (int8 quantisation, int32 accumulators, the dequant epilogue
given identical inputs, MoE grouping) must be bit-exact. Floating-point producers
whose reduction order differs from torch's CPU order (RMSNorm's sum of squares) or
whose transcendental differs from torch's (expf in SiLU/GELU) are held to one fp16 ulp.
"""
import os

import pytest
import torch

from oracle import w8a8_oracle as O

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a B200")]

DEV = "cuda"
PKG = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "fni8-serve_b200")


def gen(seed):
    return torch.Generator().manual_seed(seed)


def act_input(M, K, seed, dtype=torch.float16, outliers=True):
    """BASELINE config-0 style activations: N(0,1) with 0.1% of channels x20."""
    g = gen(seed)
    x = torch.randn(M, K, generator=g)
    if outliers and K >= 100:
        ch = torch.randperm(K, generator=g)[: max(1, K // 1000)]
        x[:, ch] *= 20
    return x.to(dtype)


def weight(N, K, seed):
    w = 0.02 * torch.randn(N, K, generator=gen(seed))
    return O.quantize_weight_rowwise(w)


def ulp_close(a, b, ulps=1):
    a, b = a.float().cpu(), b.float().cpu()
    ulp = torch.maximum(b.abs(), torch.full_like(b, 6.1e-5)) * 2.0 ** -10  # fp16 ulp, subnormals flat
    return bool(((a - b).abs() <= ulps * ulp * 1.01).all())


def act_close(got, ref, act):
    """SiLU: within one fp16 ulp, almost all exact (CUDA expf vs torch's exp only move
    the rounding of act(gate) now and then). tanh-GELU: 1 + tanh(z) cancels for z << 0,
    which turns the ulp-level difference between CUDA tanhf and torch's tanh into a
    visible relative error on outputs of magnitude < 1e-3, so the tail is held to an
    absolute bound instead."""
    if act == "silu":
        assert ulp_close(got, ref)
        assert (got == ref).float().mean() > 0.999
    else:
        torch.testing.assert_close(got.float(), ref.float(), rtol=2e-3, atol=2e-4)
        assert (got == ref).float().mean() > 0.99


# ------------------------------------------------------------------ quantisers
@pytest.mark.parametrize("M,K", [(1, 16), (3, 4096), (257, 1024), (64, 12288), (5, 100), (2, 16384), (7, 40)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_quantize_rows_bit_exact(M, K, dtype):
    import fni8

    x = act_input(M, K, 11 + M + K, dtype)
    x[0, :] = 0  # all-zero row: scale 0, codes 0
    q, s = fni8.quantize_rows(x.to(DEV))
    qr, sr = O.quantize_rows(x)
    assert torch.equal(q.cpu(), qr) and torch.equal(s.cpu(), sr)


@pytest.mark.parametrize("shape", [(4, 8, 512), (3, 1024), (130, 4096), (2, 2048), (5, 96), (9, 100)])
def test_rmsnorm_and_fused_quant(shape):
    import fni8

    K = shape[-1]
    g = gen(sum(shape))
    x = torch.randn(shape, generator=g).half()
    r = torch.randn(shape, generator=g).half()
    w = (1 + 0.1 * torch.randn(K, generator=g)).half()
    y = fni8.rmsnorm(x.to(DEV), w.to(DEV), 1e-6)
    assert ulp_close(y, O.rmsnorm(x, w, 1e-6))
    y2, nr = fni8.rmsnorm(x.to(DEV), w.to(DEV), 1e-6, residual=r.to(DEV))
    yr, nrr = O.rmsnorm(x, w, 1e-6, residual=r)
    assert torch.equal(nr.cpu(), nrr) and ulp_close(y2, yr)
    yu = fni8.rmsnorm(x.to(DEV), (0.1 * w).to(DEV), 1e-6, unit_offset=True)
    assert ulp_close(yu, O.rmsnorm(x, 0.1 * w, 1e-6, unit_offset=True))
    # fused: the int8 rows are exactly the quantisation of the (rounded) normed rows
    q, s, nr2, yn = fni8.rmsnorm_quant(x.to(DEV), w.to(DEV), 1e-6, residual=r.to(DEV), keep_normed=True)
    qr, sr = O.quantize_rows(yn.cpu().reshape(-1, K))
    assert torch.equal(q.cpu().reshape(-1, K), qr) and torch.equal(s.cpu().reshape(-1), sr)
    assert torch.equal(nr2.cpu(), nrr) and torch.equal(yn, y2)


@pytest.mark.parametrize("act", ["silu", "gelu_tanh"])
@pytest.mark.parametrize("M,I", [(6, 768), (33, 12288), (4, 100), (1, 8)])
def test_act_and_mul_and_fused_quant(act, M, I):
    import fni8

    x = (2 * torch.randn(M, 2 * I, generator=gen(M * I))).half()
    h = fni8.act_and_mul(x.to(DEV), act)
    hr = O.act_and_mul(x, act)
    act_close(h.cpu(), hr, act)
    q, s = fni8.act_and_mul_quant(x.to(DEV), act)
    qr, sr = O.quantize_rows(h.cpu())
    assert torch.equal(q.cpu(), qr) and torch.equal(s.cpu(), sr)


def test_act_and_mul_matches_reference_golden(golden):
    import fni8

    g = golden("act")
    x = torch.from_numpy(g["x"])
    for act in ("silu", "gelu_tanh"):
        ref = torch.from_numpy(g[act])
        got = fni8.act_and_mul(x.to(DEV), act).cpu()
        act_close(got, ref, act)


def test_rmsnorm_matches_reference_golden(golden):
    import fni8

    g = golden("rmsnorm")
    for tag in "abc":
        x, r, w = (torch.from_numpy(g[f"{tag}_{n}"]) for n in ("x", "r", "w"))
        assert ulp_close(fni8.rmsnorm(x.to(DEV), w.to(DEV), 1e-6), torch.from_numpy(g[f"{tag}_y"]))
        y, nr = fni8.rmsnorm(x.to(DEV), w.to(DEV), 1e-6, residual=r.to(DEV))
        assert torch.equal(nr.cpu(), torch.from_numpy(g[f"{tag}_new_res"]))
        assert ulp_close(y, torch.from_numpy(g[f"{tag}_y_res"]))


# ------------------------------------------------------------------ GEMMs
SHAPES = [(1, 128, 128), (16, 256, 512), (33, 200, 160), (64, 4096, 4096), (128, 6144, 1024),
          (256, 6144, 1024), (300, 512, 4096), (1000, 1000, 272), (129, 257, 16), (8, 4096, 12288),
          (4096, 4096, 512), (2048, 3000, 1024)]


def _int8(shape, seed):
    return torch.randint(-127, 128, shape, generator=gen(seed), dtype=torch.int8)


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_int32_bit_exact(M, N, K):
    import fni8
    from fni8 import _native as nat

    a, w = _int8((M, K), M + 1), _int8((N, K), N + 2)
    ref = O.int_mm_fast(a, w)
    paths = [nat.PATH_TILE, nat.PATH_AUTO] + ([nat.PATH_STREAM, nat.PATH_SPLITK] if M <= 256 else [])
    for p in paths:
        got = fni8.gemm_i32(a.to(DEV), w.to(DEV), path=p).cpu()
        assert torch.equal(got, ref), (p, (got - ref).abs().max())


@pytest.mark.parametrize("path", ["stream", "splitk"])
@pytest.mark.parametrize("M,N,K", [(1, 6144, 4096), (32, 4096, 4096), (7, 24576, 4096), (256, 4096, 12288),
                                   (96, 1000, 2048)])
def test_decode_gemm_repeat_and_workspace_clean(M, N, K, path):
    """Stream-K and split-K partial sums go through the shared workspace: results stay
    exact across calls of different shapes, and the workspace is zero again after each call."""
    import fni8
    from fni8 import _native as nat
    from fni8.ops import WORKSPACE

    p = nat.PATH_STREAM if path == "stream" else nat.PATH_SPLITK
    a, w = _int8((M, K), 5 * M), _int8((N, K), 7)
    ref = O.int_mm_fast(a, w)
    for _ in range(3):
        got = fni8.gemm_i32(a.to(DEV), w.to(DEV), path=p).cpu()
        assert torch.equal(got, ref)
    torch.cuda.synchronize()
    assert int(WORKSPACE.get(torch.device(DEV)).count_nonzero()) == 0
    assert fni8.device_status() == 0


@pytest.mark.parametrize("M,N,K", [(16, 256, 512), (256, 6144, 1024), (77, 4104, 1024), (1024, 2048, 2048),
                                   (4, 100, 64), (40, 4096, 12288), (130, 520, 4096)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("extras", ["none", "bias", "bias+residual"])
def test_dequant_epilogue_bit_exact(M, N, K, dtype, extras):
    import fni8
    from fni8 import _native as nat

    x = act_input(M, K, M + N, dtype)
    wq, ws = weight(N, K, K)
    q, s = O.quantize_rows(x)
    g = gen(3)
    bias = (0.1 * torch.randn(N, generator=g)).to(dtype) if extras != "none" else None
    res = torch.randn(M, N, generator=g).to(dtype) if extras == "bias+residual" else None
    ref = O.dequant(O.int_mm_fast(q, wq), s, ws, bias=bias, residual=res, out_dtype=dtype)
    qt = fni8.QTensor(wq.to(DEV), ws.to(DEV), scheme="per_row_i8")
    paths = [nat.PATH_TILE] + ([nat.PATH_STREAM, nat.PATH_SPLITK] if M <= 256 else [])
    for p in paths:
        got = fni8.linear_q(q.to(DEV), s.to(DEV), qt, bias=None if bias is None else bias.to(DEV),
                            residual=None if res is None else res.to(DEV), out_dtype=dtype, path=p).cpu()
        assert torch.equal(got, ref), (p, (got.float() - ref.float()).abs().max())


@pytest.mark.parametrize("S", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("M,N,K", [(1, 640, 2048), (17, 1000, 4096), (64, 384, 1152), (200, 4104, 8192)])
def test_splitk_every_cluster_size(M, N, K, S):
    """The split-K kernel under each cluster size (forced through FNI8_SPLITK_S in a child
    process, since the plan reads it once): int32 sums exact for every K split."""
    import subprocess
    import sys

    code = f"""
import sys, torch
sys.path.insert(0, {PKG!r})
import fni8
from fni8 import _native as nat
g = torch.Generator().manual_seed({M + N + S})
a = torch.randint(-127, 128, ({M}, {K}), generator=g, dtype=torch.int8)
w = torch.randint(-127, 128, ({N}, {K}), generator=g, dtype=torch.int8)
ref = (a.long() @ w.long().T).int()
got = fni8.gemm_i32(a.cuda(), w.cuda(), path=nat.PATH_SPLITK).cpu()
assert torch.equal(got, ref), (got - ref).abs().max()
assert fni8.device_status() == 0
print("ok")
"""
    env = dict(os.environ, FNI8_SPLITK_S=str(S))
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stderr[-2000:]


@pytest.mark.parametrize("pair", ["0", "1"])
def test_tile_gemm_with_and_without_cta_pairs(pair):
    """The tile kernel with 256-row tiles on CTA pairs (tcgen05.mma.cta_group::2) and with
    128-row tiles on single CTAs gives the same exact int32 sums, dense and grouped, for
    shapes with ragged M, N and K (both settings forced through the environment in a
    child process, since the library reads them once)."""
    import subprocess
    import sys

    code = f"""
import sys, torch
sys.path.insert(0, {PKG!r})
import fni8
from fni8 import _native as nat
from fni8.moe import grouped_gemm
g = torch.Generator().manual_seed(11)
for M, N, K in [(256, 256, 128), (300, 512, 1024), (1024, 2048, 2048), (777, 1000, 272), (4096, 768, 4096)]:
    a = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8)
    w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
    ref = (a.long() @ w.long().T).int()
    got = fni8.gemm_i32(a.cuda(), w.cuda(), path=nat.PATH_TILE).cpu()
    assert torch.equal(got, ref), ("dense", M, N, K)
E, N, K = 6, 512, 256
cnt = torch.tensor([0, 300, 17, 256, 129, 40], dtype=torch.int32)
off = torch.zeros(E, dtype=torch.int32)
off[1:] = torch.cumsum(cnt, 0)[:-1]
R = int(cnt.sum())
a = torch.randint(-127, 128, (R, K), generator=g, dtype=torch.int8)
w = torch.randint(-127, 128, (E, N, K), generator=g, dtype=torch.int8)
exp = torch.tensor([5, 0, 2, 1, 4, 3], dtype=torch.int32)
got = grouped_gemm(a.cuda(), torch.ones(R).cuda(), w.cuda(), torch.ones(E, N).cuda(), exp.cuda(), off.cuda(),
                   cnt.cuda(), out_dtype=torch.int32).cpu()
for s in range(E):
    o, c = int(off[s]), int(cnt[s])
    if c:
        assert torch.equal(got[o:o + c], (a[o:o + c].long() @ w[int(exp[s])].long().T).int()), ("grouped", s)
assert fni8.device_status() == 0
print("ok")
"""
    env = dict(os.environ, FNI8_TILE_PAIR=pair, FNI8_GROUPED_PAIR=pair)
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stderr[-2000:]


@pytest.mark.parametrize("M,K,N", [(256, 1024, 6144), (1, 4096, 6144), (8, 4096, 4096), (32, 4096, 24576),
                                   (128, 12288, 4096), (512, 4096, 6144)])
def test_linear_bit_exact_vs_oracle(M, K, N):
    """fni8.linear end to end (quant + GEMM + epilogue) equals the oracle bit for bit."""
    import fni8

    x = act_input(M, K, M * 3 + K)
    wq, ws = weight(N, K, N)
    qt = fni8.QTensor(wq.to(DEV), ws.to(DEV), scheme="per_row_i8")
    got = fni8.linear(x.to(DEV).reshape(1, M, K), qt).cpu()
    assert got.shape == (1, M, N)
    assert torch.equal(got.reshape(M, N), O.linear_w8a8(x, wq, ws, exact=False))


@pytest.mark.parametrize("M,K,N", [(1, 100, 128), (37, 40, 200), (300, 1028, 256), (5, 4, 100)])
def test_linear_any_k_multiple_of_4(M, K, N):
    """fni8-serve takes any K that is a multiple of 4 (convert.py:128); the GEMMs need 16.
    fni8.linear and linear_q pad K with zeros (weight once, activations per call): the
    outputs equal the oracle on the unpadded shapes bit for bit."""
    import fni8

    x = act_input(M, K, 7 * M + K)
    wq, ws = weight(N, K, N + 1)
    qt = fni8.QTensor(wq.to(DEV), ws.to(DEV), scheme="per_row_i8")
    ref = O.linear_w8a8(x, wq, ws, exact=False)
    for _ in range(2):  # the second call reuses the padded weight
        assert torch.equal(fni8.linear(x.to(DEV), qt).cpu(), ref)
    q, s = fni8.quantize_rows(x.to(DEV))
    assert torch.equal(fni8.linear_q(q, s, qt).cpu(), ref)


def test_first_calls_from_several_host_threads():
    """Four host threads make their first fni8.linear calls at the same moment in a fresh
    process (one-time kernel attribute setup, split-K cluster plans, the tensor-map encoder
    and the workspace are all first touched concurrently), all on the default stream; every
    result equals the oracle."""
    import subprocess
    import sys

    root = os.path.dirname(PKG)
    code = f"""
import sys, threading, torch
sys.path.insert(0, {PKG!r}); sys.path.insert(0, {root!r})
import fni8
from oracle import w8a8_oracle as O
shapes = [(1, 4096, 6144), (24, 1024, 4096), (100, 2048, 3072), (300, 1024, 2048)]
g = torch.Generator().manual_seed(5)
cases = []
for M, K, N in shapes:
    x = torch.randn(M, K, generator=g).half()
    wq, ws = O.quantize_weight_rowwise(0.02 * torch.randn(N, K, generator=g))
    cases.append((x, wq, ws, O.linear_w8a8(x, wq, ws, exact=False)))
dev = [(x.cuda(), fni8.QTensor(wq.cuda(), ws.cuda())) for x, wq, ws, _ in cases]
torch.cuda.synchronize()
start = threading.Barrier(len(cases))
out, err = [None] * len(cases), []
def run(i):
    try:
        start.wait()
        out[i] = [fni8.linear(dev[i][0], dev[i][1]) for _ in range(3)]
    except BaseException as e:
        err.append(repr(e))
ts = [threading.Thread(target=run, args=(i,)) for i in range(len(cases))]
[t.start() for t in ts]
[t.join() for t in ts]
torch.cuda.synchronize()
assert not err, err
for i, (_, _, _, ref) in enumerate(cases):
    for y in out[i]:
        assert torch.equal(y.cpu(), ref), i
assert fni8.device_status() == 0
print("ok")
"""
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stderr[-2000:]


def test_linear_matches_reference_golden(golden):
    """The reference's own acceptance bound for its int8 path (tests/test_smoke.py:67-80)
    against LinearW8A8's fp16 fallback output, plus bit-exactness against the oracle."""
    import torch.nn.functional as F

    import fni8

    g = golden("linear")
    for tag in ("smoke", "cfg0"):
        x, wq, ws, b = (torch.from_numpy(g[f"{tag}_{n}"]) for n in ("x", "wq", "ws", "bias"))
        qt = fni8.QTensor(wq.to(DEV), ws.to(DEV), scheme="per_row_i8")
        for bias, key in ((None, "y"), (b, "y_bias")):
            y = fni8.linear(x.to(DEV), qt, bias=None if bias is None else bias.to(DEV)).cpu()
            ref = torch.from_numpy(g[f"{tag}_{key}"])
            cos = F.cosine_similarity(y.flatten().float(), ref.flatten().float(), dim=0).item()
            assert cos >= 0.99 and torch.isfinite(y.float()).all()
            assert torch.equal(y, O.linear_w8a8(x, wq, ws, bias=bias, exact=True))


def test_large_prefill_gemm_exact_against_int_mm():
    """Qwen3-8B prefill shape (M=8192): int32 accumulators equal torch._int_mm (cuBLASLt
    int8, used here only as an exact integer checker) and a CPU oracle row sample."""
    import fni8

    M, N, K = 8192, 6144, 4096
    a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=DEV)
    w = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=DEV)
    got = fni8.gemm_i32(a, w)
    ref = torch._int_mm(a, w.t())
    assert torch.equal(got, ref)
    rows = torch.randperm(M, generator=gen(1))[:16]
    assert torch.equal(got[rows.to(DEV)].cpu(), O.int_mm_fast(a[rows.to(DEV)].cpu(), w.cpu()))


def test_zero_rows_and_errors():
    import fni8
    from fni8 import Fni8Error

    qt = fni8.QTensor(torch.zeros(32, 64, dtype=torch.int8, device=DEV), torch.ones(32, device=DEV))
    assert fni8.linear(torch.zeros(0, 64, dtype=torch.float16, device=DEV), qt).shape == (0, 32)
    with pytest.raises(Fni8Error, match="multiple of 16"):  # the raw GEMM keeps the TMA rule
        fni8.gemm_i32(torch.zeros(4, 40, dtype=torch.int8, device=DEV),
                      torch.zeros(32, 40, dtype=torch.int8, device=DEV))
    packed = torch.zeros(32, 64, dtype=torch.uint8, device=DEV)  # 4-bit weights for K = 128
    with pytest.raises(NotImplementedError):  # NF4 has no integer GEMM (fni8-serve uses its fp16 path)
        fni8.linear(torch.zeros(4, 128, dtype=torch.float16, device=DEV),
                    fni8.QTensor(packed, torch.ones(32, 4, device=DEV), scheme="per_group_i4", group_size=32,
                                 codebook="nf4"))
    with pytest.raises(Fni8Error, match="group_size 128"):
        fni8.linear(torch.zeros(4, 128, dtype=torch.float16, device=DEV),
                    fni8.QTensor(packed, torch.ones(32, 4, device=DEV), scheme="per_group_i4", group_size=32,
                                 codebook="int4"))
    assert fni8.device_status() == 0


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (3, 6144, 4096), (16, 4096, 12288), (17, 24576, 4096),
                                   (32, 1000, 2048), (5, 128, 16), (8, 640, 4112), (2, 300, 1024)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_decode_linear_bit_exact(M, N, K, dtype):
    """fni8.linear at decode sizes (per-token quantiser, then the split-K GEMM) equals the
    oracle bit for bit, with and without bias, and equals linear_q on the same int8 rows.
    FNI8_PATH_FUSED is reserved and refused."""
    import fni8
    from fni8 import Fni8Error
    from fni8 import _native as nat

    x = act_input(M, K, 7 * M + N, dtype)
    wq, ws = weight(N, K, K + 1)
    qt = fni8.QTensor(wq.to(DEV), ws.to(DEV))
    bias = (0.1 * torch.randn(N, generator=gen(9))).to(dtype)
    for b in (None, bias):
        got = fni8.linear(x.to(DEV), qt, bias=None if b is None else b.to(DEV)).cpu()
        assert torch.equal(got, O.linear_w8a8(x, wq, ws, bias=b, exact=False))
        q, s = fni8.quantize_rows(x.to(DEV))
        viaq = fni8.linear_q(q, s, qt, bias=None if b is None else b.to(DEV), out_dtype=dtype).cpu()
        assert torch.equal(got, viaq)
    with pytest.raises(Fni8Error, match="not built"):
        fni8.linear(x.to(DEV), qt, path=nat.PATH_FUSED)
    assert fni8.device_status() == 0
