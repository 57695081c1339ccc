"""W4A8 (per_group_i4 / int4 weights) on the sm_100a path, against the CPU oracle.

The int32 group sums are exact; the fp32 combination of the G groups follows the
oracle's order within a K slice and adds the slices in order when the kernel splits K
over a cluster. Reordering a sum of G fp32 terms moves it by at most ~2 * G * 2^-24 times
the sum of the terms' magnitudes, so the bound checked is: one unit in the last place of
the output dtype plus that reordering bound (oracle.linear_w4a8_magnitude). Nearly all
outputs are bit-identical.
"""
import pytest
import torch

from oracle import w8a8_oracle as O

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a B200")]

DEV = "cuda"


def gen(seed):
    return torch.Generator().manual_seed(seed)


def within_bound(got, ref, mag, K):
    """|got - ref| <= ulp_dtype(|ref|) + 2 * G * 2^-24 * mag, elementwise."""
    G = K // 128
    mant = 10 if ref.dtype == torch.float16 else 7
    r = ref.float().abs().clamp_min(2.0 ** -14)
    ulp = torch.exp2(torch.floor(torch.log2(r)) - mant)
    tol = ulp + 2 * G * 2.0 ** -24 * mag
    return ((got.float() - ref.float()).abs() <= tol).all().item()


def ulp_dist(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Distance in representable steps of a's dtype (fp16 / bf16), sign-aware."""
    ia = a.contiguous().view(torch.int16).to(torch.int32)
    ib = b.contiguous().view(torch.int16).to(torch.int32)
    ia = torch.where(ia < 0, -32768 - ia, ia)
    ib = torch.where(ib < 0, -32768 - ib, ib)
    return (ia - ib).abs()


def case(M, N, K, seed, dtype=torch.float16, with_bias=False):
    g = gen(seed)
    w = 0.02 * torch.randn(N, K, generator=g)
    packed, scale = O.quantize_weight_i4(w, 128)
    x = torch.randn(M, K, generator=g).to(dtype)
    bias = (0.1 * torch.randn(N, generator=g)).to(dtype) if with_bias else None
    return x, packed, scale, bias


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (5, 200, 1024), (16, 6144, 4096), (33, 4096, 12288),
                                   (64, 128, 128), (100, 1000, 2048), (130, 384, 512)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_w4a8_linear_vs_oracle(M, N, K, dtype):
    import fni8

    x, packed, scale, bias = case(M, N, K, M + N + K, dtype, with_bias=(M % 2 == 1))
    qt = fni8.QTensor(packed.to(DEV), scale.to(DEV), scheme="per_group_i4", group_size=128, codebook="int4")
    got = fni8.linear(x.to(DEV), qt, bias=None if bias is None else bias.to(DEV)).cpu()
    ref = O.linear_w4a8(x, packed, scale, 128, bias=bias)
    assert got.shape == ref.shape and got.dtype == dtype
    mag = O.linear_w4a8_magnitude(x, packed, scale, 128)
    assert within_bound(got, ref, mag, K), float((got.float() - ref.float()).abs().max())
    assert float((ulp_dist(got, ref) > 0).float().mean()) < 0.01  # almost everything is bit-identical
    assert fni8.device_status() == 0


def test_w4a8_matches_reference_i4_fixture(golden):
    """The reference's own LinearW8A8 on 4-bit weights (fp16 fallback, layers/linear.py:33-45,
    70-71): the GPU result stays within the reference tests' bound (cos >= 0.99) and within
    one fp16 ulp of the oracle."""
    import fni8

    g = golden("linear_i4")
    packed, scale = torch.from_numpy(g["packed"]), torch.from_numpy(g["scale"])
    x, bias = torch.from_numpy(g["x"]), torch.from_numpy(g["bias"])
    qt = fni8.QTensor(packed.to(DEV), scale.to(DEV), scheme="per_group_i4", group_size=int(g["group_size"]),
                      codebook="int4")
    got = fni8.linear(x.to(DEV), qt, bias=bias.to(DEV)).cpu()
    ref = torch.from_numpy(g["y_ref"])
    cos = torch.nn.functional.cosine_similarity(got.float().flatten(), ref.float().flatten(), dim=0).item()
    assert cos >= 0.99, cos
    gs = int(g["group_size"])
    ref_o = O.linear_w4a8(x, packed, scale, gs, bias=bias)
    assert within_bound(got, ref_o, O.linear_w4a8_magnitude(x, packed, scale, gs), x.shape[-1])


def test_w4a8_workspace_stays_clean_and_repeats():
    import fni8
    from fni8.ops import WORKSPACE

    x, packed, scale, _ = case(16, 4096, 4096, 7)
    qt = fni8.QTensor(packed.to(DEV), scale.to(DEV), scheme="per_group_i4", group_size=128, codebook="int4")
    first = fni8.linear(x.to(DEV), qt)
    for _ in range(3):
        assert torch.equal(fni8.linear(x.to(DEV), qt), first)  # deterministic split and order
    torch.cuda.synchronize()
    assert int(WORKSPACE.get(torch.device(DEV)).count_nonzero()) == 0
    assert fni8.device_status() == 0
