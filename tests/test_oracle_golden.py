"""Pin the CPU oracle (oracle/w8a8_oracle.py) to outputs of the reference's own code.

The fixtures in tests/golden/ were produced by fni8-serve's modules on CPU
(tests/golden/make_golden.py). Where the reference computes the same thing, the
oracle must agree exactly; where the reference's arithmetic lives in the absent `fni8`
package (activation quantisation, the int8 GEMM), the oracle is held to the
reference tests' own bound (cos >= 0.99 against the fp16 fallback,
tests/test_smoke.py:67-80) and to exact integer arithmetic.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import w8a8_oracle as O


def t(a):
    return torch.from_numpy(np.ascontiguousarray(a))


@pytest.mark.parametrize("tag", ["a", "b", "c"])
def test_rmsnorm_matches_reference(golden, tag):
    g = golden("rmsnorm")
    x, r, w = t(g[f"{tag}_x"]), t(g[f"{tag}_r"]), t(g[f"{tag}_w"])
    assert torch.equal(O.rmsnorm(x, w, 1e-6), t(g[f"{tag}_y"]))
    y, nr = O.rmsnorm(x, w, 1e-6, residual=r)
    assert torch.equal(y, t(g[f"{tag}_y_res"])) and torch.equal(nr, t(g[f"{tag}_new_res"]))
    assert torch.equal(O.rmsnorm(x, t(g[f"{tag}_wu"]), 1e-6, unit_offset=True), t(g[f"{tag}_y_unit"]))


@pytest.mark.parametrize("act", ["silu", "gelu_tanh"])
def test_act_and_mul_matches_reference(golden, act):
    g = golden("act")
    assert torch.equal(O.act_and_mul(t(g["x"]), act), t(g[act]))


@pytest.mark.parametrize("tag", ["smoke", "cfg0"])
def test_linear_oracle_vs_reference_fallback(golden, tag):
    g = golden("linear")
    x, wq, ws, bias = t(g[f"{tag}_x"]), t(g[f"{tag}_wq"]), t(g[f"{tag}_ws"]), t(g[f"{tag}_bias"])
    for y_ref, b in ((t(g[f"{tag}_y"]), None), (t(g[f"{tag}_y_bias"]), bias)):
        y = O.linear_w8a8(x, wq, ws, bias=b)
        cos = F.cosine_similarity(y.flatten().float(), y_ref.flatten().float(), dim=0).item()
        assert cos >= 0.99, cos  # the reference's own bound for its int8 path
        assert torch.isfinite(y.float()).all()
    # the reference's weight dequant (linear.py:28-31) is what the fallback multiplies with
    w16 = O.dequant_weight_fallback(wq, ws)
    assert torch.equal(F.linear(x, w16), t(g[f"{tag}_y"]))


def test_weight_quant_matches_reference_tests(golden):
    """The reference tests' _i8 fixtures: test_smoke.py computes in fp32 exactly like the
    oracle; test_layers.py computes in fp16, so the scale differs by fp16 rounding and a
    few codes by one step."""
    g = golden("i8_fixture")
    q, s = O.quantize_weight_rowwise(t(g["smoke_w"]))
    assert torch.equal(q, t(g["smoke_q"]))
    torch.testing.assert_close(s, t(g["smoke_s"]), rtol=1e-6, atol=0)
    q, s = O.quantize_weight_rowwise(t(g["layers_w"]))
    d = (q.int() - t(g["layers_q"]).int()).abs()
    assert d.max() <= 1 and (d == 0).float().mean() > 0.98
    torch.testing.assert_close(s, t(g["layers_s"]).float(), rtol=1e-3, atol=0)


def test_weight_helpers_match_reference(golden):
    """to_qtensor / merge_qtensor (fni8serve/models/weights.py:18-39) with this repo's
    quantize_int8_rowwise: fused rows quantise as one, pre-quantised rows concat exactly."""
    import fni8

    g = golden("weights")
    qkv = torch.cat([t(g[f"p_{n}_proj_weight"]) for n in "qkv"])
    q, s = fni8.quant.core.quantize_int8_rowwise(qkv)
    assert torch.equal(q, t(g["qkv_q"])) and torch.equal(s.squeeze(-1), t(g["qkv_s"]))
    assert torch.equal(t(g["gu_pre_q"]), t(g["gu_q"]))  # per-row quant: concat == quantise-as-one


@pytest.mark.parametrize("scoring", ["softmax", "sigmoid"])
def test_moe_routing_and_output_vs_reference(golden, scoring):
    g = golden(f"moe_{scoring}")
    x, gate = t(g["x"]), t(g["gate"])
    B, S, H = x.shape
    k, E = int(g["k"]), int(g["E"])
    xf = x.reshape(-1, H)
    logits = F.linear(xf.float(), gate.float())
    kw = {}
    if scoring == "sigmoid":
        kw = dict(sel_bias=t(g["bias"]), n_groups=2, topk_group=1)
    topi, topw = O.moe_route(logits, k, scoring=scoring, **kw)
    assert torch.equal(topi, t(g["topi"]))  # the reference's own routing choice
    y = O.moe_experts_w8a8(xf, topi, topw.float(), t(g["w_gu"]), t(g["s_gu"]), t(g["w_dn"]), t(g["s_dn"]),
                           exact=False)
    y_ref = t(g["y"]).reshape(-1, H)
    cos = F.cosine_similarity(y.flatten().float(), y_ref.flatten().float(), dim=0).item()
    assert cos >= 0.99, cos


def test_int_mm_fast_is_exact():
    g = torch.Generator().manual_seed(7)
    a = torch.randint(-127, 128, (33, 160), generator=g, dtype=torch.int8)
    w = torch.randint(-127, 128, (70, 160), generator=g, dtype=torch.int8)
    assert torch.equal(O.int_mm_exact(a, w), O.int_mm_fast(a, w))


def test_quantize_rows_contract():
    x = torch.tensor([[0.0, 0.0, 0.0, 0.0], [1.0, -2.0, 0.5, 2.0], [3e-8, -1e-8, 0, 0]], dtype=torch.float32)
    q, s = O.quantize_rows(x)
    assert s[0] == 0 and torch.equal(q[0], torch.zeros(4, dtype=torch.int8))
    assert torch.equal(q[1], torch.tensor([64, -127, 32, 127], dtype=torch.int8))  # 63.5 -> 64 (half-even)
    assert q[2, 0] == 127 and s[2] > 0


def test_moe_plan_is_stable_grouping():
    topi = torch.tensor([[2, 0], [0, 1], [2, 5], [1, 0]])
    counts, offsets, ros, sor = O.moe_plan(topi, 3)  # expert 5 is out of range: dropped
    assert counts.tolist() == [3, 2, 2] and offsets.tolist() == [0, 3, 5, 7]
    assert sor.tolist() == [1, 2, 7, 3, 6, 0, 4]
    assert ros[5] == -1 and all(ros[s] == r for r, s in enumerate(sor.tolist()))


def test_w4a8_oracle_against_reference_i4_path(golden):
    """per_group_i4 / int4 weights: the oracle's unpack + two's-complement decode equals the
    reference's own weight reconstruction (layers/linear.py:33-45) bit for bit, and the
    oracle's W4A8 linear stays within the reference tests' bound of its fp16 fallback."""
    g = golden("linear_i4")
    packed = torch.from_numpy(g["packed"])
    scale = torch.from_numpy(g["scale"])
    gs = int(g["group_size"])
    assert int(g["in_features"]) == 2 * packed.shape[1]
    assert torch.equal(O.dequant_weight_i4_fallback(packed, scale, gs), torch.from_numpy(g["w_ref"]))
    assert torch.equal(O.pack_i4(O.unpack_i4(packed)), packed)
    x = torch.from_numpy(g["x"])
    y = O.linear_w4a8(x, packed, scale, gs, bias=torch.from_numpy(g["bias"]))
    ref = torch.from_numpy(g["y_ref"]).float()
    cos = torch.nn.functional.cosine_similarity(y.float().flatten(), ref.flatten(), dim=0).item()
    assert cos >= 0.99, cos


@pytest.mark.parametrize("K", [4, 40, 100, 1028])
def test_zero_padding_k_is_exact(K):
    """fni8.linear pads K (any multiple of 4, fni8serve/convert.py:128) with zeros up to the
    GEMMs' multiple of 16. Zero channels leave each token's absmax, every int32 sum and so
    the dequantised output unchanged; the padded weight is built once per QTensor."""
    import fni8
    from fni8.ops import _k16_weight

    g = torch.Generator().manual_seed(K)
    x = torch.randn(9, K, generator=g).to(torch.float16)
    wq, ws = O.quantize_weight_rowwise(0.02 * torch.randn(24, K, generator=g))
    qt = fni8.QTensor(wq, ws, scheme="per_row_i8")
    wp, Kp = _k16_weight(qt, K)
    assert Kp % 16 == 0 and Kp - K < 16 and torch.equal(wp[:, :K], wq) and not wp[:, K:].any()
    assert _k16_weight(qt, K)[0] is wp
    xp = F.pad(x, (0, Kp - K))
    assert torch.equal(O.linear_w8a8(xp, wp, ws), O.linear_w8a8(x, wq, ws))
    qt.data[0, 0] = -qt.data[0, 0] - 1  # an in-place weight update rebuilds the padded copy
    wp2, _ = _k16_weight(qt, K)
    assert wp2 is not wp and torch.equal(wp2[:, :K], qt.data)
    qt.data = qt.data.clone()  # so does a replaced weight tensor
    assert _k16_weight(qt, K)[0] is not wp2


def test_nf4_fallback_weight_matches_reference(golden):
    """per_group_i4 / NF4: the reference's table lookup (low nibble first) and group scaling
    (fni8serve/layers/linear.py:33-45), computed by its own LinearW8A8 with this package's
    NF4_CODEBOOK, equal the oracle's restatement bit for bit; the fp16 fallback forward is
    F.linear on that weight; the stored table is the one the package exports today."""
    from fni8.quant.lowbit import NF4_CODEBOOK

    g = golden("linear_nf4")
    cb = t(g["codebook"])
    assert torch.equal(cb, torch.tensor(NF4_CODEBOOK, dtype=torch.float32))
    packed, scale, gs = t(g["packed"]), t(g["scale"]), int(g["group_size"])
    assert int(g["in_features"]) == 2 * packed.shape[1]
    w16 = O.dequant_weight_nf4_fallback(packed, scale, gs, cb)
    assert torch.equal(w16, t(g["w_ref"]))
    assert torch.equal(F.linear(t(g["x"]), w16), t(g["y_ref"]))


def test_moe_shared_expert_and_scaling_vs_reference(golden):
    """SparseMoE with a gated shared expert and routed_scaling_factor (moe.py:95,107-112),
    computed by the reference on CPU: the oracle's shared expert and the whole block (its
    routing with the scaling factor, routed experts, shared expert) stay within the
    reference tests' bound (cos >= 0.99 against the reference's fp16 fallback)."""
    g = golden("moe_shared")
    x, gate, sgate = t(g["x"]), t(g["gate"]), t(g["sgate"])
    B, S, H = x.shape
    k = int(g["k"])
    xf = x.reshape(-1, H)
    topi, topw = O.moe_route(F.linear(xf.float(), gate.float()), k, scaling=float(g["scaling"]))
    ys = O.moe_shared_expert(xf, t(g["sh_gu_q"]), t(g["sh_gu_s"]), t(g["sh_dn_q"]), t(g["sh_dn_s"]), sgate)
    y = O.moe_experts_w8a8(xf, topi, topw.float(), t(g["w_gu"]), t(g["s_gu"]), t(g["w_dn"]), t(g["s_dn"])) + ys
    for got, ref in ((ys, t(g["y_shared"])), (y, t(g["y"]).reshape(-1, H))):
        cos = F.cosine_similarity(got.flatten().float(), ref.flatten().float(), dim=0).item()
        assert cos >= 0.99, cos
    assert y.dtype == x.dtype


def test_moe_combine_restatement_vs_reference(golden):
    """The reference's expert-loop combine (fni8serve/models/moe.py:97-105: fp16
    `contrib * topw` added with index_add_ in expert order), run by the reference on CPU
    with every expert's contribution recorded: the oracle's restatement reproduces the
    block output bit for bit from those contributions, and this library's fp32 combine
    (one rounding) stays inside moe_combine_bound of it on every element."""
    g = golden("moe_combine")
    k = int(g["k"])
    topi, topw = O.moe_route(t(g["logits"]), k)
    assert torch.equal(topi, t(g["topi"]))  # the routing the reference chose
    y_slot = t(g["y_slot"])
    ref = t(g["y"]).reshape(-1, y_slot.shape[-1])
    assert torch.equal(O.moe_combine_reference(y_slot, topi, topw), ref)
    ours = O.moe_combine_fp32(y_slot, topw)
    assert bool(((ours.float() - ref.float()).abs() <= O.moe_combine_bound(y_slot, topw)).all())
    # a planted change in the restatement (fp32 product, no rounding to fp16) is caught
    planted = torch.zeros_like(ref)
    for e in range(int(g["E"])):
        tok, slot = (topi == e).nonzero(as_tuple=True)
        planted[tok] = (planted[tok].float() + y_slot[tok, slot].float() * topw[tok, slot].float()[:, None]).half()
    assert not torch.equal(planted, ref)
