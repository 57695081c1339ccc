"""Generate the golden fixtures in tests/golden/*.npz from the REFERENCE's own code.

Runs only where the fni8-serve sources are available (pass --reference, or set
$FNI8_REFERENCE to the checkout); the GPU box never runs it, it only reads the committed
.npz files. fni8-serve cannot be imported normally here because its kernels
package `fni8` is not installed, so this script:

  * puts this repository's drop-in `fni8` package on sys.path (only QTensor and
    quant.core.quantize_int8_rowwise are exercised: the reference's CPU paths never
    call an fni8 kernel), and
  * registers empty package objects for `fni8serve`, `fni8serve.layers` and
    `fni8serve.models` so the individual modules below load without executing the
    package __init__ files (which pull in the engine, loader and attention kernels).

Every output below is computed by fni8-serve's own modules on CPU:
    layers/norm.py RMSNorm (CPU path)          -> rmsnorm.npz
    layers/activation.py SiluAndMul/GeluAndMul -> act.npz
    layers/linear.py LinearW8A8 (fp16 fallback) -> linear.npz
    layers/linear.py LinearW8A8 with per_group_i4 / int4 weights (its weight
        reconstruction and fp16 fallback)      -> linear_i4.npz
    layers/linear.py LinearW8A8 with per_group_i4 / NF4 weights (table lookup and
        fp16 fallback)                         -> linear_nf4.npz
    models/weights.py to_qtensor/merge_qtensor -> weights.npz
    convert.py convert_hf_to_fni8 + loader.py on a tiny Qwen3 checkpoint, and
        loader.py save_training_checkpoint, through this package's .fni8 format -> convert.npz
    models/moe.py SparseMoE (softmax and sigmoid+group-limited routing) -> moe_*.npz
    models/moe.py SparseMoE with a gated shared expert and routed scaling -> moe_shared.npz
    models/moe.py SparseMoE's combine: every expert's contribution and the output the
        expert loop accumulates with index_add_ (moe.py:97-105) -> moe_combine.npz
    tests/test_layers.py::_i8 and tests/test_smoke.py::_i8 (the reference tests' own
        weight-quant fixtures)                  -> i8_fixture.npz
Inputs are seeded; every fixture stores its inputs too, so the tests need nothing else.
"""
from __future__ import annotations

import argparse
import importlib
import importlib.util
import os
import sys
import types

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def _setup(ref: str):
    sys.path.insert(0, os.path.join(REPO, "fni8-serve_b200"))
    import fni8  # this repository's drop-in package

    for name in ("fni8serve", "fni8serve.layers", "fni8serve.models"):
        mod = types.ModuleType(name)
        mod.__path__ = [os.path.join(ref, *name.split("."))]
        sys.modules[name] = mod
    L = types.SimpleNamespace()
    L.fni8 = fni8
    L.linear = importlib.import_module("fni8serve.layers.linear")
    L.norm = importlib.import_module("fni8serve.layers.norm")
    L.act = importlib.import_module("fni8serve.layers.activation")
    L.mlp = importlib.import_module("fni8serve.layers.mlp")
    L.weights = importlib.import_module("fni8serve.models.weights")
    L.moe = importlib.import_module("fni8serve.models.moe")
    return L


def _load_test_module(ref: str, fname: str, L):
    """Import one of the reference's test files to call its fixture helpers."""
    layers_pkg = sys.modules["fni8serve.layers"]
    for n in ("GatedMLP", "GeluAndMul", "RMSNorm", "SiluAndMul", "get_act_and_mul"):
        setattr(layers_pkg, n, getattr(L.mlp, n, None) or getattr(L.act, n, None) or getattr(L.norm, n, None))
    for n in ("LMHead", "RotaryEmbedding", "Sampler", "VocabEmbedding", "LinearW8A8"):
        if not hasattr(layers_pkg, n):
            setattr(layers_pkg, n, getattr(L.linear, n, None))
    top = sys.modules["fni8serve"]
    top.ServeConfig = None
    top.load_fni8_checkpoint = None
    if not hasattr(L.fni8, "save_fni8"):
        L.fni8.save_fni8 = None  # only referenced at import time by test_smoke.py
    spec = importlib.util.spec_from_file_location(f"_ref_{fname[:-3]}", os.path.join(ref, "tests", fname))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _np(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy()
    return t.detach().numpy()


def gen_rmsnorm(L) -> dict:
    g = torch.Generator().manual_seed(101)
    out = {}
    for tag, shape, dt in (("a", (4, 8, 512), torch.float16), ("b", (3, 1024), torch.float16),
                           ("c", (5, 4096), torch.float16)):
        K = shape[-1]
        x = torch.randn(shape, generator=g).to(dt)
        r = torch.randn(shape, generator=g).to(dt)
        w = (1.0 + 0.1 * torch.randn(K, generator=g)).to(torch.float16)
        eps = 1e-6
        n = L.norm.RMSNorm(K, eps=eps, weight=w.clone())
        y = n(x)
        y_r, new_r = n(x, r)
        nu = L.norm.RMSNorm(K, eps=eps, weight=(0.1 * torch.randn(K, generator=g)).to(torch.float16),
                            add_unit_offset=True)
        y_u = nu(x)
        out.update({f"{tag}_x": _np(x), f"{tag}_r": _np(r), f"{tag}_w": _np(w), f"{tag}_wu": _np(nu.weight.data),
                    f"{tag}_y": _np(y), f"{tag}_y_res": _np(y_r), f"{tag}_new_res": _np(new_r),
                    f"{tag}_y_unit": _np(y_u)})
    return out


def gen_act(L) -> dict:
    g = torch.Generator().manual_seed(202)
    x = (2 * torch.randn(6, 2 * 768, generator=g)).to(torch.float16)
    return {"x": _np(x), "silu": _np(L.act.SiluAndMul()(x)), "gelu_tanh": _np(L.act.GeluAndMul("tanh")(x))}


def gen_linear(L) -> dict:
    """LinearW8A8 on CPU = the reference's fp16 dequant fallback (linear.py:70-71)."""
    g = torch.Generator().manual_seed(303)
    out = {}
    # the shape of tests/test_smoke.py:67-80 (N=256, K=512, M=16) and a BASELINE config-0
    # slice (K=1024, 0.1% outlier channels x20)
    for tag, (M, K, N, outl) in (("smoke", (16, 512, 256, False)), ("cfg0", (64, 1024, 256, True))):
        w = (0.02 * torch.randn(N, K, generator=g)).to(torch.float16)
        qt = L.weights.to_qtensor(w)
        x = torch.randn(M, K, generator=g)
        if outl:
            ch = torch.randperm(K, generator=g)[: max(1, K // 1000)]
            x[:, ch] *= 20
        x = x.to(torch.float16)
        bias = (0.1 * torch.randn(N, generator=g)).to(torch.float16)
        y = L.linear.LinearW8A8(qt)(x)
        yb = L.linear.LinearW8A8(qt, bias)(x)
        out.update({f"{tag}_x": _np(x), f"{tag}_wq": _np(qt.data), f"{tag}_ws": _np(qt.scale),
                    f"{tag}_bias": _np(bias), f"{tag}_y": _np(y), f"{tag}_y_bias": _np(yb)})
    return out


def gen_linear_i4(L) -> dict:
    """LinearW8A8 on CPU with 4-bit weights: _dequant_weight (linear.py:33-45) and the fp16
    fallback forward. The packed codes and scales come from the oracle's int4 quantiser
    (the converter's quantize_lowbit lives in the absent fni8 package)."""
    sys.path.insert(0, REPO)
    from oracle import w8a8_oracle as O

    g = torch.Generator().manual_seed(404)
    M, K, N, gs = 16, 512, 192, 128
    w = 0.02 * torch.randn(N, K, generator=g)
    packed, scale = O.quantize_weight_i4(w, gs)
    qt = L.fni8.QTensor(packed, scale, scheme="per_group_i4", group_size=gs, codebook="int4")
    x = torch.randn(M, K, generator=g).to(torch.float16)
    bias = (0.1 * torch.randn(N, generator=g)).to(torch.float16)
    lin = L.linear.LinearW8A8(qt, bias)
    return {"x": _np(x), "packed": _np(packed), "scale": _np(scale), "bias": _np(bias), "group_size": np.int64(gs),
            "in_features": np.int64(lin.in_features), "w_ref": _np(L.linear._dequant_weight(qt)), "y_ref": _np(lin(x))}


def gen_linear_nf4(L) -> dict:
    """LinearW8A8 on CPU with NF4 weights (per_group_i4, codebook "nf4"): the reference's
    table lookup by 4-bit code, low nibble first (linear.py:33-39), times the group scale,
    and its fp16 fallback forward. The table is this package's fni8.quant.lowbit
    NF4_CODEBOOK (the reference imports it from `fni8`, linear.py:22-25); it is stored too,
    so a change to the table shows up as a fixture mismatch."""
    g = torch.Generator().manual_seed(505)
    M, K, N, gs = 8, 256, 96, 64
    codes = torch.randint(0, 16, (N, K), generator=g)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).to(torch.uint8)
    scale = 0.01 + 0.05 * torch.rand(N, K // gs, generator=g)
    qt = L.fni8.QTensor(packed, scale, scheme="per_group_i4", group_size=gs, codebook="nf4")
    x = torch.randn(M, K, generator=g).to(torch.float16)
    lin = L.linear.LinearW8A8(qt, None)
    cb = torch.tensor(L.linear.NF4_CODEBOOK, dtype=torch.float32)
    return {"x": _np(x), "packed": _np(packed), "scale": _np(scale), "group_size": np.int64(gs), "codebook": _np(cb),
            "in_features": np.int64(lin.in_features), "w_ref": _np(L.linear._dequant_weight(qt)), "y_ref": _np(lin(x))}


def gen_moe_shared(L) -> dict:
    """SparseMoE with a gated shared expert and a routed scaling factor (moe.py:95,107-112),
    softmax routing, on CPU: the block's output, and its shared expert's (gated) output."""
    g = torch.Generator().manual_seed(608)
    E, k, H, I, Is = 8, 2, 128, 64, 96
    B, S = 2, 12
    sd = {}
    for e in list(range(E)) + ["s"]:
        n = Is if e == "s" else I
        sd[f"e{e}.gate_proj.weight"] = (0.05 * torch.randn(n, H, generator=g)).to(torch.float16)
        sd[f"e{e}.up_proj.weight"] = (0.05 * torch.randn(n, H, generator=g)).to(torch.float16)
        sd[f"e{e}.down_proj.weight"] = (0.05 * torch.randn(H, n, generator=g)).to(torch.float16)
    experts = [(L.weights.gate_up_weight(sd, f"e{e}"), L.weights.to_qtensor(sd[f"e{e}.down_proj.weight"]))
               for e in range(E)]
    shared = (L.weights.gate_up_weight(sd, "es"), L.weights.to_qtensor(sd["es.down_proj.weight"]))
    gate = (0.05 * torch.randn(E, H, generator=g)).to(torch.float16)
    sgate = (0.05 * torch.randn(1, H, generator=g)).to(torch.float16)
    moe = L.moe.SparseMoE(gate=gate, experts=experts, top_k=k, norm_topk_prob=True, shared_expert=shared,
                          shared_expert_gate=sgate, routed_scaling_factor=2.5)
    x = torch.randn(B, S, H, generator=g).to(torch.float16)
    y = moe(x)
    xf = x.reshape(-1, H)
    ys = moe.shared(x).reshape(-1, H) * torch.sigmoid(F.linear(xf.float(), sgate.float())).to(x.dtype)
    return {"x": _np(x), "gate": _np(gate), "sgate": _np(sgate), "y": _np(y), "y_shared": _np(ys),
            "w_gu": np.stack([_np(gu.data) for gu, _ in experts]), "s_gu": np.stack([_np(gu.scale) for gu, _ in experts]),
            "w_dn": np.stack([_np(dn.data) for _, dn in experts]), "s_dn": np.stack([_np(dn.scale) for _, dn in experts]),
            "sh_gu_q": _np(shared[0].data), "sh_gu_s": _np(shared[0].scale), "sh_dn_q": _np(shared[1].data),
            "sh_dn_s": _np(shared[1].scale), "E": np.array(E), "k": np.array(k), "scaling": np.float32(2.5)}


def gen_convert(L) -> dict:
    """fni8-serve's own converter and loader on a tiny synthetic Qwen3 checkpoint, run over
    this package's `.fni8` format: convert_hf_to_fni8 (convert.py:254-362: safetensors in,
    its quantisation rules and 4-bit packing, FQWriter out) at 8 and 4 bits, then
    load_fni8_state_dict / checkpoint_info (loader.py:19-69), and a training checkpoint
    from save_training_checkpoint (loader.py:75-103). Stores the source weights, each
    container's bytes, and what the reference's loader reported."""
    import json
    import tempfile

    from safetensors.torch import save_file

    conv = importlib.import_module("fni8serve.convert")
    loader = importlib.import_module("fni8serve.loader")
    H, I, V, nh, nkv, hd, gs = 64, 128, 128, 4, 2, 16, 32
    cfg = {"architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3", "hidden_size": H, "intermediate_size": I,
           "num_hidden_layers": 1, "num_attention_heads": nh, "num_key_value_heads": nkv, "head_dim": hd,
           "vocab_size": V, "rms_norm_eps": 1e-6, "rope_theta": 10000.0, "max_position_embeddings": 512,
           "tie_word_embeddings": False, "torch_dtype": "bfloat16"}
    g = torch.Generator().manual_seed(606)
    sd = {"model.embed_tokens.weight": torch.randn(V, H, generator=g), "model.norm.weight": torch.ones(H),
          "lm_head.weight": 0.02 * torch.randn(V, H, generator=g)}
    p = "model.layers.0."
    for n, shape in (("self_attn.q_proj", (nh * hd, H)), ("self_attn.k_proj", (nkv * hd, H)),
                     ("self_attn.v_proj", (nkv * hd, H)), ("self_attn.o_proj", (H, nh * hd)),
                     ("mlp.gate_proj", (I, H)), ("mlp.up_proj", (I, H)), ("mlp.down_proj", (H, I))):
        sd[p + n + ".weight"] = 0.02 * torch.randn(*shape, generator=g)
    for n, size in (("self_attn.q_norm", hd), ("self_attn.k_norm", hd), ("input_layernorm", H),
                    ("post_attention_layernorm", H)):
        sd[p + n + ".weight"] = 1 + 0.1 * torch.randn(size, generator=g)
    sd = {k: v.to(torch.bfloat16).contiguous() for k, v in sd.items()}
    out = {"names": np.array(sorted(sd)), "group_size": np.int64(gs)}
    for k in sorted(sd):
        out["src/" + k] = _np(sd[k].view(torch.int16))  # bf16 bits
    with tempfile.TemporaryDirectory() as d:
        with open(os.path.join(d, "config.json"), "w") as f:
            json.dump(cfg, f)
        save_file(sd, os.path.join(d, "model.safetensors"))
        for bits in (8, 4):
            path = os.path.join(d, f"m{bits}.fni8")
            conv.convert_hf_to_fni8(d, path, weight_bits=bits, group_size=gs)
            info = loader.checkpoint_info(path)
            st = loader.load_fni8_state_dict(path, device="cpu")
            with open(path, "rb") as f:
                out[f"file{bits}"] = np.frombuffer(f.read(), dtype=np.uint8)
            out[f"info{bits}"] = np.array(json.dumps(info, sort_keys=True))
            out[f"schemes{bits}"] = np.array(json.dumps({k: getattr(v, "scheme", "tensor") for k, v in st.items()},
                                                        sort_keys=True))
        # the training checkpoint writer (loader.py:75-103): raw fp32 weights, AdamW state
        # and meta through save_fni8
        tr = types.ModuleType("fni8serve.training")
        tr.__path__ = [os.path.join(os.path.dirname(conv.__file__), "training")]
        sys.modules.setdefault("fni8serve.training", tr)
        torch.manual_seed(607)
        net = torch.nn.Sequential(torch.nn.Linear(16, 32), torch.nn.Linear(32, 8))
        opt = torch.optim.AdamW(net.parameters(), lr=1e-3)
        net(torch.randn(4, 16)).sum().backward()
        opt.step()
        path = os.path.join(d, "train.fni8")
        loader.save_training_checkpoint(path, net.state_dict(), opt, meta={"step": 7})
        with open(path, "rb") as f:
            out["train_file"] = np.frombuffer(f.read(), dtype=np.uint8)
        out["train_info"] = np.array(json.dumps(loader.checkpoint_info(path), sort_keys=True))
        for k, v in net.state_dict().items():
            out["train_sd/" + k] = _np(v)
    return out


def gen_weights(L) -> dict:
    g = torch.Generator().manual_seed(404)
    sd = {f"p.{n}_proj.weight": (0.05 * torch.randn(*s, generator=g)).to(torch.float16)
          for n, s in (("q", (64, 96)), ("k", (32, 96)), ("v", (32, 96)), ("gate", (80, 96)), ("up", (80, 96)))}
    qkv = L.weights.qkv_weight(sd, "p")
    gu = L.weights.gate_up_weight(sd, "p")
    pre = L.weights.merge_qtensor([L.weights.to_qtensor(sd["p.gate_proj.weight"]),
                                   L.weights.to_qtensor(sd["p.up_proj.weight"])])
    out = {k.replace(".", "_"): _np(v) for k, v in sd.items()}
    out.update({"qkv_q": _np(qkv.data), "qkv_s": _np(qkv.scale), "gu_q": _np(gu.data), "gu_s": _np(gu.scale),
                "gu_pre_q": _np(pre.data), "gu_pre_s": _np(pre.scale)})
    return out


def gen_i8_fixture(ref: str, L) -> dict:
    """The reference tests' own weight-quant helpers, called directly."""
    tl = _load_test_module(ref, "test_layers.py", L)
    ts = _load_test_module(ref, "test_smoke.py", L)
    torch.manual_seed(505)
    w_l = torch.randn(128, 256, dtype=torch.float16)
    torch.manual_seed(505)
    qt_l, deq_l = tl._i8(128, 256)
    torch.manual_seed(506)
    w_s = torch.randn(128, 256)
    torch.manual_seed(506)
    qt_s = ts._i8(128, 256)
    return {"layers_w": _np(w_l), "layers_q": _np(qt_l.data), "layers_s": _np(qt_l.scale), "layers_deq": _np(deq_l),
            "smoke_w": _np(w_s), "smoke_q": _np(qt_s.data), "smoke_s": _np(qt_s.scale)}


def gen_moe(L, scoring: str) -> dict:
    g = torch.Generator().manual_seed(606 if scoring == "softmax" else 607)
    E, k, H, I = 8, 2, 256, 128
    B, S = 2, 16
    sd = {}
    for e in range(E):
        sd[f"e{e}.gate_proj.weight"] = (0.05 * torch.randn(I, H, generator=g)).to(torch.float16)
        sd[f"e{e}.up_proj.weight"] = (0.05 * torch.randn(I, H, generator=g)).to(torch.float16)
        sd[f"e{e}.down_proj.weight"] = (0.05 * torch.randn(H, I, generator=g)).to(torch.float16)
    experts = [(L.weights.gate_up_weight(sd, f"e{e}"), L.weights.to_qtensor(sd[f"e{e}.down_proj.weight"]))
               for e in range(E)]
    gate = (0.05 * torch.randn(E, H, generator=g)).to(torch.float16)
    kw = {}
    bias = None
    if scoring == "sigmoid":
        bias = 0.1 * torch.randn(E, generator=g)
        kw = dict(scoring_func="sigmoid", e_score_correction_bias=bias, num_expert_groups=2, topk_group=1)
    moe = L.moe.SparseMoE(gate=gate, experts=experts, top_k=k, norm_topk_prob=True, **kw)
    x = torch.randn(B, S, H, generator=g).to(torch.float16)
    captured = {}
    real_topk = torch.topk

    def spy(inp, kk, *a, **kws):  # record the routing choice made inside moe.py
        r = real_topk(inp, kk, *a, **kws)
        if kk == k and inp.shape[-1] == E:
            captured["topi"] = r[1].clone()
        return r

    torch.topk = spy
    try:
        y = moe(x)
    finally:
        torch.topk = real_topk
    out = {"x": _np(x), "gate": _np(gate), "y": _np(y), "topi": _np(captured["topi"]),
           "w_gu": np.stack([_np(gu.data) for gu, _ in experts]), "s_gu": np.stack([_np(gu.scale) for gu, _ in experts]),
           "w_dn": np.stack([_np(dn.data) for _, dn in experts]), "s_dn": np.stack([_np(dn.scale) for _, dn in experts]),
           "E": np.array(E), "k": np.array(k)}
    if bias is not None:
        out["bias"] = _np(bias)
    return out


def gen_moe_combine(L) -> dict:
    """The reference's expert loop with each expert's output recorded (a forward hook on
    every GatedMLP): y_slot[t, j] is the contribution of the expert in slot j of token t,
    y the block output the loop accumulated in fp16 with index_add_ in expert order
    (fni8serve/models/moe.py:97-105). Four slots per token, so each output element is a
    sum of four rounded products."""
    g = torch.Generator().manual_seed(608)
    E, k, H, I = 8, 4, 64, 32
    B, S = 4, 32
    sd = {}
    for e in range(E):
        sd[f"e{e}.gate_proj.weight"] = (0.2 * torch.randn(I, H, generator=g)).to(torch.float16)
        sd[f"e{e}.up_proj.weight"] = (0.2 * torch.randn(I, H, generator=g)).to(torch.float16)
        sd[f"e{e}.down_proj.weight"] = (0.2 * torch.randn(H, I, generator=g)).to(torch.float16)
    experts = [(L.weights.gate_up_weight(sd, f"e{e}"), L.weights.to_qtensor(sd[f"e{e}.down_proj.weight"]))
               for e in range(E)]
    gate = (0.3 * torch.randn(E, H, generator=g)).to(torch.float16)
    moe = L.moe.SparseMoE(gate=gate, experts=experts, top_k=k, norm_topk_prob=True)
    x = torch.randn(B, S, H, generator=g).to(torch.float16)
    T = B * S
    captured = {}
    real_topk = torch.topk

    def spy(inp, kk, *a, **kws):
        r = real_topk(inp, kk, *a, **kws)
        if kk == k and inp.shape[-1] == E:
            captured["topi"] = r[1].clone()
        return r

    outs = {}
    hooks = [m.register_forward_hook(lambda mod, inp, out, e=e: outs.__setitem__(e, out.detach().clone()))
             for e, m in enumerate(moe.experts)]
    torch.topk = spy
    try:
        y = moe(x)
    finally:
        torch.topk = real_topk
        for h in hooks:
            h.remove()
    topi = captured["topi"]
    y_slot = torch.zeros(T, k, H, dtype=torch.float16)
    for e, o in outs.items():
        tok, slot = (topi == e).nonzero(as_tuple=True)  # the loop's own row order
        y_slot[tok, slot] = o.reshape(-1, H)
    logits = F.linear(x.reshape(-1, H).float(), gate.float())
    return {"x": _np(x), "gate": _np(gate), "logits": _np(logits), "topi": _np(topi), "y_slot": _np(y_slot),
            "y": _np(y), "E": np.array(E), "k": np.array(k)}


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--reference", default=os.environ.get("FNI8_REFERENCE"),
                    help="fni8-serve checkout (default: $FNI8_REFERENCE)")
    ap.add_argument("--only", nargs="*", help="fixture names to (re)write (default: all)")
    a = ap.parse_args()
    if a.reference is None:
        print("pass --reference <fni8-serve checkout> or set FNI8_REFERENCE", file=sys.stderr)
        return 2
    if not os.path.isdir(os.path.join(a.reference, "fni8serve")):
        print(f"fni8-serve sources not found under {a.reference}", file=sys.stderr)
        return 2
    torch.set_num_threads(4)
    L = _setup(a.reference)
    jobs = {"rmsnorm": lambda: gen_rmsnorm(L), "act": lambda: gen_act(L), "linear": lambda: gen_linear(L),
            "linear_i4": lambda: gen_linear_i4(L), "linear_nf4": lambda: gen_linear_nf4(L),
            "convert": lambda: gen_convert(L), "weights": lambda: gen_weights(L), "i8_fixture": lambda: gen_i8_fixture(a.reference, L),
            "moe_softmax": lambda: gen_moe(L, "softmax"), "moe_sigmoid": lambda: gen_moe(L, "sigmoid"),
            "moe_shared": lambda: gen_moe_shared(L), "moe_combine": lambda: gen_moe_combine(L)}
    unknown = set(a.only or ()) - set(jobs)
    if unknown:
        print(f"unknown fixtures {sorted(unknown)}; known: {sorted(jobs)}", file=sys.stderr)
        return 2
    for name, fn in jobs.items():
        if a.only and name not in a.only:
            continue
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **fn())
        print(f"wrote {path} ({os.path.getsize(path)} bytes)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
