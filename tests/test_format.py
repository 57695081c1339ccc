"""The `.fni8` container (fni8.format): the call contract fni8-serve's loader, converter
and tools use (fni8serve/loader.py:16-69, convert.py:320-356, tools/fine_tune.py:55-58),
the round trips its own tests make (tests/test_smoke.py:36-62) and the reader's checks.
The byte format itself is this library's (the original is defined inside the absent
`fni8` package), so these tests pin the contract, not the bytes. Runs without a GPU."""
import os

import pytest
import torch

from fni8 import FQReader, FQWriter, QTensor, save_fni8


def _i8(n, k, seed=0):
    g = torch.Generator().manual_seed(seed)
    return QTensor(torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8), torch.rand(n, generator=g) * 1e-2)


def _i4(n, k, group, seed=1):
    g = torch.Generator().manual_seed(seed)
    packed = torch.randint(0, 256, (n, k // 2), generator=g, dtype=torch.int64).to(torch.uint8)
    return QTensor(packed, torch.rand(n, k // group, generator=g), scheme="per_group_i4", group_size=group,
                   codebook="int4")


def _same(a: QTensor, b: QTensor):
    assert a.scheme == b.scheme and a.group_size == b.group_size and a.codebook == b.codebook
    assert a.data.dtype == b.data.dtype and torch.equal(a.data, b.data)
    assert (a.scale is None) == (b.scale is None)
    if a.scale is not None:
        assert a.scale.dtype == b.scale.dtype and torch.equal(a.scale, b.scale)


def _load_checkpoint(path, names=None, shard=None):
    """fni8serve/loader.py:19-43 (load_fni8_checkpoint) restated on the same calls."""
    with FQReader(path) as r:
        if shard is not None:
            idx = r.shards
            if shard in idx.get("experts", {}):
                names = idx["experts"][shard]
            elif shard.startswith("pp:"):
                names = idx["pp_stages"][int(shard[3:])]
            else:
                raise KeyError(shard)
        names = names if names is not None else r.names
        return r.load_many(names, "cpu")


def test_round_trip_every_scheme_and_dtype(tmp_path):
    path = str(tmp_path / "m.fni8")
    ts = {
        "mlp.up.weight": _i8(128, 256),
        "mlp.down.weight": _i4(64, 128, 32),
        "norm.weight": QTensor(torch.randn(256).half(), None, scheme="raw"),
        "embed.weight": QTensor(torch.randn(10, 16, dtype=torch.bfloat16), None, scheme="raw"),
        "router.bias": torch.randn(8),  # plain tensors are stored raw
        "step": torch.tensor(7, dtype=torch.int64),  # 0-dim
        "mask": torch.tensor([True, False, True]),
        "empty": torch.empty(0, 4),
    }
    save_fni8(path, ts)
    with FQReader(path) as r:
        assert r.names == list(ts)
        got = r.load_many(r.names, "cpu")
    for name, t in ts.items():
        want = t if isinstance(t, QTensor) else QTensor(t, None, scheme="raw")
        _same(got[name], want)


def test_header_fields_and_meta(tmp_path):
    path = str(tmp_path / "m.fni8")
    meta = {"arch": "qwen3", "weight_bits": 8, "config": {"hidden_size": 4096, "num_hidden_layers": 36}}
    save_fni8(path, {"a.weight": _i8(32, 64)}, meta=meta)
    with FQReader(path) as r:
        h = r.header
        assert h["arch"] == "qwen3" and h["quant"] == "int8" and h["version"] == 1
        assert h["__meta__"] == meta
        assert h["hidden_size"] == 4096  # model dimensions readable from the header
    save_fni8(path, {"a.weight": _i4(32, 64, 32)})
    with FQReader(path) as r:
        assert r.header["quant"] == "int4" and r.header["arch"] == "" and r.header["__meta__"] == {}


def test_shard_partial_loads(tmp_path):
    path = str(tmp_path / "m.fni8")
    ts = {f"model.layers.{i}.w": _i8(32, 64, seed=i) for i in range(4)}
    ts.update({f"experts.{e}.gate_up": _i8(16, 64, seed=10 + e) for e in range(3)})
    shards = {"pp_stages": [["model.layers.0.w", "model.layers.1.w"], ["model.layers.2.w", "model.layers.3.w"]],
              "experts": {"1": ["experts.1.gate_up"], "2": ["experts.2.gate_up"]}}
    save_fni8(path, ts, shards=shards)
    w = _load_checkpoint(path, shard="pp:1")
    assert set(w) == {"model.layers.2.w", "model.layers.3.w"}
    _same(w["model.layers.3.w"], ts["model.layers.3.w"])
    w = _load_checkpoint(path, shard="2")
    assert set(w) == {"experts.2.gate_up"}
    assert set(_load_checkpoint(path)) == set(ts)
    with pytest.raises(KeyError):
        _load_checkpoint(path, shard="nope")
    with pytest.raises(KeyError):
        save_fni8(path, ts, shards={"pp_stages": [["missing.w"]]})


def test_streaming_writer(tmp_path):
    """The converter's pattern: add tensors one by one, then finalize(meta=)."""
    path = str(tmp_path / "m.fni8")
    parts = [(f"layer{i}.w", _i8(64, 128, seed=i)) for i in range(5)]
    with FQWriter(path) as w:
        for name, qt in parts:
            w.add(name, qt)
        w.finalize(meta={"arch": "qwen3_moe", "weight_bits": 8})
    with FQReader(path) as r:
        assert r.header["arch"] == "qwen3_moe" and r.names == [n for n, _ in parts]
        for name, qt in parts:
            _same(r.load(name), qt)
    with FQWriter(path) as w:  # finalize is implied on a clean exit
        w.add("x", _i8(8, 16))
    with FQReader(path) as r:
        assert r.names == ["x"]


def test_data_parts_are_page_aligned(tmp_path):
    path = str(tmp_path / "m.fni8")
    save_fni8(path, {"a": _i8(3, 17), "b": _i8(5, 33), "c": QTensor(torch.randn(7).half(), None, scheme="raw")})
    with FQReader(path) as r:
        for e in r.header["tensors"].values():
            for part in (e["data"], e["scale"]):
                if part is not None:
                    assert part["offset"] % 4096 == 0


def test_rejects_corrupt_and_foreign_files(tmp_path):
    bad = tmp_path / "x.fni8"
    bad.write_bytes(b"not a container at all" * 4)
    with pytest.raises(ValueError, match="not a .fni8"):
        FQReader(str(bad))
    good = str(tmp_path / "m.fni8")
    save_fni8(good, {"a": _i8(8, 16)})
    raw = open(good, "rb").read()
    trunc = tmp_path / "t.fni8"
    trunc.write_bytes(raw[:-5])
    with pytest.raises(ValueError):
        FQReader(str(trunc))


def test_failed_write_leaves_no_file(tmp_path):
    path = str(tmp_path / "m.fni8")
    with pytest.raises(TypeError):
        with FQWriter(path) as w:
            w.add("ok", _i8(8, 16))
            w.add("bad", QTensor(torch.zeros(2, dtype=torch.complex64), None, scheme="raw"))
    assert not os.path.exists(path)
    with FQWriter(path) as w:
        w.add("a", _i8(8, 16))
        with pytest.raises(ValueError, match="duplicate"):
            w.add("a", _i8(8, 16))


def test_quantize_lowbit_feeds_the_converters_int4_packing():
    """fni8.quant.lowbit.quantize_lowbit as fni8serve/convert.py:69-79 calls it: codes and
    per-group scales whose packed form dequantises (linear.py:33-45's code * scale) to the
    oracle's int4 weights, and agrees with the oracle's quantiser exactly."""
    from fni8.quant.lowbit import quantize_lowbit

    from oracle import w8a8_oracle as O

    g = torch.Generator().manual_seed(5)
    w = 0.02 * torch.randn(64, 256, generator=g)
    codes, scale = quantize_lowbit(w, 4, dim=-1, group_size=128)
    assert codes.shape == (64, 256) and scale.shape == (64, 2)
    assert int(codes.min()) >= -8 and int(codes.max()) <= 7
    c = codes.to(torch.int64)
    packed = ((c[:, 0::2] & 0xF) | ((c[:, 1::2] & 0xF) << 4)).to(torch.uint8)  # the converter's packing
    ref_packed, ref_scale = O.quantize_weight_i4(w, 128)
    assert torch.equal(packed, ref_packed) and torch.equal(scale.float(), ref_scale)
    assert torch.equal(O.unpack_i4(packed), codes)
    deq = O.dequant_weight_i4_fallback(packed, scale.float(), 128).float()
    assert (deq - w).abs().max() <= scale.max() * 0.5 + 1e-3  # within half a step
    with pytest.raises(ValueError):
        quantize_lowbit(w, 4, group_size=100)


def test_nf4_codebook_is_normal_float():
    """fni8.quant.lowbit.NF4_CODEBOOK, the table fni8-serve indexes by code for NF4 weights
    (fni8serve/layers/linear.py:22-25,37-39) and NF4 LoRA adapters (training/qlora.py:31,54):
    16 ascending levels in [-1, 1] with an exact zero, 8 above and 7 below it, each the
    quantile of N(0, 1) at evenly spaced probabilities (checked with scipy's normal CDF,
    an implementation independent of the one the module uses)."""
    from scipy.stats import norm

    from fni8.quant.lowbit import NF4_CODEBOOK as cb

    assert len(cb) == 16 and cb == sorted(cb) and cb[0] == -1.0 and cb[-1] == 1.0 and cb[7] == 0.0
    offset = 0.5 * ((1 - 1 / 30) + (1 - 1 / 32))
    top = norm.ppf(offset)
    pos = [norm.cdf(v * top) for v in cb[8:]]      # 8 probabilities above 1/2
    neg = [norm.cdf(-v * top) for v in cb[:7]]     # 7 mirrored probabilities above 1/2
    for probs, count in ((pos, 8), (neg, 7)):
        step = (offset - 0.5) / count
        expect = sorted(0.5 + step * (i + 1) for i in range(count))
        assert max(abs(a - b) for a, b in zip(sorted(probs), expect)) < 1e-12
    # the reference's lookup: a float32 table indexed by 4-bit codes
    t = torch.tensor(cb, dtype=torch.float32)
    codes = torch.arange(16)
    assert torch.equal(t[codes], t) and t.abs().max() == 1.0


@pytest.mark.parametrize("bits", [8, 4])
def test_reference_converter_output_reads_back(golden, tmp_path, bits):
    """Containers written by fni8-serve's own converter (convert_hf_to_fni8 over this
    package's FQWriter, tests/golden/convert.npz) read back here exactly as the reference's
    loader saw them (same names, schemes, header and meta), and hold what the oracle
    computes from the source weights: per-row int8 codes and scales, int4 codes packed two
    per byte low nibble first (the converter's packing, convert.py:69-80), fp16 raw tensors."""
    import json

    import numpy as np

    from fni8 import FQReader
    from oracle import w8a8_oracle as O

    g = golden("convert")
    path = tmp_path / f"m{bits}.fni8"
    path.write_bytes(g[f"file{bits}"].tobytes())
    info = json.loads(str(g[f"info{bits}"]))
    schemes = json.loads(str(g[f"schemes{bits}"]))
    gs = int(g["group_size"])
    src = {n: torch.from_numpy(np.ascontiguousarray(g["src/" + n])).view(torch.bfloat16) for n in g["names"]}
    with FQReader(str(path)) as r:
        assert sorted(r.names) == sorted(src) == sorted(schemes) and len(r.names) == info["num_tensors"]
        assert (r.header["arch"], r.header["quant"], r.header["version"]) == (info["arch"], info["quant"],
                                                                                 info["version"])
        assert r.header.get("__meta__") == info["meta"] and r.shards == {}
        got = r.load_many(r.names, "cpu")
    for name, qt in got.items():
        assert (qt.scheme if qt.scheme != "raw" else "tensor") == schemes[name], name
        w = src[name].float()
        if qt.scheme == "per_row_i8":
            q, s = O.quantize_weight_rowwise(w)
            assert torch.equal(qt.data, q) and torch.equal(qt.scale, s), name
        elif qt.scheme == "per_group_i4":
            packed, s = O.quantize_weight_i4(w, gs)
            assert qt.codebook == "int4" and qt.group_size == gs
            assert torch.equal(qt.data, packed) and torch.equal(qt.scale, s), name
        else:
            assert torch.equal(qt.data, src[name].to(torch.float16)), name


def test_reference_training_checkpoint_reads_back(golden, tmp_path):
    """fni8-serve's training checkpoint writer (save_training_checkpoint, loader.py:75-103:
    raw fp32 weights, optimizer buffers under optimizer.state.*, training meta) over this
    format: the container it wrote reads back with every weight exact and its meta intact."""
    import json

    import numpy as np

    from fni8 import FQReader

    g = golden("convert")
    path = tmp_path / "train.fni8"
    path.write_bytes(g["train_file"].tobytes())
    info = json.loads(str(g["train_info"]))
    sd = {k[len("train_sd/"):]: torch.from_numpy(np.ascontiguousarray(g[k])) for k in g
          if k.startswith("train_sd/")}
    with FQReader(str(path)) as r:
        meta = r.header.get("__meta__")
        assert meta == info["meta"] and meta["training"] is True and meta["step"] == 7
        assert len(r.names) == info["num_tensors"] and set(sd) <= set(r.names)
        assert any(n.startswith("optimizer.state.") for n in r.names)
        got = r.load_many(r.names, "cpu")
    for name, ref in sd.items():
        assert got[name].scheme == "raw" and torch.equal(got[name].data, ref), name
