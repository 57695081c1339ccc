"""Torch-facing wrappers of the sm_100a W8A8 kernels.

These are the functions fni8-serve's layers import from `fni8`:

    fni8.linear(x, qt, bias=None)                         fni8serve/layers/linear.py:67-69
    fni8.rmsnorm(x, w, eps, residual=None, unit_offset=)   fni8serve/layers/norm.py:45-58
    fni8.act_and_mul(x, "silu" | "gelu_tanh")              fni8serve/layers/activation.py:21-41

plus the fused producers the reference does not have (`rmsnorm_quant`,
`act_and_mul_quant`, `linear_q`) and raw access for tests (`quantize_rows`,
`gemm_i32`). Every op runs on the current CUDA stream, allocates its outputs from the
PyTorch caching allocator and never synchronises, so the decode step can be captured in
a CUDA graph as the reference engine does (fni8serve/engine/cuda_graph.py). CPU tensors
are rejected: the reference routes CPU inputs to its own fp16 fallback before calling
`fni8` (linear.py:58-71, norm.py:48-58, activation.py:15-25), and this package has no
CPU path of its own.
"""
from __future__ import annotations

import ctypes
import threading

import torch

from . import _native as nat
from .qtensor import QTensor

_DT = {torch.float16: nat.F16, torch.bfloat16: nat.BF16}
_ACT = {"silu": nat.ACT_SILU, "gelu_tanh": nat.ACT_GELU_TANH, "gelu_pytorch_tanh": nat.ACT_GELU_TANH}

# Fused int8 hand-off: fni8.rmsnorm and fni8.act_and_mul can leave the int8 rows and
# scales of their output on the tensor, so the fni8.linear that consumes it (QKV / gate_up
# after the norm, down after the activation) skips its own quantisation pass. The side-car
# is only trusted while the tensor is unmodified (same storage, shape and version counter).
FUSE_NORM_QUANT = True
FUSE_ACT_QUANT = True
_SIDECAR_MIN_K = 512


def _vp(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(dev: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _need_cuda(x: torch.Tensor, what: str) -> None:
    if not x.is_cuda:
        raise RuntimeError(f"fni8.{what}: expected a CUDA tensor (fni8-serve_b200 has no CPU path)")


def _act_dtype(x: torch.Tensor, what: str) -> int:
    try:
        return _DT[x.dtype]
    except KeyError:
        raise TypeError(f"fni8.{what}: activations must be float16 or bfloat16, got {x.dtype}") from None


# ------------------------------------------------------------------ GEMM workspace
class _Workspace:
    """Per-device GEMM workspace: zeroed once, kept zero by the kernels, never freed.

    Sized for the largest decode problem (M <= 256) of the stream-K kernel and of the
    split-K kernel, so it is allocated once, before any CUDA-graph capture, and reused by
    every call. Calls on different streams of one device must not overlap while they
    share it.
    """

    def __init__(self):
        self._bufs: dict[int, torch.Tensor] = {}
        self._lock = threading.Lock()

    def get(self, dev: torch.device) -> torch.Tensor:
        idx = dev.index if dev.index is not None else torch.cuda.current_device()
        buf = self._bufs.get(idx)
        if buf is None:
            with self._lock:
                buf = self._bufs.get(idx)
                if buf is None:
                    # stream-K: G slots of 128 x 256 int32 + G counters, G <= SM count;
                    # split-K: one 128 x 256 int32 slab per CTA, up to 2 CTAs per SM
                    sms = torch.cuda.get_device_properties(idx).multi_processor_count
                    nbytes = 2 * sms * (128 * 256 + 1) * 4
                    buf = torch.zeros(nbytes, dtype=torch.uint8, device=torch.device("cuda", idx))
                    self._bufs[idx] = buf
        return buf


WORKSPACE = _Workspace()


def _ws(dev: torch.device):
    buf = WORKSPACE.get(dev)
    return ctypes.c_void_p(buf.data_ptr()), ctypes.c_size_t(buf.numel())


# ------------------------------------------------------------------ quantisers
def quantize_rows(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-token absmax int8 quantisation of x[..., K] -> (q int8 [..., K], scale fp32 [...])."""
    _need_cuda(x, "quantize_rows")
    dt = _act_dtype(x, "quantize_rows")
    K = x.shape[-1]
    x2 = x.reshape(-1, K).contiguous()
    M = x2.shape[0]
    q = torch.empty((M, K), dtype=torch.int8, device=x.device)
    s = torch.empty((M,), dtype=torch.float32, device=x.device)
    nat.call("fni8_quantize_rows_i8", _vp(x2), dt, M, K, _vp(q), _vp(s), _stream(x.device))
    return q.reshape(*x.shape), s.reshape(x.shape[:-1])


def _attach_sidecar(y: torch.Tensor, q: torch.Tensor, s: torch.Tensor) -> None:
    y._fni8_q = (q, s, y.data_ptr(), tuple(y.shape), y._version)


def _sidecar(x: torch.Tensor):
    sc = getattr(x, "_fni8_q", None)
    if sc is None:
        return None
    q, s, ptr, shape, ver = sc
    if ptr != x.data_ptr() or shape != tuple(x.shape) or ver != x._version:
        return None
    return q, s


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, residual: torch.Tensor | None = None,
            unit_offset: bool = False):
    """fni8.rmsnorm: returns the normed tensor, or (normed, x + residual) with a residual."""
    return _rmsnorm(x, w, eps, residual, unit_offset, quant=FUSE_NORM_QUANT)


def rmsnorm_quant(x: torch.Tensor, w: torch.Tensor, eps: float, residual: torch.Tensor | None = None,
                  unit_offset: bool = False, keep_normed: bool = False):
    """Fused RMSNorm -> per-token int8: returns (q, scale[, new_residual][, normed])."""
    _need_cuda(x, "rmsnorm_quant")
    dt = _act_dtype(x, "rmsnorm_quant")
    K = x.shape[-1]
    x2 = x.reshape(-1, K).contiguous()
    M = x2.shape[0]
    wv = w.to(device=x.device, dtype=x.dtype).contiguous()
    q = torch.empty((M, K), dtype=torch.int8, device=x.device)
    s = torch.empty((M,), dtype=torch.float32, device=x.device)
    y = torch.empty_like(x2) if keep_normed else None
    r2 = ro = None
    if residual is not None:
        r2 = residual.reshape(-1, K).to(x.dtype).contiguous()
        ro = torch.empty_like(x2)
    nat.call("fni8_rmsnorm_quant_i8", _vp(x2), _vp(r2), _vp(wv), dt, M, K, ctypes.c_float(eps), int(unit_offset),
             _vp(y), _vp(ro), _vp(q), _vp(s), _stream(x.device))
    out = [q.reshape(*x.shape), s.reshape(x.shape[:-1])]
    if ro is not None:
        out.append(ro.reshape(x.shape))
    if y is not None:
        out.append(y.reshape(x.shape))
    return tuple(out)


def _rmsnorm(x, w, eps, residual, unit_offset, quant):
    _need_cuda(x, "rmsnorm")
    dt = _act_dtype(x, "rmsnorm")
    K = x.shape[-1]
    x2 = x.reshape(-1, K).contiguous()
    M = x2.shape[0]
    wv = w.to(device=x.device, dtype=x.dtype).contiguous()
    y = torch.empty_like(x2)
    r2 = ro = None
    if residual is not None:
        r2 = residual.reshape(-1, K).to(x.dtype).contiguous()
        ro = torch.empty_like(x2)
    st = _stream(x.device)
    use_q = quant and K >= _SIDECAR_MIN_K and K % 16 == 0
    if use_q:
        q = torch.empty((M, K), dtype=torch.int8, device=x.device)
        s = torch.empty((M,), dtype=torch.float32, device=x.device)
        nat.call("fni8_rmsnorm_quant_i8", _vp(x2), _vp(r2), _vp(wv), dt, M, K, ctypes.c_float(eps),
                 int(unit_offset), _vp(y), _vp(ro), _vp(q), _vp(s), st)
    else:
        nat.call("fni8_rmsnorm", _vp(x2), _vp(r2), _vp(wv), dt, M, K, ctypes.c_float(eps), int(unit_offset), _vp(y),
                 _vp(ro), st)
    y = y.reshape(x.shape)
    if use_q:
        _attach_sidecar(y, q, s)
    if ro is None:
        return y
    return y, ro.reshape(x.shape)


def act_and_mul(x: torch.Tensor, act: str = "silu") -> torch.Tensor:
    """fni8.act_and_mul: act(x[..., :I]) * x[..., I:] for the merged gate_up output."""
    _need_cuda(x, "act_and_mul")
    dt = _act_dtype(x, "act_and_mul")
    if act not in _ACT:
        raise ValueError(f"fni8.act_and_mul: unsupported activation {act!r}")
    two_i = x.shape[-1]
    if two_i % 2:
        raise ValueError("fni8.act_and_mul: last dim must be even (gate | up)")
    I = two_i // 2
    x2 = x.reshape(-1, two_i).contiguous()
    M = x2.shape[0]
    out = torch.empty((M, I), dtype=x.dtype, device=x.device)
    use_q = FUSE_ACT_QUANT and I >= _SIDECAR_MIN_K and I % 16 == 0
    if use_q:
        # the down projection that consumes the product finds its int8 rows ready
        q = torch.empty((M, I), dtype=torch.int8, device=x.device)
        s = torch.empty((M,), dtype=torch.float32, device=x.device)
        nat.call("fni8_act_and_mul_dual", _vp(x2), dt, _ACT[act], M, I, _vp(out), _vp(q), _vp(s), _stream(x.device))
    else:
        nat.call("fni8_act_and_mul", _vp(x2), dt, _ACT[act], M, I, _vp(out), _stream(x.device))
    y = out.reshape(*x.shape[:-1], I)
    if use_q:
        _attach_sidecar(y, q.reshape(*x.shape[:-1], I), s.reshape(x.shape[:-1]))
    return y


def act_and_mul_quant(x: torch.Tensor, act: str = "silu") -> tuple[torch.Tensor, torch.Tensor]:
    """Fused act_and_mul -> per-token int8: (q int8 [..., I], scale fp32 [...])."""
    _need_cuda(x, "act_and_mul_quant")
    dt = _act_dtype(x, "act_and_mul_quant")
    if act not in _ACT:
        raise ValueError(f"fni8.act_and_mul_quant: unsupported activation {act!r}")
    I = x.shape[-1] // 2
    x2 = x.reshape(-1, 2 * I).contiguous()
    M = x2.shape[0]
    q = torch.empty((M, I), dtype=torch.int8, device=x.device)
    s = torch.empty((M,), dtype=torch.float32, device=x.device)
    nat.call("fni8_act_and_mul_quant_i8", _vp(x2), dt, _ACT[act], M, I, _vp(q), _vp(s), _stream(x.device))
    return q.reshape(*x.shape[:-1], I), s.reshape(x.shape[:-1])


# ------------------------------------------------------------------ GEMMs
def _check_weight(qt: QTensor, x_dev: torch.device, K: int, what: str) -> None:
    if qt.scheme != "per_row_i8":
        raise NotImplementedError(f"fni8.{what}: scheme {qt.scheme!r} is not implemented on sm_100a "
                                  "(per_row_i8 here; per_group_i4 through fni8.linear)")
    if qt.data.dtype != torch.int8 or qt.data.dim() != 2:
        raise TypeError(f"fni8.{what}: per_row_i8 data must be a 2-D int8 tensor")
    if qt.data.shape[1] != K:
        raise ValueError(f"fni8.{what}: in_features {qt.data.shape[1]} != activation K {K}")
    if qt.data.device != x_dev or qt.scale.device != x_dev:
        raise RuntimeError(f"fni8.{what}: weight and activation are on different devices")
    if not qt.data.is_contiguous() or not qt.scale.is_contiguous() or qt.scale.dtype != torch.float32:
        raise TypeError(f"fni8.{what}: weight data/scale must be contiguous (scale fp32)")


def _k16_weight(qt: QTensor, K: int) -> tuple[torch.Tensor, int]:
    """(weight, K) with K a multiple of 16, the row-stride rule of the GEMMs' TMA maps.
    fni8-serve accepts any K that is a multiple of 4 (convert.py:128); zero input channels
    add nothing to the int32 sums (nor to a token's absmax), so a weight padded with zero
    columns, and activations padded with zeros, give the same outputs bit for bit. The
    padded weight is built on the first call and kept on the QTensor (call once before a
    CUDA-graph capture, like the GEMM workspace); it is rebuilt if the weight tensor is
    replaced or modified in place."""
    if K % 16 == 0:
        return qt.data, K
    Kp = (K + 15) // 16 * 16
    cached = getattr(qt, "_fni8_k16", None)
    if cached is not None and cached[0] is qt.data and cached[1] == qt.data._version:
        return cached[2], Kp
    wp = torch.zeros((qt.data.shape[0], Kp), dtype=torch.int8, device=qt.data.device)
    wp[:, :K] = qt.data
    qt._fni8_k16 = (qt.data, qt.data._version, wp)
    return wp, Kp


def linear_q(q: torch.Tensor, scale: torch.Tensor, qt: QTensor, bias: torch.Tensor | None = None,
             residual: torch.Tensor | None = None, out_dtype: torch.dtype = torch.float16,
             path: int = nat.PATH_AUTO) -> torch.Tensor:
    """W8A8 GEMM on pre-quantised activations q[..., K] (int8) with per-token scale[...]."""
    _need_cuda(q, "linear_q")
    K = q.shape[-1]
    _check_weight(qt, q.device, K, "linear_q")
    w, Kp = _k16_weight(qt, K)
    q2 = q.reshape(-1, K).contiguous()
    if Kp != K:
        q2 = torch.nn.functional.pad(q2, (0, Kp - K))
    s2 = scale.reshape(-1).to(torch.float32).contiguous()
    M, N = q2.shape[0], qt.data.shape[0]
    odt = _DT[out_dtype]
    out = torch.empty((M, N), dtype=out_dtype, device=q.device)
    b = bias.to(out_dtype).contiguous() if bias is not None else None
    r = residual.reshape(M, N).to(out_dtype).contiguous() if residual is not None else None
    ws, wsb = _ws(q.device)
    nat.call("fni8_gemm_w8a8_ex", _vp(q2), _vp(s2), _vp(w), _vp(qt.scale), _vp(b), _vp(r), _vp(out), odt, M, N,
             Kp, path, ws, wsb, _stream(q.device))
    return out.reshape(*q.shape[:-1], N)


def linear_act_q(q: torch.Tensor, scale: torch.Tensor, gate_up: QTensor, act: str = "silu",
                 out_dtype: torch.dtype = torch.float16) -> torch.Tensor:
    """act_and_mul(gate_up(x)) on pre-quantised activations q[..., K] with per-token scale:
    the merged gate_up weight [2I, K] (gate rows first, fni8serve/models/weights.py:49-50)
    runs on the tile GEMM whose epilogue applies act(gate) * up, so only the [..., I]
    product is written. Equal bit for bit to act_and_mul(linear_q(q, scale, gate_up)).
    Needs I % 128 == 0 and no bias (fni8.mlp.GatedMLP checks both)."""
    _need_cuda(q, "linear_act_q")
    if act not in _ACT:
        raise ValueError(f"fni8.linear_act_q: unsupported activation {act!r}")
    K = q.shape[-1]
    _check_weight(gate_up, q.device, K, "linear_act_q")
    w, Kp = _k16_weight(gate_up, K)
    q2 = q.reshape(-1, K).contiguous()
    if Kp != K:
        q2 = torch.nn.functional.pad(q2, (0, Kp - K))
    s2 = scale.reshape(-1).to(torch.float32).contiguous()
    M, I = q2.shape[0], gate_up.data.shape[0] // 2
    out = torch.empty((M, I), dtype=out_dtype, device=q.device)
    nat.call("fni8_gemm_w8a8_act", _vp(q2), _vp(s2), _vp(w), _vp(gate_up.scale), _ACT[act], _vp(out), _DT[out_dtype],
             M, I, Kp, _stream(q.device))
    return out.reshape(*q.shape[:-1], I)


def linear_q_peer_cols(q: torch.Tensor, scale: torch.Tensor, shard: QTensor, peers, n_peers: int, ld: int,
                       col_off: int, bias: torch.Tensor | None = None, out_dtype: torch.dtype = torch.float16) -> None:
    """W8A8 GEMM of a column shard on pre-quantised rows q[M, K] whose output element (m, n)
    is stored to element (m, col_off + n) of each of the n_peers buffers in `peers` (a ctypes
    array of device pointers; row stride ld elements; this GPU's own or NVLink peers' memory):
    the shard's part of a column all-gather, computed and sent in one call
    (C: fni8_gemm_w8a8_peer_cols). Nothing is returned."""
    _need_cuda(q, "linear_q_peer_cols")
    K = q.shape[-1]
    _check_weight(shard, q.device, K, "linear_q_peer_cols")
    w, Kp = _k16_weight(shard, K)
    q2 = q.reshape(-1, K).contiguous()
    if Kp != K:
        q2 = torch.nn.functional.pad(q2, (0, Kp - K))
    s2 = scale.reshape(-1).to(torch.float32).contiguous()
    M, N = q2.shape[0], shard.data.shape[0]
    b = bias.to(out_dtype).contiguous() if bias is not None else None
    # decode sizes run the split-K GEMM into a local [M, N] buffer before the copy out
    tmp = torch.empty((M, N), dtype=out_dtype, device=q.device) if M <= 256 else None
    ws, wsb = _ws(q.device)
    nat.call("fni8_gemm_w8a8_peer_cols", _vp(q2), _vp(s2), _vp(w), _vp(shard.scale), _vp(b), _DT[out_dtype], M, N, Kp,
             peers, n_peers, ld, col_off, _vp(tmp), tmp.numel() * 2 if tmp is not None else 0, ws, wsb,
             _stream(q.device))


def _linear_w4a8(x: torch.Tensor, qt: QTensor, bias: torch.Tensor | None) -> torch.Tensor:
    """per_group_i4 / int4 weights (W4A8): packed data [N, K/2] uint8, scale [N, K/g] fp32."""
    if qt.codebook not in (None, "int4"):
        raise NotImplementedError(f"fni8.linear: per_group_i4 codebook {qt.codebook!r} has no integer GEMM "
                                  "(fni8-serve routes NF4 weights to its fp16 fallback)")
    dt = _act_dtype(x, "linear")
    K = x.shape[-1]
    if qt.data.dim() != 2 or qt.data.shape[1] * 2 != K or qt.data.dtype not in (torch.uint8, torch.int8):
        raise ValueError(f"fni8.linear: per_group_i4 data {tuple(qt.data.shape)} does not pack K={K}")
    if qt.data.device != x.device or qt.scale.device != x.device:
        raise RuntimeError("fni8.linear: weight and activation are on different devices")
    N = qt.data.shape[0]
    gs = int(qt.group_size or 0)
    ws_ = qt.scale.to(torch.float32).contiguous()
    if gs <= 0 or K % gs or ws_.numel() != N * (K // gs):
        raise ValueError(f"fni8.linear: per_group_i4 scale {tuple(qt.scale.shape)} does not match N={N}, "
                         f"K={K}, group_size={gs}")
    x2 = x.reshape(-1, K).contiguous()
    M = x2.shape[0]
    out = torch.empty((M, N), dtype=x.dtype, device=x.device)
    q = torch.empty((M, K), dtype=torch.int8, device=x.device)
    s = torch.empty((M,), dtype=torch.float32, device=x.device)
    b = bias.to(x.dtype).contiguous() if bias is not None else None
    ws, wsb = _ws(x.device)
    nat.call("fni8_linear_w4a8", _vp(x2), dt, _vp(qt.data.contiguous()), _vp(ws_), gs, _vp(b), _vp(out), M, N, K,
             _vp(q), _vp(s), ws, wsb, _stream(x.device))
    return out.reshape(*x.shape[:-1], N)


def linear(x: torch.Tensor, qt: QTensor, bias: torch.Tensor | None = None, path: int = nat.PATH_AUTO) -> torch.Tensor:
    """fni8.linear: per-token int8 quantisation of x, int8 GEMM, dequant epilogue (+bias).

    `path` (not in the reference signature) forces a kernel; the default picks by shape.
    per_group_i4 / int4 weights run the W4A8 GEMM."""
    _need_cuda(x, "linear")
    if qt.scheme == "per_group_i4":
        return _linear_w4a8(x, qt, bias)
    dt = _act_dtype(x, "linear")
    K = x.shape[-1]
    _check_weight(qt, x.device, K, "linear")
    N = qt.data.shape[0]
    sc = _sidecar(x) if path == nat.PATH_AUTO else None
    if sc is not None:
        return linear_q(sc[0], sc[1], qt, bias=bias, out_dtype=x.dtype).reshape(*x.shape[:-1], N)
    w, Kp = _k16_weight(qt, K)
    x2 = x.reshape(-1, K).contiguous()
    if Kp != K:
        x2 = torch.nn.functional.pad(x2, (0, Kp - K))
    M = x2.shape[0]
    out = torch.empty((M, N), dtype=x.dtype, device=x.device)
    q = torch.empty((M, Kp), dtype=torch.int8, device=x.device)
    s = torch.empty((M,), dtype=torch.float32, device=x.device)
    b = bias.to(x.dtype).contiguous() if bias is not None else None
    ws, wsb = _ws(x.device)
    nat.call("fni8_linear_w8a8_ex", _vp(x2), dt, _vp(w), _vp(qt.scale), _vp(b), _vp(out), M, N, Kp, _vp(q),
             _vp(s), path, ws, wsb, _stream(x.device))
    return out.reshape(*x.shape[:-1], N)


def gemm_i32(a: torch.Tensor, w: torch.Tensor, path: int = nat.PATH_AUTO) -> torch.Tensor:
    """Raw int32 accumulators a[M, K] @ w[N, K]^T (bit-exact check of the int8 MMA)."""
    _need_cuda(a, "gemm_i32")
    if a.dtype != torch.int8 or w.dtype != torch.int8:
        raise TypeError("fni8.gemm_i32: int8 operands expected")
    a2, w2 = a.contiguous(), w.contiguous()
    M, K = a2.shape
    N = w2.shape[0]
    out = torch.empty((M, N), dtype=torch.int32, device=a.device)
    ws, wsb = _ws(a.device)
    nat.call("fni8_gemm_w8a8_i32", _vp(a2), _vp(w2), _vp(out), M, N, K, path, ws, wsb, _stream(a.device))
    return out


def device_status() -> int:
    """Synchronise and return (and clear) the device watchdog code of the current device;
    0 means healthy. A non-zero code means a kernel left its loop on a timed-out wait and
    its outputs are void; the abandoned kernel may have left partial sums in the GEMM
    workspace, so this device's WORKSPACE is zeroed again before the next GEMM reads it
    (the library re-zeroes its own allocation-free scratch)."""
    code = ctypes.c_int(0)
    st = nat.lib().fni8_device_status(ctypes.byref(code))
    if st not in (nat.OK, nat.ERR_DEVICE_TIMEOUT):
        nat.check(st, "fni8_device_status")
    if code.value != 0:
        buf = WORKSPACE._bufs.get(torch.cuda.current_device())
        if buf is not None:
            buf.zero_()
            torch.cuda.synchronize()
    return code.value


def watchdog_selftest(wait_us: int = 20000, dirty_scratch: bool = False) -> None:
    """Launch the failure-detection self-test on the current stream: a kernel whose bounded
    wait on a flag that nothing sets gives up after `wait_us` and records a watchdog code
    (read it with device_status()); with dirty_scratch it first leaves non-zero partial
    sums in the allocation-free GEMM's scratch, as an abandoned reduction would."""
    nat.call("fni8_watchdog_selftest", int(wait_us), int(bool(dirty_scratch)),
             _stream(torch.device("cuda", torch.cuda.current_device())))
