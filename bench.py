"""Benchmark of the B200 W8A8 path on BASELINE.json's configurations.

    python bench.py [--config C] [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints ONE JSON line (rank 0). BASELINE.json's metric has three parts — prefill TOPS,
decode GB/s, and MoE tokens/s on 1-8 GPUs — and the default run (no --config) reports
all three in one line:

  * top level: BASELINE config 3, the Qwen3-30B-A3B-shaped MoE expert layer (E=128,
    top-8, H=2048, I=768) at 4096 tokens per GPU, expert-parallel over the ranks under
    torchrun (weak scaling: each rank routes its own 4096 tokens and owns E/N experts;
    rows cross NVLink as peer-memory stores). Metric: whole-job tokens/s. This is the
    part of the path that shards, so the 1->8 GPU runs measure it.
  * at N=1 also the keyed sub-blocks "decode" (for each decode batch
    M in {1, 8, 32, 128, 256} the four Qwen3-8B fni8.linear calls QKV 4096->6144,
    O 4096->4096, gate_up 4096->24576, down 12288->4096; 20 linears, 965 MB of distinct
    weights per step; HBM GB/s) and "prefill" (fused RMSNorm+quant ->
    QKV, O, gate_up -> SiLU*up+quant -> down at M=8192; TOP/s), each with its own
    roofline, cpu_baseline and e2e. The dense paths run replicas only, so they are not
    repeated at N>1.

--config 0..4 runs one configuration alone (0 single linear, 1 decode, 2 prefill,
3 MoE, 4 column-parallel K=8192 N=28672 sweep).

--impl reference times the reference's own CPU path for the same workload on the
host cores: the oracle port (torch._int_mm + fp32 dequant, oracle/w8a8_oracle.py),
because the reference's kernels package (fni8) is not available here.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "fni8-serve_b200"))
sys.path.insert(0, ROOT)

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
INT8_DENSE_NOMINAL_TOPS = 4500.0  # B200 dense int8 tensor-core peak (vendor figure)

QWEN3_8B = [("qkv", 4096, 6144), ("o", 4096, 4096), ("gate_up", 4096, 24576), ("down", 12288, 4096)]
DECODE_M = [1, 8, 32, 128, 256]


# ------------------------------------------------------------------ environment helpers
def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
    return dict(FALLBACK_PEAKS, source="fallback")


def committed_traffic(key):
    """dram bytes per launch of the dominant kernel from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        return json.load(open(p)).get(key)
    return None


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons of this GPU, sampled every 2 ms through
    NVML while the timed region runs (read-only queries; falls back to `nvidia-smi -lms 200`
    when NVML is unavailable)."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown"}
    Q = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.uuid = str(torch.cuda.get_device_properties(device).uuid)
        self.samples, self.max_mhz, self.stop = [], None, threading.Event()
        self.thread = self.p = self.f = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            u = self.uuid if self.uuid.startswith("GPU-") else "GPU-" + self.uuid
            try:
                self.h = pynvml.nvmlDeviceGetHandleByUUID(u)
            except Exception:
                self.h = pynvml.nvmlDeviceGetHandleByUUID(u.encode())
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM))
        except Exception:
            self.nv = None

    def _poll(self):
        nv = self.nv
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self.stop.is_set():
            try:
                self.samples.append((float(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)),
                                     int(get_reasons(self.h))))
            except Exception:
                pass
            self.stop.wait(0.002)

    def __enter__(self):
        if self.nv is not None:
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            return self
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None
        return self

    def __exit__(self, *a):
        if self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=5)
        if self.p is not None:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()

    def summary(self):
        if self.nv is not None:
            if not self.samples:
                return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"]}
            sm = sorted(s for s, _ in self.samples)
            reasons = sorted({name for _, r in self.samples for bit, name in self.REASONS.items() if r & bit})
            return {"sm_mhz": sm[len(sm) // 2], "sm_min_mhz": sm[0], "sm_max_mhz": self.max_mhz, "reasons": reasons,
                    "samples": len(self.samples), "source": "nvml, 2 ms"}
        rows = []
        if self.f is not None:
            self.f.flush()
            for ln in open(self.f.name):
                c = [x.strip() for x in ln.split(",")]
                if len(c) < 10:
                    continue
                u = c[1][4:] if c[1].startswith("GPU-") else c[1]
                if self.uuid.replace("GPU-", "") not in u and u not in self.uuid:
                    continue
                rows.append(c)
            os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = sorted(float(r[2]) for r in rows if r[2].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[6 + i].lower().startswith("active")})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": float(rows[0][3]), "reasons": reasons,
                "samples": len(rows), "source": "nvidia-smi, 200 ms"}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def init_dist(world, local):
    if world > 1 and not torch.distributed.is_initialized():
        import datetime

        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(v, world):
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def flush_l2(buf):
    buf.add_(1)  # 256 MB written: evicts the 126 MB L2 between timed iterations


# ------------------------------------------------------------------ workloads
def make_weight(N, K, seed, device):
    """int8 per-row weights + fp32 scales generated on the device (N(0, 0.02) quantised)."""
    import fni8

    g = torch.Generator(device=device).manual_seed(seed)
    w = torch.randn(N, K, generator=g, device=device, dtype=torch.float32) * 0.02
    q, s = fni8.quant.core.quantize_int8_rowwise(w)
    return fni8.QTensor(q.contiguous(), s.squeeze(-1).contiguous(), scheme="per_row_i8")


def act(M, K, seed, device, outliers=True):
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(M, K, generator=g, device=device)
    if outliers:
        ch = torch.randperm(K, generator=g, device=device)[: max(1, K // 1000)]
        x[:, ch] *= 20
    return x.half()


def decode_bytes(M, K, N):
    # weights + per-row scales + fp16 activations in + fp16 outputs out
    return N * K + 4 * N + 2 * M * K + 2 * M * N


class DecodeSet:
    """20 fni8.linear calls, distinct weights each."""

    def __init__(self, device, ms=DECODE_M):
        self.items = []
        seed = 0
        for M in ms:
            for name, K, N in QWEN3_8B:
                seed += 1
                self.items.append((M, name, K, N, make_weight(N, K, seed, device), act(M, K, 1000 + seed, device)))
        self.bytes = sum(decode_bytes(M, K, N) for M, _, K, N, _, _ in self.items)

    def step(self):
        import fni8

        return [fni8.linear(x, qt) for (_, _, _, _, qt, x) in self.items]


def time_graph(fn, steps, warmup, world, flush=None):
    """Capture fn() in a CUDA graph; time `steps` replays with CUDA events (max over ranks)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()  # eager warm-up (allocates the GEMM workspace outside capture)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    barrier(world)
    times = []
    for _ in range(steps):
        if flush is not None:
            flush()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        times.append((a, b))
    torch.cuda.synchronize()
    barrier(world)
    total_ms = sum(a.elapsed_time(b) for a, b in times)
    del graph
    return max_over_ranks(total_ms, world)


def per_launch_ms(fn, reps=20):
    """Average device time of one fn() launch sequence: `reps` back-to-back calls captured
    in one CUDA graph, timed with CUDA events around its replays (the best of three), so
    no host launch gap falls between the calls. The launches keep their L2 state between
    calls (the kernel's own weights dominate its traffic at the shapes timed here)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(reps):
            fn()
    graph.replay()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(3):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        torch.cuda.synchronize()
        best = min(best, a.elapsed_time(b) / reps)
    del graph
    return best


def time_eager(fn, steps, warmup, world, flush=None):
    """Time `steps` eager calls of fn() with CUDA events (for steps that synchronise with
    the host, e.g. expert-parallel all_to_all split sizes); max over ranks."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    total = 0.0
    for _ in range(steps):
        if flush is not None:
            flush()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        total += a.elapsed_time(b)
    barrier(world)
    return max_over_ranks(total, world)


def time_pipelined(items, steps, warmup, world, slots=2):
    """End-to-end timing through the public API with host buffers, the way a server runs:
    per item (hx pinned host input, dxs device input slots, fn public call, hy pinned host
    output; fn may return a list of tensors and hy be the matching list) the host->device
    copy runs on one stream, fn on a second and the device->host copy of its result on a
    third, ordered by events, so copies of one item overlap the compute of another. Every
    copy of every step is inside the timed region (CUDA events on the launching stream,
    joined with the three streams); max over ranks."""
    s_in, s_cmp, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    free = {}  # (item, slot) -> event: the compute that read that device slot is done
    drained = {}  # (item, slot) -> event: the D2H of the outputs computed from that slot is done

    def one(k):
        slot = k % slots
        for i, (hx, dxs, fn, hy) in enumerate(items):
            dx = dxs[slot]
            ev = free.get((i, slot))
            if ev is not None:
                s_in.wait_event(ev)
            with torch.cuda.stream(s_in):
                dx.copy_(hx, non_blocking=True)
            e_in = torch.cuda.Event()
            e_in.record(s_in)
            s_cmp.wait_event(e_in)
            ev = drained.get((i, slot))
            if ev is not None:  # static (graph) outputs of this slot were copied out
                s_cmp.wait_event(ev)
            with torch.cuda.stream(s_cmp):
                y = fn(dx)
            e_c = torch.cuda.Event()
            e_c.record(s_cmp)
            free[(i, slot)] = e_c
            s_out.wait_event(e_c)
            ys, hys = (y, hy) if isinstance(y, (list, tuple)) else ([y], [hy])
            with torch.cuda.stream(s_out):
                for yt, ht in zip(ys, hys):
                    ht.copy_(yt, non_blocking=True)
            e_o = torch.cuda.Event()
            e_o.record(s_out)
            drained[(i, slot)] = e_o
            for yt in ys:
                yt.record_stream(s_out)

    for k in range(warmup):
        one(k)
    torch.cuda.synchronize()
    barrier(world)
    cur = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(cur)
    for st in (s_in, s_cmp, s_out):
        st.wait_event(a)
    for k in range(steps):
        one(warmup + k)
    for st in (s_in, s_cmp, s_out):
        e = torch.cuda.Event()
        e.record(st)
        cur.wait_event(e)
    b.record(cur)
    torch.cuda.synchronize()
    return max_over_ranks(a.elapsed_time(b), world)


def graph_per_slot(slots, calls):
    """Capture calls(xd) -> outputs in one CUDA graph per device input slot (the way a
    decode runner replays a step); returns replay(xd) -> that slot's static outputs."""
    graphs = {}
    cap = torch.cuda.Stream()
    cap.wait_stream(torch.cuda.current_stream())
    for xd in slots:
        with torch.cuda.stream(cap):
            calls(xd)  # eager warm-up outside the capture
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap):
                out = calls(xd)
        graphs[xd.data_ptr()] = (g, out)
    torch.cuda.current_stream().wait_stream(cap)
    torch.cuda.synchronize()

    def replay(xd):
        g, o = graphs[xd.data_ptr()]
        g.replay()
        return o

    return replay


# ------------------------------------------------------------------ configs (our arm)
def run_config1(args, world, rank, dev):
    import fni8
    from fni8 import _native as nat
    from fni8.ops import WORKSPACE

    ds = DecodeSet(dev)
    WORKSPACE.get(dev)
    pk = peaks()
    with ClockSampler(dev) as clk:
        ms_total = time_graph(ds.step, args.steps, args.warmup, world)
    clocks = clk.summary()
    ms_step = ms_total / args.steps
    value = world * ds.bytes / (ms_step * 1e-3) / 1e9

    # dominant kernel: the weight-streaming W8A8 GEMM. The 20 GEMM launches alone (on
    # int8 activations prepared beforehand) are captured in one graph per decode batch M
    # and timed with CUDA events around the replays.
    gemm_ms, gemm_bytes, per = 0.0, 0, {}
    for M in DECODE_M:
        rows = [it for it in ds.items if it[0] == M]
        qs = [fni8.quantize_rows(x) for (*_, x) in rows]

        def gemms(rows=rows, qs=qs):
            for (_, _, _, _, qt, _), (q, s) in zip(rows, qs):
                fni8.linear_q(q, s, qt)

        t = time_graph(gemms, args.steps, args.warmup, world) / args.steps
        b = sum(N * K + 4 * N + M * K + 4 * M + 2 * M * N for (_, _, K, N, _, _) in rows)
        gemm_ms += t
        gemm_bytes += b
        per[f"M{M}"] = round(b / (t * 1e-3) / 1e9, 1)
    achieved = gemm_bytes / (gemm_ms * 1e-3) / 1e9

    # end to end through the public API with host buffers: H2D of each linear's input
    # from pinned memory, fni8.linear, D2H of its output, every step (copies and compute
    # on separate streams, pipelined across the step's linears)
    # The step's 20 inputs travel as one pinned buffer; the 20 fni8.linear calls of a step
    # are captured in a CUDA graph per input slot (a decode runner's replay), so the host
    # issues one replay per step instead of 20 eager calls.
    sizes = [x.numel() for (*_, x) in ds.items]
    hx = torch.cat([x.reshape(-1) for (*_, x) in ds.items]).cpu().pin_memory()
    hy = torch.empty(sum(M * N for (M, _, _, N, _, _) in ds.items), dtype=torch.float16).pin_memory()
    h2d = hx.numel() * 2
    d2h = hy.numel() * 2
    slots = [torch.empty_like(hx, device=dev) for _ in range(2)]

    def calls(xd):
        outs, off = [], 0
        for (M, _, K, _, qt, _), n in zip(ds.items, sizes):
            outs.append(fni8.linear(xd[off:off + n].view(M, K), qt))
            off += n
        return torch.cat([o.reshape(-1) for o in outs])  # the step's results, one D2H

    replay = graph_per_slot(slots, calls)
    e2e_ms = time_pipelined([(hx, slots, replay, hy)], args.steps, args.warmup, world, slots=2) / args.steps
    e2e = world * ds.bytes / (e2e_ms * 1e-3) / 1e9
    del replay

    line = {
        "metric": "W8A8 decode GB/s (Qwen3-8B QKV/O/gate_up/down at M=1,8,32,128,256; % of HBM)",
        "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8", "data": "synthetic",
        "config": {"workload": "BASELINE config 1: Qwen3-8B decode-step linear set", "M": DECODE_M,
                   "gemms": [f"{n}:K{k}xN{nn}" for n, k, nn in QWEN3_8B], "bytes_per_step": ds.bytes,
                   "l2": "inputs larger than L2 (distinct weights per linear, 965 MB per step)",
                   "parallelism": f"replicas{world}", "timing": "CUDA graph replay, CUDA events"},
        "frac_of_hbm": round(value / world / pk["hbm_gbs"], 3),
        "frac_of_8tbs_nominal": round(value / world / 8000.0, 3),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / pk["hbm_gbs"], 3), "traffic": committed_traffic("decode_gemm"),
                     "kernel": "w8a8_splitk_kernel (M<=128, and QKV/O/down at M=256) / CTA-pair w8a8_tile_kernel (gate_up at M=256): the 20 decode GEMMs, graph-replayed, per-M graphs",
                     "peak_source": pk["source"] + " (MEASURED_PEAKS.json hbm_gbs)",
                     "gemm_gbs_per_M": per, "gemm_us_per_step": round(gemm_ms * 1e3, 2)},
        "e2e": {"value": round(e2e, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(e2e_ms, 4),
                "api": "fni8.linear x20 captured in a CUDA graph per input slot (decode-runner replay), "
                       "results gathered into one buffer; pinned host buffers; H2D, replay and D2H on three "
                       "streams, steps pipelined"},
        "gpu_launches": 40 * args.steps,
        "clocks": clocks,
    }
    return line, ds


def run_config2(args, world, rank, dev):
    """Prefill: fused RMSNorm+quant -> QKV, O, gate_up with SiLU*up in its epilogue -> quant -> down,
    M=8192 (the drop-in GatedMLP's fused path)."""
    import fni8

    M = 8192
    g = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn(M, 4096, generator=g, device=dev).half()
    gamma = (1 + 0.1 * torch.randn(4096, generator=g, device=dev)).half()
    W = {name: make_weight(N, K, 100 + i, dev) for i, (name, K, N) in enumerate(QWEN3_8B)}
    ops = sum(2 * M * K * N for _, K, N in QWEN3_8B)
    flush_buf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def step():
        q, s = fni8.rmsnorm_quant(x, gamma, 1e-6)
        fni8.linear_q(q, s, W["qkv"])
        fni8.linear_q(q, s, W["o"])
        hq, hs = fni8.quantize_rows(fni8.linear_act_q(q, s, W["gate_up"]))
        return fni8.linear_q(hq, hs, W["down"])

    pk = peaks()
    with ClockSampler(dev) as clk:
        ms_total = time_graph(step, args.steps, args.warmup, world, flush=lambda: flush_l2(flush_buf))
    clocks = clk.summary()
    ms_step = ms_total / args.steps
    value = world * ops / (ms_step * 1e-3) / 1e12
    q, s = fni8.rmsnorm_quant(x, gamma, 1e-6)
    t_gu = per_launch_ms(lambda: fni8.linear_act_q(q, s, W["gate_up"]), reps=10)
    ach = 2 * M * 4096 * 24576 / (t_gu * 1e-3) / 1e12
    t_gu_plain = per_launch_ms(lambda: fni8.linear_q(q, s, W["gate_up"]), reps=10)
    # no int8 peak is measured on this pool: this library's tile GEMM at 8192^3 stands beside
    # the nominal figure
    a8 = torch.randint(-127, 128, (8192, 8192), generator=g, device=dev, dtype=torch.int8)
    s8 = torch.rand(8192, generator=g, device=dev) * 1e-2
    w8 = make_weight(8192, 8192, 99, dev)
    t8 = per_launch_ms(lambda: fni8.linear_q(a8, s8, w8), reps=10)
    own_peak = {"value": round(2 * 8192 ** 3 / (t8 * 1e-3) / 1e12, 1), "unit": "TOP/s",
                "what": "w8a8_tile_kernel (CTA pairs), M=N=K=8192, CUDA events, 10 launches"}
    del a8, s8, w8
    xh = x.cpu().pin_memory()
    yh = torch.empty(M, 4096, dtype=torch.float16).pin_memory()

    def e2e_fn(xd):
        q, s = fni8.rmsnorm_quant(xd, gamma, 1e-6)
        fni8.linear_q(q, s, W["qkv"])
        fni8.linear_q(q, s, W["o"])
        hq, hs = fni8.quantize_rows(fni8.linear_act_q(q, s, W["gate_up"]))
        return fni8.linear_q(hq, hs, W["down"])

    # H2D of a step's hidden state, the step, D2H of its output: three streams, steps
    # pipelined (two device input slots)
    e2e_ms = time_pipelined([(xh, [torch.empty_like(x) for _ in range(2)], e2e_fn, yh)], args.steps, args.warmup,
                            world) / args.steps
    line = {
        "metric": "W8A8 prefill TOPS (Qwen3-8B 4 GEMMs at M=8192, fused RMSNorm+quant; % int8 TC peak)",
        "value": round(value, 1), "unit": "TOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8", "data": "synthetic",
        "config": {"workload": "BASELINE config 2: Qwen3-8B prefill M=8192", "ops_per_step": ops,
                   "l2": "flushed between steps (256 MB write)", "parallelism": f"replicas{world}"},
        "frac_of_int8_nominal": round(value / world / INT8_DENSE_NOMINAL_TOPS, 3),
        "int8_peak_own_kernel": own_peak,
        "roofline": {"bound": "tensor", "achieved": round(ach, 1), "peak": INT8_DENSE_NOMINAL_TOPS,
                     "unit": "TOP/s", "frac": round(ach / INT8_DENSE_NOMINAL_TOPS, 3),
                     "traffic": committed_traffic("prefill_gate_up_act"),
                     "kernel": "w8a8_tile_kernel<256,0,1,ACTMUL>, CTA pairs (gate_up with SiLU*up in the epilogue)",
                     "gate_up_plain_tops": round(2 * M * 4096 * 24576 / (t_gu_plain * 1e-3) / 1e12, 1),
                     "peak_source": "nominal dense int8 (no measured int8 peak); 2x measured bf16 = "
                                    f"{2 * pk['bf16_tflops']:.0f}"},
        "e2e": {"value": round(world * ops / (e2e_ms * 1e-3) / 1e12, 1), "unit": "TOP/s",
                "h2d_bytes_per_step": xh.numel() * 2, "d2h_bytes_per_step": yh.numel() * 2,
                "ms_per_step": round(e2e_ms, 4),
                "api": "fni8 rmsnorm_quant / linear_q / linear_act_q / quantize_rows (eager, pinned host buffers; "
                       "H2D, compute and D2H on three streams, steps pipelined)"},
        "gpu_launches": 6 * args.steps,
        "clocks": clocks,
    }
    return line, None


def base_line(metric, value, unit, world, args, ms_step, config, dtype="int8", scaling="weak"):
    return {"metric": metric, "value": round(value, 3), "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": scaling,
            "vs_baseline": None, "dtype": dtype, "data": "synthetic", "config": config}


def run_config0(args, world, rank, dev):
    """one fni8.linear, M=256 K=1024 N=6144 (Qwen3-0.6B gate_up)."""
    import fni8

    M, K, N = 256, 1024, 6144
    qt = make_weight(N, K, 1, dev)
    x = act(M, K, 2, dev)
    flush_buf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    ops = 2 * M * N * K
    with ClockSampler(dev) as clk:
        ms = time_graph(lambda: fni8.linear(x, qt), args.steps, args.warmup, world,
                        flush=lambda: flush_l2(flush_buf)) / args.steps
    xh = x.cpu().pin_memory()
    yh = torch.empty(M, N, dtype=torch.float16).pin_memory()
    slots = [torch.empty_like(x) for _ in range(3)]
    replay = graph_per_slot(slots, lambda xd: fni8.linear(xd, qt))
    e2e_ms = time_pipelined([(xh, slots, replay, yh)], args.steps, args.warmup, world, slots=3) / args.steps
    del replay
    line = base_line("W8A8 linear TOP/s (M=256 K=1024 N=6144; % int8 TC peak)", world * ops / (ms * 1e-3) / 1e12,
                     "TOP/s", world, args, ms,
                     {"workload": "BASELINE config 0: single W8A8 linear", "M": M, "K": K, "N": N,
                      "l2": "flushed between steps (256 MB write)", "parallelism": f"replicas{world}"})
    line["roofline"] = {"bound": "tensor", "achieved": round(ops / (ms * 1e-3) / 1e12, 1),
                        "peak": INT8_DENSE_NOMINAL_TOPS, "unit": "TOP/s",
                        "frac": round(ops / (ms * 1e-3) / 1e12 / INT8_DENSE_NOMINAL_TOPS, 4),
                        "traffic": committed_traffic("cfg0_linear"), "kernel": "quantise + w8a8_tile_kernel",
                        "note": "3.2 GOP in one launch pair: launch-latency bound, not tensor bound"}
    line["e2e"] = {"value": round(world * ops / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TOP/s",
                   "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * N * 2, "ms_per_step": round(e2e_ms, 4),
                   "api": "fni8.linear captured in a CUDA graph per input slot; pinned host buffers; H2D, "
                          "replay and D2H on three streams, steps pipelined"}
    line["gpu_launches"] = 2 * args.steps
    line["clocks"] = clk.summary()
    return line, None


MOE = dict(T=4096, E=128, k=8, H=2048, I=768)


def moe_inputs(dev, rank):
    """BASELINE config 3 inputs: tokens N(0,1); router logits N(0,1) + a per-expert bias
    -1.1*log(rank) over a seeded expert ranking (Zipf s=1.1 weights), shared by all ranks."""
    T, E, H = MOE["T"], MOE["E"], MOE["H"]
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    x = torch.randn(T, H, generator=g, device=dev).half()
    order = torch.randperm(E, generator=torch.Generator().manual_seed(7))
    zipf = torch.empty(E)
    zipf[order] = -1.1 * torch.log(torch.arange(1, E + 1, dtype=torch.float32))
    logits = torch.randn(T, E, generator=g, device=dev) + zipf.to(dev)
    return x, logits


def moe_experts_on(dev, lo, hi):
    """Experts [lo, hi) of the config-3 layer: the same seeded weights on every rank."""
    return moe_experts_ids(dev, range(lo, hi))


def moe_experts_ids(dev, ids):
    """The config-3 experts `ids`, in that order (weights seeded by expert id)."""
    from fni8.moe import ExpertStack

    H, I = MOE["H"], MOE["I"]
    gu = [make_weight(2 * I, H, 5000 + e, dev) for e in ids]
    dn = [make_weight(H, I, 9000 + e, dev) for e in ids]
    return ExpertStack(torch.stack([w.data for w in gu]), torch.stack([w.scale for w in gu]),
                       torch.stack([w.data for w in dn]), torch.stack([w.scale for w in dn]))


def run_config3(args, world, rank, dev):
    """Qwen3-30B-A3B-shaped MoE layer, expert-parallel over the ranks."""
    import fni8.moe as moe
    from fni8.parallel import ExpertParallelMoE, balanced_placement, experts_of_rank

    T, E, k, H, I = MOE["T"], MOE["E"], MOE["k"], MOE["H"], MOE["I"]
    x, logits = moe_inputs(dev, rank)
    place = None
    if world > 1:
        # experts placed by the routed load (rows per expert over all ranks' tokens) of one
        # routing, measured before the timed steps: greedy longest-load-first, E/P per rank
        load = torch.bincount(moe.route(logits, k)[0].reshape(-1).long(), minlength=E)
        torch.distributed.all_reduce(load)
        place = balanced_placement(load.cpu(), world)
        stack = moe_experts_ids(dev, experts_of_rank(place, world, rank))
    else:
        stack = moe_experts_on(dev, 0, E)
    ops = 2 * T * k * (2 * I * H + H * I)
    if world == 1:
        def step():
            topi, topw = moe.route(logits, k)
            return moe.experts(x, topi, topw, stack)

        with ClockSampler(dev) as clk:
            ms = time_graph(step, args.steps, args.warmup, world) / args.steps
        timing = "CUDA graph replay"
    else:
        ep = ExpertParallelMoE(stack, E, max_tokens=T, placement=place)

        def step():
            topi, topw = moe.route(logits, k)
            return ep(x, topi, topw)

        with ClockSampler(dev) as clk:
            if ep.transport == "p2p":  # no host sync in the layer: CUDA graph replay
                ms = time_graph(step, args.steps, args.warmup, world) / args.steps
            else:
                ms = time_eager(step, args.steps, args.warmup, world) / args.steps
        timing = ("CUDA graph replay (peer-memory exchange over NVLink)" if ep.transport == "p2p" else
                  "eager (all_to_all split sizes visit the host), CUDA events")
    # grouped-GEMM share: the two grouped launches of the single-GPU step alone (gate_up with
    # SiLU*up in its epilogue, then down), on the routed inputs
    topi, topw = moe.route(logits, k)
    from fni8.moe import grouped_gemm, grouped_gemm_act, plan, quantize_scatter
    from fni8.ops import quantize_rows

    counts, offsets, ros, sor = plan(topi, E)
    n = int(offsets[-1].item())
    aq, as_ = quantize_scatter(x, ros, k, n)
    iota = torch.arange(E, dtype=torch.int32, device=dev)
    full = moe_experts_on(dev, 0, E) if world > 1 else stack
    hq, hs = quantize_rows(grouped_gemm_act(aq, as_, full.w_gu, full.s_gu, iota, offsets[:E], counts))
    t_gu = per_launch_ms(lambda: grouped_gemm_act(aq, as_, full.w_gu, full.s_gu, iota, offsets[:E], counts), reps=10)
    t_dn = per_launch_ms(lambda: grouped_gemm(hq, hs, full.w_dn, full.s_dn, iota, offsets[:E], counts), reps=10)
    ach = ops / ((t_gu + t_dn) * 1e-3) / 1e12
    ops_gu = 2 * T * k * 2 * I * H
    ach_gu = ops_gu / (t_gu * 1e-3) / 1e12
    wbytes = E * (2 * I * H + H * I)
    # algorithmic bytes of the gate_up launch: the 128 experts' weights and scales, the routed
    # int8 rows and scales read, the [rows, I] fp16 product written
    bytes_gu = E * (2 * I * H + 2 * I * 4) + n * (H + 4) + n * I * 2
    gbs_gu = bytes_gu / (t_gu * 1e-3) / 1e9
    line = base_line("MoE expert layer tokens/s (E=128 top-8 H=2048 I=768, W8A8 grouped GEMM, expert parallel)",
                     world * T / (ms * 1e-3), "tokens/s", world, args, ms,
                     {"workload": "BASELINE config 3: Qwen3-30B-A3B-shaped MoE layer", "tokens_per_rank": T,
                      "experts": E, "top_k": k, "hidden": H, "intermediate": I, "router": "N(0,1)+Zipf(1.1) bias",
                      "parallelism": f"ep{world}", "timing": timing,
                      "expert_placement": ("one GPU" if world == 1 else
                                           "balanced by the routed load of one routing of every rank's tokens, "
                                           "measured before the timed steps (greedy longest-load-first, E/P per rank)"),
                      "l2": "inputs larger than L2 (604 MB of expert weights)"})
    line["frac_tensor_vs_nominal"] = round(ach / INT8_DENSE_NOMINAL_TOPS, 3)
    line["frac_weights_vs_hbm"] = round(wbytes / ((t_gu + t_dn) * 1e-3) / 1e9 / peaks()["hbm_gbs"], 3)
    # Both bounds are close for this layer (309 GOP vs 604 MB of weights); the roofline object
    # carries the larger of the gate_up launch's two fractions, the other beside it.
    hbm = peaks()["hbm_gbs"]
    frac_t, frac_h = ach_gu / INT8_DENSE_NOMINAL_TOPS, gbs_gu / hbm
    common = {"traffic": committed_traffic("moe_grouped_act"),
              "kernel": "w8a8_tile_kernel<256,1,0,ACTMUL>: grouped gate_up of all 128 experts with SiLU*up in "
                        "its epilogue (one launch, device time from a CUDA graph of 10 launches)",
              "algorithmic_bytes_per_launch": bytes_gu, "gate_up_us": round(t_gu * 1e3, 1),
              "down_us": round(t_dn * 1e3, 1), "both_grouped_launches_tops": round(ach, 1),
              "weights_gbs": round(wbytes / ((t_gu + t_dn) * 1e-3) / 1e9, 1)}
    if frac_h >= frac_t:
        line["roofline"] = {"bound": "hbm", "achieved": round(gbs_gu, 1), "peak": hbm, "unit": "GB/s",
                            "frac": round(frac_h, 3), "tensor_tops": round(ach_gu, 1),
                            "tensor_frac_vs_nominal": round(frac_t, 3), **common}
    else:
        line["roofline"] = {"bound": "tensor", "achieved": round(ach_gu, 1), "peak": INT8_DENSE_NOMINAL_TOPS,
                            "unit": "TOP/s", "frac": round(frac_t, 3), "hbm_gbs": round(gbs_gu, 1),
                            "hbm_frac": round(frac_h, 3), **common}
    line["roofline"]["peak_source"] = "hbm: MEASURED_PEAKS.json hbm_gbs; int8: nominal dense 4500 TOP/s"
    # end to end: H2D of the step's tokens and router logits (one pinned buffer), routing +
    # experts (a CUDA graph per input slot on one GPU; eager under expert parallelism, whose
    # all_to_all split sizes visit the host), D2H of the layer output; three streams
    nx, nl = x.numel() * 2, logits.numel() * 4
    hin = torch.empty(nx + nl, dtype=torch.uint8).pin_memory()
    hin[:nx].copy_(x.reshape(-1).view(torch.uint8).cpu())
    hin[nx:].copy_(logits.reshape(-1).view(torch.uint8).cpu())
    hout = torch.empty(T, H, dtype=x.dtype).pin_memory()

    def layer(xd):
        xv = xd[:nx].view(x.dtype).view(T, H)
        lv = xd[nx:].view(torch.float32).view(T, E)
        topi, topw = moe.route(lv, k)
        return moe.experts(xv, topi, topw, stack) if world == 1 else ep(xv, topi, topw)

    slots = [torch.empty_like(hin, device=dev) for _ in range(2)]
    graphed = world == 1 or ep.transport == "p2p"
    fn = graph_per_slot(slots, layer) if graphed else layer
    e2e_ms = time_pipelined([(hin, slots, fn, hout)], args.steps, args.warmup, world) / args.steps
    del fn
    if world > 1:
        ep.close()
    line["e2e"] = {"value": round(world * T / (e2e_ms * 1e-3), 1), "unit": "tokens/s", "h2d_bytes_per_step": nx + nl,
                   "d2h_bytes_per_step": hout.numel() * 2, "ms_per_step": round(e2e_ms, 4),
                   "api": ("fni8.moe route + experts" if world == 1 else f"fni8.moe route + ExpertParallelMoE "
                           f"({ep.transport})") + (" captured in a CUDA graph per input slot" if graphed else
                                                   " (eager)") +
                          "; pinned host buffers; H2D, layer and D2H on three streams, steps pipelined"}
    # route, plan (3), quantise-scatter, gate_up+SiLU, quantise, down, combine; under expert
    # parallelism: route, quantise, plan (3), dispatch, gate_up+SiLU, quantise, down, return,
    # combine
    line["gpu_launches"] = (9 if world == 1 else 11) * args.steps
    line["clocks"] = clk.summary()
    return line, None


def run_config4(args, world, rank, dev):
    """K=8192 N=28672, M in {16, 512, 4096}, N sharded over the ranks."""
    from fni8.parallel import ColumnParallelLinearW8A8, shard_rows

    K, N = 8192, 28672
    Ms = [16, 512, 4096]
    full = make_weight(N, K, 77, dev)
    shard = shard_rows(full, world, rank)
    del full
    xs = [act(M, K, 10 + M, dev) for M in Ms]
    # p2p: each rank's GEMM stores its columns into every rank's output over NVLink
    cp = ColumnParallelLinearW8A8(shard, max_rows=max(Ms)) if world > 1 else None
    import fni8

    def step():
        for x in xs:
            (cp(x) if cp is not None else fni8.linear(x, shard))

    ops = sum(2 * M * N * K for M in Ms)
    with ClockSampler(dev) as clk:
        if cp is None or cp.transport == "p2p":  # no host synchronisation in the step
            ms = time_graph(step, args.steps, args.warmup, world) / args.steps
        else:
            ms = time_eager(step, args.steps, args.warmup, world) / args.steps
    per = {}
    n = N // world
    for M, x in zip(Ms, xs):
        t = per_launch_ms(lambda x=x: fni8.linear(x, shard), reps=10)
        per[f"M{M}_shard"] = {"us": round(t * 1e3, 1), "TOP/s": round(2 * M * n * K / (t * 1e-3) / 1e12, 1),
                              "GB/s": round((n * K + 2 * M * K + 2 * M * n) / (t * 1e-3) / 1e9, 1)}
        if cp is not None:
            # the whole column-parallel call: quantise, GEMM with the all-gather stores, the
            # ordering barrier. Bound: the slower of the shard's int8 work at the nominal
            # peak and the (world-1)/world of the output each rank receives over NVLink at the
            # measured 770 GB/s per direction.
            tg = per_launch_ms(lambda x=x: cp(x), reps=10)
            recv = (world - 1) * M * n * 2
            bound_us = max(2 * M * n * K / (INT8_DENSE_NOMINAL_TOPS * 1e12), recv / 770e9) * 1e6
            per[f"M{M}_shard"].update({"gathered_us": round(tg * 1e3, 1),
                                       "nvlink_recv_GBs": round(recv / (tg * 1e-3) / 1e9, 1),
                                       "bound_us": round(bound_us, 1), "frac_of_bound": round(bound_us / (tg * 1e3), 3)})
    line = base_line("Column-parallel W8A8 TOP/s (K=8192 N=28672, M=16/512/4096, N sharded, all-gather)",
                     ops / (ms * 1e-3) / 1e12, "TOP/s", world, args, ms,
                     {"workload": "BASELINE config 4: column-parallel dense sweep", "K": K, "N": N, "M": Ms,
                      "parallelism": f"column{world}", "l2": "inputs larger than L2 (235 MB of weights)"},
                     scaling="strong")
    line["per_gpu"] = round(ops / (ms * 1e-3) / 1e12 / world, 1)
    line["shard_kernels"] = per
    line["roofline"] = {"bound": "tensor", "achieved": per["M4096_shard"]["TOP/s"], "peak": INT8_DENSE_NOMINAL_TOPS,
                        "unit": "TOP/s", "frac": round(per["M4096_shard"]["TOP/s"] / INT8_DENSE_NOMINAL_TOPS, 3),
                        "traffic": committed_traffic("sweep_m4096"), "kernel": "w8a8_tile_kernel, CTA pairs (M=4096 shard)"}
    # end to end: H2D of the three activation batches (one pinned buffer), the three linears
    # (a CUDA graph per input slot on one GPU; eager with the all-gather otherwise), D2H of
    # the full [M, N] outputs gathered into one buffer; three streams
    sizes = [x.numel() for x in xs]
    hin = torch.cat([x.reshape(-1) for x in xs]).cpu().pin_memory()
    hout = torch.empty(sum(M * N for M in Ms), dtype=torch.float16).pin_memory()

    def sweep(xd):
        res = torch.empty(hout.numel(), dtype=torch.float16, device=dev)
        off, o2 = 0, 0
        for M, sz in zip(Ms, sizes):
            xv = xd[off:off + sz].view(M, K)
            y = cp(xv) if cp is not None else fni8.linear(xv, shard)  # p2p: a view of the layer's buffer
            res[o2:o2 + y.numel()].copy_(y.reshape(-1))
            off, o2 = off + sz, o2 + y.numel()
        return res

    slots = [torch.empty_like(hin, device=dev) for _ in range(2)]
    fn = graph_per_slot(slots, sweep) if cp is None or cp.transport == "p2p" else sweep
    e2e_ms = time_pipelined([(hin, slots, fn, hout)], args.steps, args.warmup, world) / args.steps
    del fn
    line["e2e"] = {"value": round(ops / (e2e_ms * 1e-3) / 1e12, 1), "unit": "TOP/s", "h2d_bytes_per_step": hin.numel() * 2,
                   "d2h_bytes_per_step": hout.numel() * 2, "ms_per_step": round(e2e_ms, 4),
                   "api": ("fni8.linear x3 captured in a CUDA graph per input slot" if world == 1 else
                           "ColumnParallelLinearW8A8 x3 (GEMM with the all-gather stores over NVLink) captured in "
                           "a CUDA graph per input slot") +
                          "; pinned host buffers; H2D, linears and D2H on three streams, steps pipelined"}
    # per linear a quantiser and a GEMM; under p2p the decode-size (M=16) GEMM adds the copy out
    line["gpu_launches"] = (7 if cp is not None else 6) * args.steps
    line["clocks"] = clk.summary()
    if cp is not None:
        cp.close()
    return line, None


# ------------------------------------------------------------------ reference arm (CPU)
METRICS = {
    0: ("W8A8 linear TOP/s (M=256 K=1024 N=6144; % int8 TC peak)", "TOP/s"),
    1: ("W8A8 decode GB/s (Qwen3-8B QKV/O/gate_up/down at M=1,8,32,128,256; % of HBM)", "GB/s"),
    2: ("W8A8 prefill TOPS (Qwen3-8B 4 GEMMs at M=8192, fused RMSNorm+quant; % int8 TC peak)", "TOP/s"),
    3: ("MoE expert layer tokens/s (E=128 top-8 H=2048 I=768, W8A8 grouped GEMM, expert parallel)", "tokens/s"),
    4: ("Column-parallel W8A8 TOP/s (K=8192 N=28672, M=16/512/4096, N sharded, all-gather)", "TOP/s"),
}


def cpu_workload(config):
    """The reference's CPU int8 path for a config on the host cores (the oracle port:
    torch._int_mm int8->int32 + fp32 dequant, oracle/w8a8_oracle.py), as
    (step, work per step, scale to the metric's unit, sample description). Large configs
    run a fixed fraction of the workload per step; the rate is what is reported."""
    from oracle import w8a8_oracle as O

    g = torch.Generator().manual_seed(0)

    def qw(N, K):
        return O.quantize_weight_rowwise(0.02 * torch.randn(N, K, generator=g))

    if config == 0:
        M, K, N = 256, 1024, 6144
        wq, ws = qw(N, K)
        x = torch.randn(M, K, generator=g).half()
        return (lambda: O.linear_w8a8(x, wq, ws, exact=False)), 2 * M * N * K, 1e12, "the full config-0 linear"
    if config == 1:
        items = []
        for M in DECODE_M:
            for name, K, N in QWEN3_8B:
                wq, ws = qw(N, K)
                items.append((wq, ws, torch.randn(M, K, generator=g).half()))
        nbytes = sum(decode_bytes(x.shape[0], w.shape[1], w.shape[0]) for w, _, x in items)

        def step():
            for wq, ws, x in items:
                O.linear_w8a8(x, wq, ws, exact=False)

        return step, nbytes, 1e9, "the full config-1 step (20 linears)"
    if config == 2:
        M = 512
        x = torch.randn(M, 4096, generator=g).half()
        gamma = torch.ones(4096, dtype=torch.float16)
        ws = {name: qw(N, K) for name, K, N in QWEN3_8B}

        def step():
            q, s = O.quantize_rows(O.rmsnorm(x, gamma, 1e-6))
            O.dequant(O.int_mm_fast(q, ws["qkv"][0]), s, ws["qkv"][1])
            O.dequant(O.int_mm_fast(q, ws["o"][0]), s, ws["o"][1])
            h = O.dequant(O.int_mm_fast(q, ws["gate_up"][0]), s, ws["gate_up"][1])
            hq, hs = O.quantize_rows(O.act_and_mul(h))
            O.dequant(O.int_mm_fast(hq, ws["down"][0]), hs, ws["down"][1])

        ops = sum(2 * M * K * N for _, K, N in QWEN3_8B)
        return step, ops, 1e12, "the config-2 chain at M=512 tokens (1/16 of M=8192) per step"
    if config == 3:
        T, E, k, H, I = 256, MOE["E"], MOE["k"], MOE["H"], MOE["I"]
        w_gu = torch.empty(E, 2 * I, H, dtype=torch.int8)
        s_gu = torch.empty(E, 2 * I)
        w_dn = torch.empty(E, H, I, dtype=torch.int8)
        s_dn = torch.empty(E, H)
        for e in range(E):
            w_gu[e], s_gu[e] = qw(2 * I, H)
            w_dn[e], s_dn[e] = qw(H, I)
        x = torch.randn(T, H, generator=g).half()
        zipf = -1.1 * torch.log(torch.arange(1, E + 1, dtype=torch.float32))[torch.randperm(E, generator=g)]
        logits = torch.randn(T, E, generator=g) + zipf

        def step():
            topi, topw = O.moe_route(logits, k)
            O.moe_experts_w8a8(x, topi, topw.float(), w_gu, s_gu, w_dn, s_dn, exact=False)

        return step, T, 1.0, "256 of the 4096 tokens per step through all 128 experts (moe.py:99-105 loop)"
    if config == 4:
        K, N = 8192, 28672 // 8
        wq, ws = qw(N, K)
        xs = [torch.randn(M, K, generator=g).half() for M in (16, 512, 4096)]

        def step():
            for x in xs:
                O.linear_w8a8(x, wq, ws, exact=False)

        return step, sum(2 * x.shape[0] * N * K for x in xs), 1e12, "one 1/8 column shard (N=3584) at M=16/512/4096"
    raise ValueError(config)


def reference_arm(args, world, rank, config=None):
    """The reference's CPU int8 path on the host cores (oracle port), same config/metric."""
    if rank != 0:
        return None
    config = args.config if config is None else config
    torch.set_num_threads(os.cpu_count() or 1)
    step, work, scale, sample = cpu_workload(config)
    for _ in range(max(1, min(args.warmup, 2))):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    v = work / dt / scale
    metric, unit = METRICS[config]
    return {"metric": metric, "value": round(v, 4), "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic", "impl": "reference",
            "config": {"workload": f"BASELINE config {config}", "parallelism": "host cores"},
            "cpu_baseline": {"value": round(v, 4), "unit": unit, "cores": torch.get_num_threads(), "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(v, 4), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# keyed sub-blocks of the default line: every dense config at N=1; at N>1 the column-parallel
# sweep (config 4), the one dense config whose work is sharded over the ranks
SUB_BLOCKS = {"decode": 1, "prefill": 2, "linear": 0, "sweep": 4}
SUB_BLOCKS_MULTI = {"sweep": 4}
_RUN_KEYS = ("n_gpus", "steps", "warmup", "vs_baseline", "data", "impl")


def _sub_blocks(world):
    return SUB_BLOCKS if world == 1 else SUB_BLOCKS_MULTI


def _sub_block(line):
    """A config's line as a keyed sub-block of the default line (run-wide keys dropped)."""
    return {k: v for k, v in line.items() if k not in _RUN_KEYS}


def headline(args, world, rank, dev):
    """The default line: the MoE layer (config 3, expert-parallel at N>1) at the top level;
    the dense configs as keyed sub-blocks (all of them at N=1, the column-parallel sweep at
    N>1)."""
    runners = {0: run_config0, 1: run_config1, 2: run_config2, 4: run_config4}
    line, _ = run_config3(args, world, rank, dev)
    blocks = _sub_blocks(world)
    line["config"]["sub_blocks"] = {k: f"BASELINE config {c}" for k, c in blocks.items()}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_sample(3)
    torch.cuda.empty_cache()
    for key, c in blocks.items():
        sub, keep = runners[c](args, world, rank, dev)
        del keep
        torch.cuda.empty_cache()
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            sub["cpu_baseline"] = cpu_baseline_sample(c)
        line[key] = _sub_block(sub)
    return line


def reference_headline(args, world, rank):
    """The reference arm of the default line: the same workloads on the host cores."""
    line = reference_arm(args, world, rank, config=3)
    if line is None:
        return None
    blocks = _sub_blocks(world)
    line["config"]["sub_blocks"] = {k: f"BASELINE config {c}" for k, c in blocks.items()}
    for key, c in blocks.items():
        line[key] = _sub_block(reference_arm(args, world, rank, config=c))
    return line


def cpu_baseline_sample(config, seconds=8.0):
    """Bounded CPU sample of the same workload for the cpu_baseline key of our line."""
    torch.set_num_threads(os.cpu_count() or 1)
    step, work, scale, sample = cpu_workload(config)
    step()
    n, t0 = 0, time.perf_counter()
    while True:
        step()
        n += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = (time.perf_counter() - t0) / n
    return {"value": round(work / dt / scale, 4), "unit": METRICS[config][1], "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"{n} steps of {sample}"}


def json_channel():
    """The JSON line goes to the original stdout; everything else written to fd 1 for the
    rest of the run (NCCL's version banner, library notices) is sent to stderr, so rank 0's
    stdout carries exactly one line."""
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    return os.fdopen(saved, "w")


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=None, choices=[0, 1, 2, 3, 4],
                    help="one configuration alone (default: MoE line with decode/prefill sub-blocks)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_env()
    out = json_channel()

    if args.impl == "reference":
        line = reference_arm(args, world, rank) if args.config is not None else reference_headline(args, world, rank)
        if line is not None:
            print(json.dumps(line), file=out, flush=True)
        return 0

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    init_dist(world, local)
    runners = {0: run_config0, 1: run_config1, 2: run_config2, 3: run_config3, 4: run_config4}
    if args.config is None:
        line = headline(args, world, rank, dev)
    else:
        line, _ = runners[args.config](args, world, rank, dev)
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_sample(args.config)
    if rank == 0:
        print(json.dumps(line), file=out, flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
