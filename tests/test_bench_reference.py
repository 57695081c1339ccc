"""bench.py's reference arm runs on the host alone (the CPU W8A8 path BASELINE.json names:
int8 matmul + fp32 dequant) and prints the one-line JSON contract: checked here without a
GPU on the smallest config."""
import json
import os
import subprocess
import sys

from conftest import ROOT

KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"}


def test_reference_arm_prints_the_contract_line():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--config", "0",
                          "--steps", "1", "--warmup", "1"], capture_output=True, text=True, timeout=600, env=env,
                         cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    assert KEYS <= set(d), KEYS - set(d)
    assert d["impl"] == "reference" and d["value"] > 0 and d["unit"] == "TOP/s"
    assert d["warmup"] >= 3  # the contract's minimum
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0


def test_reference_arm_under_torchrun_prints_once():
    """The driver launches the reference arm for N > 1 exactly like our arm (torchrun, one
    process per GPU): rank 0 alone times the host path and prints; the other ranks exit 0
    without work, so the run yields exactly one JSON line with n_gpus = N."""
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", str(port), os.path.join(ROOT, "bench.py"), "--impl", "reference", "--gpus", "2",
           "--config", "0", "--steps", "1", "--warmup", "3"]
    out = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["value"] > 0


def test_reference_arm_default_line_carries_the_three_metrics():
    """The default run (no --config) is BASELINE.json's metric in one line: MoE tokens/s at
    the top level, decode GB/s and prefill TOP/s as keyed sub-blocks at N=1, each a timed
    run of the host path with its own cpu_baseline."""
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "1"], capture_output=True, text=True, timeout=900, env=env, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    assert KEYS <= set(d) and d["unit"] == "tokens/s" and d["value"] > 0
    for key, unit in (("decode", "GB/s"), ("prefill", "TOP/s")):
        sub = d[key]
        assert sub["unit"] == unit and sub["value"] > 0 and sub["cpu_baseline"]["value"] == sub["value"]
        assert sub["e2e"]["h2d_bytes_per_step"] == 0
