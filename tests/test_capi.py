"""The C ABI library loads, exports every function include/fni8_b200.h declares, and
rejects bad arguments on the host before any launch (runs without a GPU)."""
import ctypes
import os
import re
import subprocess

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "fni8_b200.h")


def declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^FNI8_API\s+[\w\s\*]+?\b(fni8_\w+)\s*\(", src, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    from fni8 import _native

    if not os.path.exists(_native.LIB_PATH):
        pytest.fail(f"{_native.LIB_PATH} not built (run python fni8-serve_b200/build.py)")
    return _native.lib()


def test_header_declares_entry_points():
    names = declared()
    assert len(names) >= 20
    for must in ("fni8_linear_w8a8", "fni8_gemm_w8a8", "fni8_rmsnorm_quant_i8", "fni8_grouped_gemm_w8a8",
                 "fni8_moe_route", "fni8_moe_experts_w8a8"):
        assert must in names


def test_library_exports_every_declared_symbol(lib):
    from fni8 import _native

    out = subprocess.run(["nm", "-D", "--defined-only", _native.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    missing = [n for n in declared() if n not in exported]
    assert not missing, missing
    assert set(_native.SIGNATURES) == set(declared()), "ctypes table out of sync with the header"
    for n in declared():
        getattr(lib, n)  # resolvable through ctypes


def test_library_has_no_libcuda_dependency():
    from fni8 import _native

    out = subprocess.run(["readelf", "-d", _native.LIB_PATH], capture_output=True, text=True, check=True).stdout
    assert "libcuda.so" not in out  # loads on a machine without the driver


def test_status_strings(lib):
    from fni8 import _native as n

    assert lib.fni8_abi_version() == 1
    assert lib.fni8_status_string(n.OK) == b"ok"
    assert b"invalid" in lib.fni8_status_string(n.ERR_INVALID)
    assert lib.fni8_status_string(99) == b"unknown status"


def test_argument_validation_without_launch(lib):
    """Every one of these fails on the host, before any CUDA call."""
    from fni8 import _native as n

    p = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    # K not a multiple of 16
    assert lib.fni8_gemm_w8a8(p, p, p, p, None, None, p, n.F16, 4, 8, 24, None, 0, None) == n.ERR_UNSUPPORTED
    assert b"multiple of 16" in lib.fni8_last_error_message()
    # negative M, bad dtype, bad path
    assert lib.fni8_gemm_w8a8(p, p, p, p, None, None, p, n.F16, -1, 8, 32, None, 0, None) == n.ERR_INVALID
    assert lib.fni8_gemm_w8a8(p, p, p, p, None, None, p, 7, 4, 8, 32, None, 0, None) == n.ERR_INVALID
    assert lib.fni8_gemm_w8a8_ex(p, p, p, p, None, None, p, n.F16, 4, 8, 32, 9, None, 0, None) == n.ERR_INVALID
    assert lib.fni8_gemm_w8a8_ex(p, p, p, p, None, None, p, n.F16, 300, 8, 32, n.PATH_STREAM, None, 0,
                                 None) == n.ERR_UNSUPPORTED
    # quantiser: null output, bad dtype
    assert lib.fni8_quantize_rows_i8(p, n.F16, 4, 32, None, None, None) == n.ERR_INVALID
    assert lib.fni8_quantize_rows_i8(p, n.F32, 4, 32, p, p, None) == n.ERR_INVALID
    # rmsnorm: residual without residual_out
    assert lib.fni8_rmsnorm(p, p, p, n.F16, 4, 32, ctypes.c_float(1e-6), 0, p, None, None) == n.ERR_INVALID
    assert lib.fni8_act_and_mul(p, n.F16, 5, 4, 32, p, None) == n.ERR_INVALID
    # MoE
    assert lib.fni8_moe_route(p, 4, 2000, 2, 0, None, 0, 0, 1, ctypes.c_float(1.0), n.F16, p, p,
                              None) == n.ERR_INVALID
    assert lib.fni8_moe_route(p, 4, 8, 9, 0, None, 0, 0, 1, ctypes.c_float(1.0), n.F16, p, p, None) == n.ERR_INVALID
    assert lib.fni8_moe_route(p, 4, 8, 2, 0, None, 3, 1, 1, ctypes.c_float(1.0), n.F16, p, p,
                              None) == n.ERR_INVALID  # 8 experts do not split into 3 groups
    assert lib.fni8_moe_plan(p, 16, 8, p, p, p, p, None, 0, None) == n.ERR_WORKSPACE
    assert lib.fni8_grouped_gemm_w8a8(p, p, 16, p, p, 4, 64, 40, p, p, p, 4, p, n.F16,
                                      None) == n.ERR_UNSUPPORTED
    assert lib.fni8_moe_experts_w8a8(p, n.F16, 8, 256, p, p, 2, p, p, p, p, 600, 128, 0, p, p, 1 << 30,
                                     None) == n.ERR_UNSUPPORTED  # more experts than one grouped launch takes
    # expert-parallel exchange: world, expert split, row width, slot range, dtype
    peers = (ctypes.c_void_p * 2)(16, 32)
    pp = ctypes.cast(peers, ctypes.c_void_p)
    assert lib.fni8_ep_dispatch_i8(p, p, p, p, 16, 9, 0, 4, 512, p, pp, pp, pp, 100, 100, None) == n.ERR_INVALID
    assert lib.fni8_ep_dispatch_i8(p, p, p, p, 15, 2, 0, 4, 512, p, pp, pp, pp, 100, 100, None) == n.ERR_INVALID
    assert lib.fni8_ep_dispatch_i8(p, p, p, p, 16, 2, 0, 4, 520, p, pp, pp, pp, 100, 100, None) == n.ERR_UNSUPPORTED
    assert lib.fni8_ep_dispatch_i8(p, p, p, p, 16, 2, 0, 4, 512, p, pp, pp, pp, 100, 1 << 24,
                                   None) == n.ERR_UNSUPPORTED  # tags hold slots below 2^24
    assert lib.fni8_ep_dispatch_i8(p, p, p, p, 16, 2, 2, 4, 512, p, pp, pp, pp, 100, 100, None) == n.ERR_INVALID
    assert lib.fni8_ep_return(p, n.F32, p, 100, p, 512, 2, pp, 100, None) == n.ERR_INVALID
    assert lib.fni8_ep_return(p, n.F16, p, 100, p, 12, 2, pp, 100, None) == n.ERR_UNSUPPORTED
    # fused expert return: world, row width
    assert lib.fni8_grouped_gemm_w8a8_scatter(p, p, 16, p, p, 4, 64, 64, p, p, p, 4, p, pp, 9, 100, n.F16,
                                              None) == n.ERR_INVALID
    assert lib.fni8_grouped_gemm_w8a8_scatter(p, p, 16, p, p, 4, 48, 64, p, p, p, 4, p, pp, 2, 100, n.F16,
                                              None) == n.ERR_UNSUPPORTED
    assert lib.fni8_grouped_gemm_w8a8_scatter(p, p, 16, p, p, 4, 64, 64, p, p, p, 4, p, pp, 2, 100, n.I32,
                                              None) == n.ERR_INVALID
    # column all-gather GEMM: destination count, shard width, column range, alignment
    pc = lib.fni8_gemm_w8a8_peer_cols
    assert pc(p, p, p, p, None, n.F16, 4, 64, 256, pp, 0, 256, 0, None, 0, None, 0, None) == n.ERR_INVALID
    assert pc(p, p, p, p, None, n.F16, 4, 64, 256, pp, 9, 256, 0, None, 0, None, 0, None) == n.ERR_INVALID
    assert pc(p, p, p, p, None, n.F16, 4, 48, 256, pp, 2, 256, 0, None, 0, None, 0, None) == n.ERR_UNSUPPORTED
    assert pc(p, p, p, p, None, n.F16, 4, 64, 256, pp, 2, 256, 200, None, 0, None, 0, None) == n.ERR_INVALID
    assert pc(p, p, p, p, None, n.F16, 4, 64, 256, pp, 2, 260, 4, None, 0, None, 0, None) == n.ERR_ALIGN
    assert pc(p, p, p, p, None, n.F32, 4, 64, 256, pp, 2, 256, 0, None, 0, None, 0, None) == n.ERR_INVALID
    assert pc(p, p, p, p, None, n.F16, 0, 64, 256, pp, 2, 256, 0, None, 0, None, 0, None) == n.OK
    assert lib.fni8_ipc_alloc(0, ctypes.byref(ctypes.c_void_p()), p) == n.ERR_INVALID
    assert lib.fni8_ipc_open(None, ctypes.byref(ctypes.c_void_p())) == n.ERR_INVALID
    assert lib.fni8_act_and_mul_quant_i8_rows(p, n.F16, 0, 4, 32, None, p, p, None) == n.ERR_INVALID
    # watchdog self-test: the wait budget must lie in 1 us .. 1 s
    assert lib.fni8_watchdog_selftest(0, 0, None) == n.ERR_INVALID
    assert lib.fni8_watchdog_selftest(2_000_000, 1, None) == n.ERR_INVALID
    # zero-size work is a successful no-op (no launch)
    assert lib.fni8_ep_dispatch_i8(None, None, None, None, 16, 2, 0, 4, 512, None, pp, pp, pp, 0, 0, None) == n.OK
    assert lib.fni8_ep_return(None, n.F16, None, 0, None, 512, 2, pp, 0, None) == n.OK
    assert lib.fni8_ipc_close(None) == n.OK and lib.fni8_ipc_free(None) == n.OK
    assert lib.fni8_gemm_w8a8(None, None, None, None, None, None, None, n.F16, 0, 8, 32, None, 0, None) == n.OK
    assert lib.fni8_quantize_rows_i8(p, n.F16, 0, 32, None, None, None) == n.OK


def test_workspace_sizes(lib):
    assert lib.fni8_gemm_workspace_bytes(512, 64, 64) == 0  # tile path needs none
    assert lib.fni8_moe_plan_workspace_bytes(32768, 128) >= 32 * 128 * 4
    assert lib.fni8_moe_experts_workspace_bytes(4096, 2048, 8, 128, 768) > 32768 * 2048


def test_ops_reject_cpu_tensors():
    """No CPU path: the product ops raise instead of computing on the host."""
    import torch

    import fni8

    x = torch.randn(4, 64, dtype=torch.float16)
    qt = fni8.QTensor(torch.zeros(32, 64, dtype=torch.int8), torch.ones(32), scheme="per_row_i8")
    for fn in (lambda: fni8.linear(x, qt), lambda: fni8.rmsnorm(x, torch.ones(64), 1e-6),
               lambda: fni8.act_and_mul(x), lambda: fni8.quantize_rows(x)):
        with pytest.raises(RuntimeError, match="CUDA"):
            fn()
