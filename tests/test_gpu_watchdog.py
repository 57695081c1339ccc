"""Failure detection on the GPU without a fault: a bounded wait that runs out.

Every spin-wait in the library's kernels gives up after a wall-clock budget, records a
code and lets the kernel end (fni8_common.cuh). fni8_watchdog_selftest launches a kernel
whose wait is on a flag that nothing sets, with a 20 ms budget, so the timeout path runs
on a healthy GPU. The test checks that
  * fni8_device_status reports the code once (and FNI8_ERR_DEVICE_TIMEOUT at the C ABI),
  * the shared scratch an abandoned reduction may leave dirty is zero again — the Python
    GEMM workspace and the allocation-free GEMM's built-in array, both deliberately filled
    with non-zero words before the timeout,
  * the context still works: GEMMs on both scratch areas are bit-exact afterwards.
"""
import ctypes

import pytest
import torch

from oracle import w8a8_oracle as O

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a B200")]


def _vp(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def test_bounded_wait_timeout_is_reported_once_and_scratch_recovered():
    import fni8
    from fni8 import _native as nat
    from fni8 import ops

    g = torch.Generator().manual_seed(3)
    M, N, K = 8, 6144, 4096
    a = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8)
    w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
    a_s = torch.rand(M, generator=g) * 0.01 + 1e-3
    w_s = torch.rand(N, generator=g) * 0.01 + 1e-3
    ref = O.dequant(O.int_mm_fast(a, w), a_s, w_s)
    qt = fni8.QTensor(w.cuda(), w_s.cuda())
    assert torch.equal(fni8.linear_q(a.cuda(), a_s.cuda(), qt).cpu(), ref)  # workspace exists now
    assert fni8.device_status() == 0

    ws = ops.WORKSPACE.get(torch.device("cuda", torch.cuda.current_device()))
    ws.fill_(0x5A)  # the partial sums an abandoned split-K / stream-K kernel could leave
    ops.watchdog_selftest(wait_us=20000, dirty_scratch=True)
    lib = nat.lib()
    code = ctypes.c_int(0)
    assert lib.fni8_device_status(ctypes.byref(code)) == nat.ERR_DEVICE_TIMEOUT
    assert code.value == 0x2F0
    assert b"0x2f0" in lib.fni8_last_error_message()
    ops.watchdog_selftest(wait_us=20000)
    assert fni8.device_status() == 0x2F0  # the Python wrapper re-zeroes the workspace
    assert fni8.device_status() == 0  # reported once
    assert int(torch.count_nonzero(ws)) == 0

    # the context still runs kernels, and both scratch areas are clean: bit-exact results
    for path in (nat.PATH_SPLITK, nat.PATH_STREAM, nat.PATH_AUTO):
        assert torch.equal(fni8.linear_q(a.cuda(), a_s.cuda(), qt, path=path).cpu(), ref), path
    out = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    d = [t.cuda() for t in (a, a_s, w, w_s)]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    nat.check(lib.fni8_gemm_w8a8_noalloc(*map(_vp, d), None, None, _vp(out), nat.F16, M, N, K, stream),
              "fni8_gemm_w8a8_noalloc")
    assert torch.equal(out.cpu(), ref)
    assert fni8.device_status() == 0



def test_peer_barrier_single_rank_and_timeout():
    """The peer-memory barrier (fni8_peer_barrier) on one GPU: with one rank it passes at
    once and all-gathers its payload; with a second "rank" whose flag nothing ever sets it
    gives up after its bound, fni8_device_status reports it once, and the GPU then runs a
    GEMM exactly (no rank waits for good)."""
    import ctypes

    import fni8
    from fni8 import _native as nat

    dev = torch.device("cuda", 0)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    flags = torch.zeros(2, dtype=torch.int32, device=dev)
    epoch = torch.zeros(1, dtype=torch.int32, device=dev)
    src = torch.arange(7, dtype=torch.int32, device=dev) + 100
    dst = torch.zeros(2 * 7, dtype=torch.int32, device=dev)
    pf = (ctypes.c_void_p * 1)(flags.data_ptr())
    pd = (ctypes.c_void_p * 1)(dst.data_ptr())
    for i in range(3):
        nat.call("fni8_peer_barrier", ctypes.cast(pf, ctypes.c_void_p), 1, 0, ctypes.c_void_p(epoch.data_ptr()),
                 ctypes.c_void_p(src.data_ptr()), 7, ctypes.cast(pd, ctypes.c_void_p), 1000000, st)
    torch.cuda.synchronize()
    assert int(epoch.item()) == 3 and int(flags[0].item()) == 3
    assert torch.equal(dst[:7].cpu(), torch.arange(7, dtype=torch.int32) + 100)
    assert fni8.device_status() == 0
    # rank 0 of 2: flags[1] (rank 1's word in this rank's buffer) is never set
    flags2 = torch.zeros(2, dtype=torch.int32, device=dev)
    other = torch.zeros(2, dtype=torch.int32, device=dev)  # stands in for rank 1's buffer
    pf2 = (ctypes.c_void_p * 2)(flags2.data_ptr(), other.data_ptr())
    epoch2 = torch.zeros(1, dtype=torch.int32, device=dev)
    nat.call("fni8_peer_barrier", ctypes.cast(pf2, ctypes.c_void_p), 2, 0, ctypes.c_void_p(epoch2.data_ptr()), None,
             0, None, 2000, st)
    torch.cuda.synchronize()
    assert int(other[0].item()) == 1  # this rank's arrival was stored into the peer's buffer
    assert fni8.device_status() == 0x703  # the barrier's code
    assert fni8.device_status() == 0  # reported once
    a = torch.randint(-127, 128, (64, 256), dtype=torch.int8, device=dev)
    w = torch.randint(-127, 128, (128, 256), dtype=torch.int8, device=dev)
    assert torch.equal(fni8.gemm_i32(a, w).cpu(), a.cpu().int() @ w.cpu().int().T)
