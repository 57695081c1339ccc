"""The allocation-free GEMM entry point (fni8_gemm_w8a8_noalloc), through the C ABI.

Some callers of this library cannot allocate device memory for a workspace: a serving
engine that has reserved all of HBM for weights and KV cache up front, or a host program
binding the C ABI through a bare FFI that has no device allocator. For them the skinny
GEMM takes its scratch from an array built into the library. This file calls that entry
point and checks every result against the CPU oracle (exact int32 sums, then the dequant
epilogue) and against fni8_gemm_w8a8_ex running the same stream-K kernel with a
caller-provided workspace: both are exact integer GEMMs with the same epilogue, so the
outputs must be identical. Identical calls are repeated three times in a row: the kernels
must hand the shared array back zeroed, or the repeats would differ.

It lives in its own file that sorts last, so a run that stops at the first failure has
already run every other test; it also passes when run alone in a fresh process.
"""
import ctypes

import pytest
import torch

from oracle import w8a8_oracle as O

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a B200")]


def _case(M, N, K, seed, dtype):
    g = torch.Generator().manual_seed(seed)
    a = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8)
    w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
    a_scale = torch.rand(M, generator=g) * 0.01 + 1e-3
    w_scale = torch.rand(N, generator=g) * 0.01 + 1e-3
    bias = torch.randn(N, generator=g).to(dtype)
    residual = torch.randn(M, N, generator=g).to(dtype)
    return a, a_scale, w, w_scale, bias, residual


def _vp(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("with_bias,with_residual", [(True, False), (False, False), (True, True), (False, True)])
def test_noalloc_gemm_matches_oracle_and_workspace_entry_point(dtype, with_bias, with_residual):
    from fni8 import _native as nat

    lib = nat.lib()
    dt = nat.F16 if dtype == torch.float16 else nat.BF16
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # the regular entry point's caller-provided workspace, zeroed once as it requires
    wsb = lib.fni8_gemm_workspace_bytes(32, 24576, 12288)
    ws = torch.zeros(max(wsb, 16), dtype=torch.uint8, device="cuda")
    for call, (M, N, K) in enumerate([(8, 6144, 4096), (32, 4096, 12288), (1, 640, 4112)]):
        a, a_scale, w, w_scale, bias, residual = _case(M, N, K, 100 + call, dtype)
        b = bias if with_bias else None
        r = residual if with_residual else None
        ref = O.dequant(O.int_mm_fast(a, w), a_scale, w_scale, bias=b, residual=r, out_dtype=dtype)
        d = [t.cuda() if t is not None else None for t in (a, a_scale, w, w_scale, b, r)]
        via_ws = torch.empty(M, N, dtype=dtype, device="cuda")
        nat.check(lib.fni8_gemm_w8a8_ex(*map(_vp, d), _vp(via_ws), dt, M, N, K, nat.PATH_STREAM, _vp(ws), ws.numel(),
                                        stream), "fni8_gemm_w8a8_ex")
        for rep in range(3):  # the same call three times: the built-in array must come back zeroed
            got = torch.full((M, N), float("nan"), dtype=dtype, device="cuda")
            nat.check(lib.fni8_gemm_w8a8_noalloc(*map(_vp, d), _vp(got), dt, M, N, K, stream),
                      "fni8_gemm_w8a8_noalloc")
            torch.cuda.synchronize()
            got_c = got.cpu()
            assert torch.equal(got_c, ref), f"call {call} rep {rep}: max diff {(got_c.float() - ref.float()).abs().max()}"
        assert torch.equal(via_ws.cpu(), ref)
    from fni8 import device_status

    assert device_status() == 0


def test_noalloc_gemm_rejects_sizes_beyond_its_scratch():
    """More than 32 rows is refused before any pointer is read. (The other limit, more than
    4 MiB of partial tiles, cannot be reached on a 148-SM B200 at 32 rows: the stream-K
    kernel then needs 148 x (128 x 32 + 1) int32 = 2.4 MB.)"""
    from fni8 import _native as nat

    lib = nat.lib()
    p = ctypes.c_void_p(16)  # never dereferenced: the size check fails first
    assert lib.fni8_gemm_w8a8_noalloc(p, p, p, p, None, None, p, nat.F16, 33, 4096, 4096, None) == \
        nat.ERR_UNSUPPORTED
    assert b"at most 32 rows" in lib.fni8_last_error_message()
