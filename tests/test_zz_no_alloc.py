"""The allocation-free GEMM entry point (fni8_gemm_w8a8_noalloc) against the regular one.

Some callers of this library cannot allocate device memory for a workspace: a serving
engine that has reserved all of HBM for weights and KV cache up front, or a host program
binding the C ABI through a bare FFI that has no device allocator. For them the skinny
GEMM takes its scratch from an array built into the library. This file calls that entry
point through the C ABI twice in a row and checks each result against
fni8_gemm_w8a8_ex on the same skinny (stream-K) kernel with a caller-provided workspace;
both are exact integer GEMMs with the same epilogue, so the outputs must be identical.

It lives in its own file that sorts last, so a run that stops at the first failure has
already run every other test; it also passes when run alone in a fresh process.
"""
import ctypes

import pytest
import torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a B200")]


def _case(M, N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randint(-127, 128, (M, K), generator=g, device="cuda", dtype=torch.int8)
    w = torch.randint(-127, 128, (N, K), generator=g, device="cuda", dtype=torch.int8)
    a_scale = torch.rand(M, generator=g, device="cuda") * 0.01 + 1e-3
    w_scale = torch.rand(N, generator=g, device="cuda") * 0.01 + 1e-3
    bias = torch.randn(N, generator=g, device="cuda").half()
    return a, a_scale, w, w_scale, bias


def _vp(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def test_noalloc_gemm_matches_workspace_entry_point():
    from fni8 import _native as nat

    lib = nat.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # the regular entry point's caller-provided workspace, zeroed once as it requires
    wsb = lib.fni8_gemm_workspace_bytes(32, 24576, 12288)
    ws = torch.zeros(max(wsb, 16), dtype=torch.uint8, device="cuda")
    for call, (M, N, K) in enumerate([(8, 6144, 4096), (32, 4096, 12288)]):
        a, a_scale, w, w_scale, bias = _case(M, N, K, 100 + call)
        ref = torch.empty(M, N, dtype=torch.float16, device="cuda")
        got = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
        nat.check(lib.fni8_gemm_w8a8_ex(_vp(a), _vp(a_scale), _vp(w), _vp(w_scale), _vp(bias), None, _vp(ref),
                                        nat.F16, M, N, K, nat.PATH_STREAM, _vp(ws), ws.numel(), stream),
                  "fni8_gemm_w8a8_ex")
        nat.check(lib.fni8_gemm_w8a8_noalloc(_vp(a), _vp(a_scale), _vp(w), _vp(w_scale), _vp(bias), None, _vp(got),
                                             nat.F16, M, N, K, stream), "fni8_gemm_w8a8_noalloc")
        torch.cuda.synchronize()
        assert torch.equal(got, ref), f"call {call}: max diff {(got.float() - ref.float()).abs().max()}"


def test_noalloc_gemm_rejects_sizes_beyond_its_scratch():
    from fni8 import _native as nat

    lib = nat.lib()
    p = ctypes.c_void_p(16)  # never dereferenced: the size check fails first
    assert lib.fni8_gemm_w8a8_noalloc(p, p, p, p, None, None, p, nat.F16, 33, 4096, 4096, None) == \
        nat.ERR_UNSUPPORTED
    assert b"at most 32 rows" in lib.fni8_last_error_message()
