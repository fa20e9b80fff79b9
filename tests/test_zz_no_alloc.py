"""The no-allocation entry point, checked last.

d1_gemm_wgrad_noalloc serves callers that cannot allocate device memory (a host
framework that owns all of HBM, a plugin that must not call cudaMalloc after
start-up): its split-K scratch is a fixed array inside the library. This test
calls it through the C ABI and compares it with the regular path, where the
caller provides the scratch slabs (d1_gemm + d1_reduce_slabs), on two calls in a
row, and checks that an oversized request is refused. The file is named so that
pytest collects it after every other test.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_no_alloc_weight_gradient_matches_the_caller_scratch_path():
    from d1._lib import ERR_TOO_LARGE, library
    lib = library()
    M, N, K, splits = 256, 1832, 16384, 8
    g = torch.Generator(device='cuda').manual_seed(17)
    a = torch.randn(M, K, device='cuda', generator=g).to(torch.bfloat16)
    b = torch.randn(N, K, device='cuda', generator=g).to(torch.bfloat16)
    used = lib.d1_gemm_splits(K, splits)
    ld = (N + 3) // 4 * 4
    slabs = torch.empty((used, M, ld), device='cuda')
    assert lib.d1_gemm(a.data_ptr(), K, b.data_ptr(), K, M, N, K, None, 0, None, 0, None, 0, None, 0,
                       slabs.data_ptr(), ld, used, 0) == 0
    ref = slabs[:, :, :N].sum(0)  # same per-element order as the library's reductions
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        out = torch.full((M, N), float('nan'), device='cuda')
        assert lib.d1_gemm_wgrad_noalloc(a.data_ptr(), K, b.data_ptr(), K, M, N, K, out.data_ptr(), N, splits,
                                         stream) == 0
        torch.cuda.synchronize()
        assert torch.isfinite(out).all(), call
        assert torch.allclose(out, ref, rtol=1e-6, atol=1e-4), (call, (out - ref).abs().max().item())
    exact = (a.float() @ b.float().T)
    assert torch.allclose(out, exact, rtol=1e-4, atol=1e-2)
    big = lib.d1_gemm_wgrad_noalloc(a.data_ptr(), K, b.data_ptr(), K, M, N, K, out.data_ptr(), N, 64, stream)
    assert big == ERR_TOO_LARGE
