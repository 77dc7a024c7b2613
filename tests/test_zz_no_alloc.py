"""vitb200_gemm_noalloc: the GEMM entry point for callers that cannot allocate
device memory (a C or ctypes program without a device allocator, a host whose
memory belongs to another framework's pool, a request path that cannot take
cudaMalloc's synchronisation). It keeps its TF32-pair scratch in a fixed array
inside the library, so its results must equal those of vitb200_gemm (which uses
a caller workspace), call after call, even though every call reuses the same
scratch. This file is collected last so that a failure here leaves every other
test already run.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _gemm_ws(vlib, x, w, b, res, epi):
    M, K = x.shape
    N = w.shape[0]
    y = torch.full((M, N), float("nan"), device=x.device)
    ws = torch.empty(max(vlib.lib.vitb200_gemm_workspace_bytes(M, K, N), 1), dtype=torch.uint8,
                     device=x.device)
    vlib.check(vlib.lib.vitb200_gemm(x.data_ptr(), w.data_ptr(), b.data_ptr(),
                                     res.data_ptr() if res is not None else None, y.data_ptr(),
                                     M, K, N, epi, ws.data_ptr(), ws.numel(),
                                     torch.cuda.current_stream().cuda_stream), "vitb200_gemm")
    return y


def _gemm_noalloc(vlib, x, w, b, res, epi):
    M, K = x.shape
    N = w.shape[0]
    y = torch.full((M, N), float("nan"), device=x.device)
    vlib.check(vlib.lib.vitb200_gemm_noalloc(x.data_ptr(), w.data_ptr(), b.data_ptr(),
                                             res.data_ptr() if res is not None else None,
                                             y.data_ptr(), M, K, N, epi,
                                             torch.cuda.current_stream().cuda_stream),
               "vitb200_gemm_noalloc")
    return y


def test_noalloc_matches_workspace_gemm_twice(vlib, cuda):
    # Two calls in a row: the second (smaller, odd K) runs on scratch still
    # holding the first call's pairs.
    cases = [((1024, 768, 1024), vlib.EPI_BIAS_GELU), ((300, 257, 700), vlib.EPI_BIAS_RESID)]
    torch.manual_seed(11)
    for (m, k, n), epi in cases:
        x = torch.randn(m, k, device=cuda)
        w = torch.randn(n, k, device=cuda) * 0.05
        b = torch.randn(n, device=cuda)
        res = torch.randn(m, n, device=cuda) if epi == vlib.EPI_BIAS_RESID else None
        ref = _gemm_ws(vlib, x, w, b, res, epi)
        out = _gemm_noalloc(vlib, x, w, b, res, epi)
        torch.cuda.synchronize()
        assert not torch.isnan(out).any()
        torch.testing.assert_close(out, ref, atol=1e-4, rtol=1e-5)


def test_noalloc_rejects_oversize(vlib, cuda):
    x = torch.empty(1, 4, device=cuda)
    st = vlib.lib.vitb200_gemm_noalloc(x.data_ptr(), x.data_ptr(), None, None, x.data_ptr(),
                                       4096, 1024, 1024, vlib.EPI_NONE,
                                       torch.cuda.current_stream().cuda_stream)
    assert st == vlib.E_WORKSPACE


def test_noalloc_rejects_sizes_that_would_wrap(vlib, cuda):
    # M * Kp overflows 64 bits: rejected by the size check, nothing launched.
    x = torch.empty(1, 4, device=cuda)
    for m, k, n in (((1 << 62), 1024, 16), (16, 1024, (1 << 31) - 1)):
        st = vlib.lib.vitb200_gemm_noalloc(x.data_ptr(), x.data_ptr(), None, None, x.data_ptr(),
                                           m, k, n, vlib.EPI_NONE,
                                           torch.cuda.current_stream().cuda_stream)
        assert st == vlib.E_WORKSPACE
