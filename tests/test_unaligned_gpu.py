"""Tensors that start one float past a 16-byte boundary (storage offset 1),
through the C-ABI GEMM and the per-op wrappers.

The reference feeds offset-by-one views of X and W to its C-ABI GEMM on a
non-default stream, twice per shape with fresh data in the same buffers, over
odd and zero K, M and N (tests/test_cute_pipeline.py:15-40 of the reference
project), at atol 1e-4 / rtol 1e-5 against FP64. This suite does the same and
also offsets the bias, the residual and the output, so the epilogue's scalar
paths (taken when a row or vector is not 16-byte aligned) run; their results
must equal the aligned call's bit for bit, and nothing outside the output view
may be written.
"""
import pytest
import torch
import torch.nn.functional as F

import vit_cuda
from oracle import vit_oracle as orc
from test_gemm_gpu import check_fp32_parity, run_gemm

pytestmark = pytest.mark.gpu

CASES = [(35, k, 37) for k in (0, 1, 31, 32, 33, 64, 65, 96, 97, 257, 1025)]
CASES += [(0, 65, 37), (35, 65, 0), (300, 768, 768), (197, 768, 3072)]
EPIS = {"none": 0, "bias": 1, "gelu": 2, "resid": 3}


def offset_empty(shape, device, offset=1, fill=float("nan")):
    """A tensor of `shape` starting `offset` floats into a larger buffer (not
    16-byte aligned for offset 1); returns (view, whole buffer)."""
    n = 1
    for d in shape:
        n *= d
    buf = torch.full((n + offset + 4,), fill, device=device)
    return buf[offset:offset + n].view(shape), buf


def offset_copy(t, offset=1):
    v, _ = offset_empty(tuple(t.shape), t.device, offset)
    v.copy_(t)
    return v


def gemm_views(vlib, x, w, bias, res, y, epi):
    M, K = x.shape
    N = w.shape[0]
    ws = torch.empty(max(vlib.lib.vitb200_gemm_workspace_bytes(M, K, N), 1), dtype=torch.uint8,
                     device=x.device)
    vlib.check(vlib.lib.vitb200_gemm(x.data_ptr(), w.data_ptr(),
                                     bias.data_ptr() if epi != "none" else None,
                                     res.data_ptr() if epi == "resid" else None, y.data_ptr(),
                                     M, K, N, EPIS[epi], ws.data_ptr(), ws.numel(),
                                     torch.cuda.current_stream().cuda_stream), "vitb200_gemm")


@pytest.mark.parametrize("case", range(len(CASES)))
def test_gemm_offset_views_reused(vlib, cuda, case):
    m, k, n = CASES[case]
    gen = torch.Generator(device=cuda).manual_seed(100 + case)
    stream = torch.cuda.Stream(cuda)
    with torch.cuda.stream(stream):
        x, _ = offset_empty((m, k), cuda)
        w, _ = offset_empty((n, k), cuda)
        bias, _ = offset_empty((n,), cuda)
        res, _ = offset_empty((m, n), cuda)
        for _ in range(2):  # the same buffers refilled (the reference's reuse check)
            for t in (x, w, bias, res):
                t.copy_(torch.randn(t.shape, device=cuda, generator=gen))
            for epi in EPIS:
                y, ybuf = offset_empty((m, n), cuda, fill=1234.5)
                gemm_views(vlib, x, w, bias, res, y, epi)
                aligned = run_gemm(vlib, x.contiguous().clone(), w.clone(), bias.clone(),
                                   res.clone() if epi == "resid" else None, epi)
                stream.synchronize()
                if m and n:
                    check_fp32_parity(y, x, w, bias, res, epi)
                    torch.testing.assert_close(y, aligned, atol=0, rtol=0)
                assert ybuf[0].item() == 1234.5 and (ybuf[1 + m * n:] == 1234.5).all()


def test_gemm_bias_offset_views(cuda):
    """vit_cuda.gemm_bias (reference csrc/ops/gemm_wrapper.cpp:16-59) on offset
    X, W and bias, 2-D and 3-D, against the oracle's linear at the reference
    GEMM tests' tolerance."""
    torch.manual_seed(3)
    for shape in ((8, 768), (2, 197, 768)):
        x = torch.randn(shape)
        w = torch.randn(3072, 768) * 0.05
        b = torch.randn(3072)
        out = vit_cuda.gemm_bias(offset_copy(x.to(cuda)), offset_copy(w.to(cuda)),
                                 offset_copy(b.to(cuda)))
        torch.testing.assert_close(out.double().cpu(), orc.linear(x, w, b), atol=1e-4,
                                   rtol=1e-5)


def test_mlp_forward_offset_views(cuda):
    """vit_cuda.mlp_forward (reference csrc/ops/mlp_wrapper.cpp:20-64) on offset
    X, W1, b1, W2 and b2: [O, H] against the oracle at the reference MLP test's
    tolerances (tests/test_mlp.py: H atol 5e-4, O atol 3e-2 rtol 3e-3 with
    unit-variance weights)."""
    torch.manual_seed(4)
    x = torch.randn(2, 197, 768)
    w1, b1 = torch.randn(3072, 768), torch.randn(3072)
    w2, b2 = torch.randn(768, 3072), torch.randn(768)
    o, h = vit_cuda.mlp_forward(*(offset_copy(t.to(cuda)) for t in (x, w1, b1, w2, b2)))
    eo, eh = orc.mlp(x, w1, b1, w2, b2)
    torch.testing.assert_close(h.double().cpu(), eh, atol=5e-4, rtol=0)
    torch.testing.assert_close(o.double().cpu(), eo, atol=3e-2, rtol=3e-3)
    # and the same values as the aligned call
    o2, h2 = vit_cuda.mlp_forward(*(t.to(cuda) for t in (x, w1, b1, w2, b2)))
    torch.testing.assert_close(o, o2, atol=0, rtol=0)
    torch.testing.assert_close(h, h2, atol=0, rtol=0)
