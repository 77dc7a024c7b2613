"""TF32x3 tcgen05 GEMM through the C ABI (vitb200_gemm / vitb200_gemm_pairs).

Mirrors the reference's C-ABI GEMM checks (tests/test_cute_gemm.py:18-114 of the
reference project: odd and zero shapes, the three epilogues, an FP64
expectation at atol 1e-4 / rtol 1e-5, the TF32x3-vs-single-TF32 error ratio,
NaN-prefilled outputs, a non-default stream) and adds the ViT shapes, the
residual epilogue and every tile configuration.
"""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

SHAPES = [
    (1, 1, 1), (3, 63, 67), (31, 33, 31), (32, 32, 32), (35, 65, 37),
    (8, 768, 3072), (394, 768, 2304), (197, 3072, 768), (300, 257, 1000),
    (0, 17, 19), (3, 17, 0), (3, 0, 7),
]
EPILOGUES = ["none", "bias", "gelu", "resid"]
# More output tiles than SMs, so each persistent CTA runs several tiles and both
# epilogue warpgroups take turns (odd chunk counts included: K=300 -> 5 chunks).
MULTI_TILE = [(4096, 768, 3072), (3000, 64, 1000), (2100, 300, 1300), (50432, 768, 768)]


def run_gemm(vlib, x, w, bias=None, residual=None, epi="bias"):
    M, K = x.shape
    N = w.shape[0]
    code = {"none": vlib.EPI_NONE, "bias": vlib.EPI_BIAS, "gelu": vlib.EPI_BIAS_GELU,
            "resid": vlib.EPI_BIAS_RESID}[epi]
    y = torch.full((M, N), float("nan"), device=x.device)
    ws_bytes = vlib.lib.vitb200_gemm_workspace_bytes(M, K, N)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
    st = vlib.lib.vitb200_gemm(x.data_ptr(), w.data_ptr(),
                               bias.data_ptr() if bias is not None else None,
                               residual.data_ptr() if residual is not None else None,
                               y.data_ptr(), M, K, N, code, ws.data_ptr(), ws.numel(),
                               torch.cuda.current_stream().cuda_stream)
    vlib.check(st, "vitb200_gemm")
    return y


def expected(x, w, bias, residual, epi):
    e = x.double() @ w.double().t()
    if epi != "none":
        e = e + bias.double()
    if epi == "gelu":
        e = F.gelu(e, approximate="none")
    if epi == "resid":
        e = residual.double() + e
    return e.float()


def check_fp32_parity(y, x, w, bias, res, epi):
    """The reference's bar (atol 1e-4, rtol 1e-5 against FP64) for the reduction
    lengths its tests use (K <= 768); for longer unit-variance reductions, where
    plain FP32 accumulation itself exceeds that bar, the error must be no larger
    than cuBLAS FP32's (TF32 disabled) on the same inputs."""
    e = expected(x, w, bias, res, epi)
    if x.shape[1] <= 768:
        torch.testing.assert_close(y, e, atol=1e-4, rtol=1e-5)
        return
    e64 = x.double() @ w.double().t()
    f32 = x @ w.t()
    ours = (y.double() - e.double()).abs().max().item()
    cublas = (f32.double() - e64).abs().max().item()
    assert ours <= max(1.5 * cublas, 1e-4), (ours, cublas)


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("epi", EPILOGUES)
def test_gemm_shapes(vlib, cuda, shape, epi):
    torch.manual_seed(0)
    m, k, n = shape
    x = torch.randn(m, k, device=cuda)
    w = torch.randn(n, k, device=cuda)
    bias = torch.randn(n, device=cuda)
    res = torch.randn(m, n, device=cuda)
    y = run_gemm(vlib, x, w, bias, res if epi == "resid" else None, epi)
    check_fp32_parity(y, x, w, bias, res, epi)


@pytest.mark.parametrize("shape", MULTI_TILE)
@pytest.mark.parametrize("epi", ["bias", "resid"])
def test_gemm_multi_tile(vlib, cuda, shape, epi):
    torch.manual_seed(3)
    m, k, n = shape
    x = torch.randn(m, k, device=cuda)
    w = torch.randn(n, k, device=cuda)
    bias = torch.randn(n, device=cuda)
    res = torch.randn(m, n, device=cuda)
    y = run_gemm(vlib, x, w, bias, res if epi == "resid" else None, epi)
    check_fp32_parity(y, x, w, bias, res, epi)


@pytest.mark.parametrize("variant", [1, 2, 3, 4, 5, 6, 7, 8])
@pytest.mark.parametrize("shape", [(394, 768, 2304), (200, 3072, 768), (130, 96, 520),
                                   (2100, 300, 1300)])
def test_gemm_variants(vlib, cuda, variant, shape):
    old = vlib.lib.vitb200_set_gemm_variant(variant)
    try:
        torch.manual_seed(1)
        m, k, n = shape
        x = torch.randn(m, k, device=cuda)
        w = torch.randn(n, k, device=cuda) * 0.02
        bias = torch.randn(n, device=cuda) * 0.02
        y = run_gemm(vlib, x, w, bias, None, "gelu")
        torch.testing.assert_close(y, expected(x, w, bias, None, "gelu"), atol=1e-5, rtol=1e-5)
    finally:
        vlib.lib.vitb200_set_gemm_variant(old)


def test_residual_correction(vlib, cuda):
    """Three TF32 products beat one rounded product by > 100x in RMSE
    (reference tests/test_cute_gemm.py:69-86)."""
    torch.manual_seed(1)
    x = torch.randn(127, 257, device=cuda)
    w = torch.randn(129, 257, device=cuda)
    reference = x.double() @ w.double().t()
    actual = run_gemm(vlib, x, w, None, None, "none")

    def round_tf32(t):
        bits = t.view(torch.int32)
        return ((bits + 0xFFF + ((bits >> 13) & 1)) & -8192).view(torch.float32)

    single = round_tf32(x).double() @ round_tf32(w).double().t()
    err = (actual.double() - reference).square().mean().sqrt().item()
    single_err = (single - reference).square().mean().sqrt().item()
    assert err < single_err / 100, (err, single_err)


def test_current_stream(vlib, cuda):
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        x = torch.randn(19, 77, device=cuda)
        w = torch.randn(35, 77, device=cuda)
        bias = torch.randn(35, device=cuda)
        y = run_gemm(vlib, x, w, bias, None, "bias")
        e = F.linear(x.double(), w.double(), bias.double()).float()
    stream.synchronize()
    torch.testing.assert_close(y, e, atol=1e-4, rtol=1e-5)


def test_gemm_pairs_pair_output(vlib, cuda):
    """The epilogue's TF32 pair output re-sums to the fp32 output."""
    torch.manual_seed(2)
    M, K, N = 256, 768, 3072
    x = torch.randn(M, K, device=cuda)
    w = torch.randn(N, K, device=cuda) * 0.02
    b = torch.randn(N, device=cuda) * 0.02
    s = torch.cuda.current_stream().cuda_stream
    xp = torch.empty(2, M, K, device=cuda)
    wp = torch.empty(2, N, K, device=cuda)
    vlib.check(vlib.lib.vitb200_split_tf32(x.data_ptr(), M, K, K, xp.data_ptr(), K, s), "split")
    vlib.check(vlib.lib.vitb200_split_tf32(w.data_ptr(), N, K, K, wp.data_ptr(), K, s), "split")
    torch.testing.assert_close(xp[0] + xp[1], x, atol=0, rtol=2e-7)
    y = torch.full((M, N), float("nan"), device=cuda)
    yp = torch.full((2, M, N), float("nan"), device=cuda)
    vlib.check(vlib.lib.vitb200_gemm_pairs(xp.data_ptr(), wp.data_ptr(), b.data_ptr(), None,
                                           y.data_ptr(), N, yp.data_ptr(), M, K, N,
                                           vlib.EPI_BIAS_GELU, s), "gemm_pairs")
    e = F.gelu(x.double() @ w.double().t() + b.double(), approximate="none").float()
    torch.testing.assert_close(y, e, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(yp[0] + yp[1], y, atol=0, rtol=2e-7)
    # hi has its low 13 mantissa bits clear (exactly representable in TF32)
    assert int((yp[0].view(torch.int32) & 0x1FFF).abs().max().item()) == 0


def test_bad_arguments(vlib, cuda):
    lib = vlib.lib
    s = torch.cuda.current_stream().cuda_stream
    x = torch.randn(4, 8, device=cuda)
    y = torch.empty(4, 4, device=cuda)
    # bias epilogue without a bias
    assert lib.vitb200_gemm(x.data_ptr(), x.data_ptr(), None, None, y.data_ptr(), 4, 8, 4,
                            vlib.EPI_BIAS, None, 0, s) == vlib.E_INVALID_ARG
    # workspace too small
    assert lib.vitb200_gemm(x.data_ptr(), x.data_ptr(), None, None, y.data_ptr(), 4, 8, 4,
                            vlib.EPI_NONE, y.data_ptr(), 16, s) == vlib.E_WORKSPACE
    # misaligned pair pointer
    assert lib.vitb200_gemm_pairs(x.data_ptr() + 4, x.data_ptr(), None, None, y.data_ptr(), 4,
                                  None, 1, 4, 4, vlib.EPI_NONE, s) == vlib.E_ALIGNMENT


def test_gelu_epilogue_accuracy(vlib, cuda):
    """The GEMM epilogue's GELU (a fitted polynomial for the normal tail and one
    ex2; no erff) against float64 GELU and against torch's fp32 GELU on the
    GPU: X holds 16,384 values over [-12, 12] plus tiny ones, W = I, so
    Y = GELU(X) up to the TF32x3 identity product (2^-22 relative)."""
    torch.manual_seed(7)
    k = 256
    vals = torch.cat([torch.linspace(-12, 12, 64 * k - 2 * k),
                      torch.logspace(-30, 0, k) * torch.sign(torch.randn(k)),
                      torch.randn(k) * 3])
    x = vals.view(64, k).to(cuda)
    w = torch.eye(k, device=cuda)
    b = torch.zeros(k, device=cuda)
    y = run_gemm(vlib, x, w, b, None, "gelu").double()
    x64 = x.double()
    g64 = F.gelu(x64, approximate="none")
    err = (y - g64).abs()
    assert (err <= 2.5e-6 * x64.abs() + 1e-37).all(), err.max().item()
    g32 = F.gelu(x, approximate="none").double()  # CUDA's erff-based GELU in fp32
    assert ((y - g32).abs() <= 3e-6 * x64.abs() + 1e-37).all()
    # FP16-split path: same epilogue code, bounded inputs
    from test_gemm_f16_gpu import run_f16
    xs = (x[:, :] / 2).contiguous()
    yf = run_f16(vlib, xs, w, b, None, "gelu").double()
    gf = F.gelu(xs.double(), approximate="none")
    # (the FP16 split itself is exact to 2^-22 relative + 2^-36 absolute)
    assert ((yf - gf).abs() <= 2.5e-6 * xs.double().abs() + 1e-10).all()
