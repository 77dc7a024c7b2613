"""Three-product FP16-split GEMM through the C ABI (vitb200_split_f16 +
vitb200_gemm_f16), held to the same FP32-parity bar as the TF32x3 GEMM
(reference tests/test_cute_gemm.py:18-114: FP64 expectation, atol 1e-4 /
rtol 1e-5 for K <= 768, odd and zero shapes, the epilogues), plus the split's
own error bound and range check, and an accuracy comparison with TF32x3.
"""
import pytest
import torch

from test_gemm_gpu import EPILOGUES, MULTI_TILE, SHAPES, check_fp32_parity, expected, run_gemm
from vit_cuda.split import F16_LO_SCALE, f16_combine, f16_planes, f16_weight

pytestmark = pytest.mark.gpu


def run_f16(vlib, x, w, bias=None, residual=None, epi="bias", want_h16=False):
    M, K = x.shape
    N = w.shape[0]
    code = {"none": vlib.EPI_NONE, "bias": vlib.EPI_BIAS, "gelu": vlib.EPI_BIAS_GELU,
            "resid": vlib.EPI_BIAS_RESID}[epi]
    a = f16_planes(x, 2)
    wp, acc_scale = f16_weight(w)
    assert a.shape[2] == wp.shape[2]
    y = torch.full((M, N), float("nan"), device=x.device)
    yh = torch.full((2, M, N), -1, dtype=torch.int16, device=x.device) if want_h16 else None
    st = vlib.lib.vitb200_gemm_f16(a.data_ptr(), wp.data_ptr(), acc_scale,
                                   bias.data_ptr() if bias is not None else None,
                                   residual.data_ptr() if residual is not None else None,
                                   y.data_ptr(), N, yh.data_ptr() if yh is not None else None,
                                   M, a.shape[2], N, code, torch.cuda.current_stream().cuda_stream)
    vlib.check(st, "vitb200_gemm_f16")
    return (y, yh) if want_h16 else y


def test_split_error_bound(vlib, cuda):
    """|x - hi - lo * 2^-11| <= 2^-22 |x| + 2^-36 over 14 decades of magnitude;
    the third plane is hi * 2^11 exactly; padding columns are zero."""
    torch.manual_seed(0)
    mag = torch.pow(10.0, torch.empty(64, 1000, device=cuda).uniform_(-10, 3.5))
    x = (torch.randn(64, 1000, device=cuda) * mag).clamp(-30000.0, 30000.0)
    p = f16_planes(x, 2)
    assert p.shape == (2, 64, 1000)
    err = (f16_combine(p) - x.double()).abs()
    bound = x.double().abs() * 2.0 ** -22 + 2.0 ** -36
    assert bool((err <= bound).all()), float((err / bound).max())
    # the weight form: magnitudes below 16, third plane = hi * 2^11 exactly
    w = (x / 2000.0).clamp(-15.9, 15.9)
    pw = f16_planes(w, 3)
    hi = pw[0].view(torch.float16).double()
    assert torch.equal(pw[2].view(torch.float16).double(), hi * F16_LO_SCALE)
    q = f16_planes(torch.randn(5, 13, device=cuda), 2)
    assert q.shape == (2, 5, 16) and int(q[:, :, 13:].abs().max()) == 0


def test_split_range_error(vlib, cuda):
    """A magnitude the split cannot hold is reported, not passed on silently."""
    x = torch.ones(4, 8, device=cuda)
    x[2, 3] = 40000.0
    f16_planes(x, 2)
    assert vlib.device_error(clear=True) == 6
    f16_planes(torch.ones(4, 8, device=cuda) * 30000.0, 2)
    assert vlib.device_error(clear=True) == 0


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("epi", EPILOGUES)
def test_gemm_f16_shapes(vlib, cuda, shape, epi):
    torch.manual_seed(0)
    m, k, n = shape
    x = torch.randn(m, k, device=cuda)
    w = torch.randn(n, k, device=cuda)
    bias = torch.randn(n, device=cuda)
    res = torch.randn(m, n, device=cuda)
    y = run_f16(vlib, x, w, bias, res if epi == "resid" else None, epi)
    check_fp32_parity(y, x, w, bias, res, epi)


@pytest.mark.parametrize("shape", MULTI_TILE)
@pytest.mark.parametrize("epi", ["bias", "resid"])
def test_gemm_f16_multi_tile(vlib, cuda, shape, epi):
    torch.manual_seed(3)
    m, k, n = shape
    x = torch.randn(m, k, device=cuda)
    w = torch.randn(n, k, device=cuda)
    bias = torch.randn(n, device=cuda)
    res = torch.randn(m, n, device=cuda)
    y = run_f16(vlib, x, w, bias, res if epi == "resid" else None, epi)
    check_fp32_parity(y, x, w, bias, res, epi)


@pytest.mark.parametrize("variant", [9, 10, 11, 12, 13, 14, 15])
@pytest.mark.parametrize("shape", [(394, 768, 2304), (200, 3072, 768), (130, 96, 520),
                                   (2100, 300, 1300)])
def test_gemm_f16_variants(vlib, cuda, variant, shape):
    old = vlib.lib.vitb200_set_gemm_variant(variant)
    try:
        torch.manual_seed(1)
        m, k, n = shape
        x = torch.randn(m, k, device=cuda)
        w = torch.randn(n, k, device=cuda) * 0.02
        bias = torch.randn(n, device=cuda) * 0.02
        y = run_f16(vlib, x, w, bias, None, "gelu")
        torch.testing.assert_close(y, expected(x, w, bias, None, "gelu"), atol=1e-5, rtol=1e-5)
    finally:
        vlib.lib.vitb200_set_gemm_variant(old)


@pytest.mark.parametrize("scale", [1e-4, 1.0, 300.0])
def test_f16_matches_tf32x3_accuracy(vlib, cuda, scale):
    """Error against FP64 within 2x of the TF32x3 GEMM's on the same inputs,
    for small, unit and large activations (ViT fc2 shape, K = 3072)."""
    torch.manual_seed(4)
    x = torch.randn(1024, 3072, device=cuda) * scale
    w = torch.randn(768, 3072, device=cuda) * 0.02
    e = x.double() @ w.double().t()
    f16 = (run_f16(vlib, x, w, None, None, "none").double() - e).square().mean().sqrt().item()
    tf32 = (run_gemm(vlib, x, w, None, None, "none").double() - e).square().mean().sqrt().item()
    assert f16 <= 2.0 * tf32, (f16, tf32)


def test_gemm_f16_split_output(vlib, cuda):
    """The epilogue's FP16 split of the result re-sums to the fp32 output."""
    torch.manual_seed(2)
    M, K, N = 1024, 768, 3072
    x = torch.randn(M, K, device=cuda)
    w = torch.randn(N, K, device=cuda) * 0.02
    b = torch.randn(N, device=cuda) * 0.02
    y, yh = run_f16(vlib, x, w, b, None, "gelu", want_h16=True)
    torch.testing.assert_close(y, expected(x, w, b, None, "gelu"), atol=1e-5, rtol=1e-5)
    err = (f16_combine(yh) - y.double()).abs()
    assert bool((err <= y.double().abs() * 2.0 ** -22 + 2.0 ** -36).all())


def test_gemm_f16_bad_arguments(vlib, cuda):
    lib = vlib.lib
    s = torch.cuda.current_stream().cuda_stream
    a = torch.zeros(2, 4, 8, dtype=torch.int16, device=cuda)
    y = torch.empty(4, 4, device=cuda)
    # Kp not a multiple of 8
    assert lib.vitb200_gemm_f16(a.data_ptr(), a.data_ptr(), 1.0, None, None, y.data_ptr(), 4, None,
                                4, 4, 4, vlib.EPI_NONE, s) == vlib.E_INVALID_ARG
    # no output
    assert lib.vitb200_gemm_f16(a.data_ptr(), a.data_ptr(), 1.0, None, None, None, 4, None, 4, 8,
                                4, vlib.EPI_NONE, s) == vlib.E_INVALID_ARG
    # misaligned operand
    assert lib.vitb200_gemm_f16(a.data_ptr() + 2, a.data_ptr(), 1.0, None, None, y.data_ptr(), 4,
                                None, 4, 8, 4, vlib.EPI_NONE, s) == vlib.E_ALIGNMENT


# Batch-1 ViT-B/16 block GEMMs (M = 197 rows: qkv, proj, fc2) and an odd K
# (620: 10 K blocks of 64 for the FP16 kind, 20 of 32 for TF32, the last one
# ragged in both) whose tile grids fill few SMs, so their launches split K;
# fc1 (96 tiles of 64 columns, too many to split) forced onto 128-wide tiles,
# which split.
SPLIT_K_CASES = [((197, 768, 2304), None), ((197, 768, 768), None), ((197, 3072, 768), None),
                 ((130, 620, 200), None), ((197, 768, 3072), "bn128")]


@pytest.mark.parametrize("kind", ["f16", "tf32"])
@pytest.mark.parametrize("shape,forced", SPLIT_K_CASES)
@pytest.mark.parametrize("epi", ["bias", "gelu", "resid"])
def test_split_k(vlib, cuda, kind, shape, forced, epi):
    """Small launches split K over a cluster of CTAs per output tile (partial
    tiles added in split order over distributed shared memory). FP32 parity
    with split-K on and off; on, results repeat bitwise, and (for K >= 768)
    differ in the last bits from the unsplit sums, which shows the split ran."""
    torch.manual_seed(5)
    m, k, n = shape
    variant = {None: 0, "bn128": 10 if kind == "f16" else 1}[forced]
    old_variant = vlib.lib.vitb200_set_gemm_variant(variant)
    try:
        _, ksplit = vlib.gemm_plan(m, k, n, kind == "f16")
        assert ksplit > 1
        x = torch.randn(m, k, device=cuda)
        w = torch.randn(n, k, device=cuda) * 0.05
        bias = torch.randn(n, device=cuda)
        res = torch.randn(m, n, device=cuda) if epi == "resid" else None

        def run():
            if kind == "f16":
                return run_f16(vlib, x, w, bias, res, epi)
            return run_gemm(vlib, x, w, bias, res, epi)

        y1, y2 = run(), run()
        old = vlib.lib.vitb200_set_split_k(0)
        try:
            assert vlib.gemm_plan(m, k, n, kind == "f16")[1] == 1
            y0 = run()
        finally:
            vlib.lib.vitb200_set_split_k(old)
    finally:
        vlib.lib.vitb200_set_gemm_variant(old_variant)
    assert old == 1
    assert torch.equal(y1, y2)
    check_fp32_parity(y1, x, w, bias, res, epi)
    check_fp32_parity(y0, x, w, bias, res, epi)
    if k >= 768:
        assert not torch.equal(y0, y1)
    assert vlib.device_error(clear=True) == 0


def test_large_launches_do_not_split(vlib, cuda):
    """Batch-256 shapes run on CTA pairs, unsplit; so does any M >= 1024."""
    for f16 in (True, False):
        for k, n in ((768, 2304), (768, 768), (768, 3072), (3072, 768)):
            v, d = vlib.gemm_plan(50432, k, n, f16)
            assert d == 1 and v == (15 if f16 else 6)
        assert vlib.gemm_plan(1024, 768, 768, f16)[1] == 1


@pytest.mark.parametrize("kind", ["f16", "tf32"])
@pytest.mark.parametrize("epi", ["bias", "gelu", "resid"])
def test_forced_split_k_every_d(vlib, cuda, kind, epi):
    """Every K split d = 2..8 (vitb200_set_gemm_split), including those for
    which the tile's eight warp slabs are shared out unevenly among the
    cluster's CTAs (d = 3, 5, 6, 7): FP32 parity, bitwise repeatable, and a
    different summation from the unsplit launch (the split ran). K = 64 * 840
    K blocks divide by every d; 4 output tiles keep d CTAs each in one wave."""
    torch.manual_seed(11)
    m, k, n = 197, 64 * 840, 128
    x = torch.randn(m, k, device=cuda)
    w = torch.randn(n, k, device=cuda) * 0.05
    bias = torch.randn(n, device=cuda)
    res = torch.randn(m, n, device=cuda) if epi == "resid" else None

    def run():
        if kind == "f16":
            return run_f16(vlib, x, w, bias, res, epi)
        return run_gemm(vlib, x, w, bias, res, epi)

    old = vlib.lib.vitb200_set_gemm_split(1)
    try:
        assert vlib.gemm_plan(m, k, n, kind == "f16")[1] == 1
        y0 = run()
        for d in range(2, 9):
            vlib.lib.vitb200_set_gemm_split(d)
            assert vlib.gemm_plan(m, k, n, kind == "f16")[1] == d
            y1, y2 = run(), run()
            assert torch.equal(y1, y2), d
            assert not torch.equal(y0, y1), d
            check_fp32_parity(y1, x, w, bias, res, epi)
    finally:
        vlib.lib.vitb200_set_gemm_split(old)
    assert old == 0
    assert vlib.device_error(clear=True) == 0
