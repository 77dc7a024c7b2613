"""Guard bands, standing in for compute-sanitizer (closed on this pool): every
output and workspace an entry point writes sits inside a larger buffer whose
leading and trailing bands hold a sentinel, and after the call both bands must
be untouched. Catches writes past the end (or before the start) of a buffer by
the GEMM epilogues (ragged M / N / K tails, split-K clusters, FP16-split
output planes), the attention (ragged T) and the whole forward's workspace
carving, at sizes where every tail is partial."""
import ctypes

import pytest
import torch

from vit_cuda import ViTCUDA
from vit_cuda.split import f16_planes, f16_weight
from vit_cuda.weights import synthetic_images, synthetic_state_dict

pytestmark = pytest.mark.gpu

G = 4096  # guard elements on each side


def guarded(n, device, dtype=torch.float32, fill=1234.5):
    buf = torch.full((n + 2 * G,), fill, dtype=dtype, device=device)
    return buf, buf[G:G + n]


def bands_intact(buf, fill=1234.5):
    return bool((buf[:G] == fill).all()) and bool((buf[-G:] == fill).all())


def stream():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("shape", [(197, 768, 768), (197, 3072, 768), (130, 620, 200),
                                   (35, 65, 37), (2100, 300, 1300), (1, 768, 1000)])
@pytest.mark.parametrize("epi", ["bias", "gelu", "resid"])
def test_gemm_tf32_bands(vlib, cuda, shape, epi):
    torch.manual_seed(0)
    M, K, N = shape
    code = {"bias": vlib.EPI_BIAS, "gelu": vlib.EPI_BIAS_GELU, "resid": vlib.EPI_BIAS_RESID}[epi]
    x = torch.randn(M, K, device=cuda)
    w = torch.randn(N, K, device=cuda) * 0.05
    b = torch.randn(N, device=cuda)
    res = torch.randn(M, N, device=cuda) if epi == "resid" else None
    ybuf, y = guarded(M * N, cuda)
    nws = max(1, vlib.lib.vitb200_gemm_workspace_bytes(M, K, N))
    wbuf, ws = guarded(nws, cuda, torch.uint8, 165)
    vlib.check(vlib.lib.vitb200_gemm(x.data_ptr(), w.data_ptr(), b.data_ptr(),
                                     res.data_ptr() if res is not None else None, y.data_ptr(),
                                     M, K, N, code, ws.data_ptr(), nws, stream()), "gemm")
    torch.cuda.synchronize()
    assert bands_intact(ybuf) and bands_intact(wbuf, 165)
    assert not torch.isnan(y).any() and not (y == 1234.5).any()


@pytest.mark.parametrize("shape", [(197, 768, 2304), (197, 3072, 768), (130, 620, 200),
                                   (2100, 300, 1300)])
@pytest.mark.parametrize("h16", [False, True])
def test_gemm_f16_bands(vlib, cuda, shape, h16):
    torch.manual_seed(1)
    M, K, N = shape
    x = torch.randn(M, K, device=cuda)
    w = torch.randn(N, K, device=cuda) * 0.05
    b = torch.randn(N, device=cuda)
    a = f16_planes(x, 2)
    wp, acc = f16_weight(w)
    ybuf, y = guarded(M * N, cuda)
    hbuf, h = guarded(2 * M * N, cuda, torch.int16, 12345) if h16 else (None, None)
    vlib.check(vlib.lib.vitb200_gemm_f16(a.data_ptr(), wp.data_ptr(), acc, b.data_ptr(), None,
                                         y.data_ptr(), N, h.data_ptr() if h16 else None, M,
                                         a.shape[2], N,
                                         vlib.EPI_BIAS_GELU if h16 else vlib.EPI_BIAS, stream()),
               "gemm_f16")
    torch.cuda.synchronize()
    assert bands_intact(ybuf)
    if h16:
        assert bands_intact(hbuf, 12345)


@pytest.mark.parametrize("B,T", [(2, 197), (1, 577), (3, 50), (1, 1), (2, 65), (13, 197),
                                 (7, 577)])
def test_attention_f16_bands(vlib, cuda, B, T):
    torch.manual_seed(2)
    E = 768
    q, k, v = (torch.randn(B, T, E, device=cuda) for _ in range(3))
    obuf, o = guarded(B * T * E, cuda)
    nws = max(1, vlib.lib.vitb200_attention_f16_workspace_bytes(B, T, 12))
    wbuf, ws = guarded(nws, cuda, torch.uint8, 165)
    vlib.check(vlib.lib.vitb200_attention_f16(q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                              o.data_ptr(), B, T, 12, E, E, E, E, 0.125, 1.0,
                                              1.0, ws.data_ptr(), nws, stream()), "attention")
    torch.cuda.synchronize()
    assert bands_intact(obuf) and bands_intact(wbuf, 165)


@pytest.mark.parametrize("batch", [1, 3])
def test_forward_bands(vlib, cuda, batch):
    """The whole forward through the C ABI with a guarded workspace (carved into
    its activations and operand splits) and guarded logits; batch 1 runs its
    block GEMMs as split-K clusters."""
    state = synthetic_state_dict(seed=3, img_size=224, depth=2)
    model = ViTCUDA(state_dict={k: v.to(cuda) for k, v in state.items()}).to(cuda).eval()
    model.prepare()
    x = synthetic_images(batch, 224, seed=3).to(cuda)
    params = model.params
    nws = int(vlib.lib.vitb200_vit_workspace_bytes(ctypes.byref(params), batch))
    wbuf, ws = guarded(nws, cuda, torch.uint8, 165)
    lbuf, logits = guarded(batch * 1000, cuda)
    vlib.check(vlib.lib.vitb200_vit_forward(ctypes.byref(params), x.data_ptr(), logits.data_ptr(),
                                            batch, ws.data_ptr(), nws, stream()), "forward")
    torch.cuda.synchronize()
    assert bands_intact(wbuf, 165) and bands_intact(lbuf)
    with torch.no_grad():
        ref = model(x)
    torch.testing.assert_close(logits.view(batch, 1000), ref, atol=0, rtol=0)
