"""FP16-split tensor-core attention (vitb200_attention_f16) against the float64
oracle, with the reference's attention bar (tests/test_flash_attn.py of the
reference project: softmax(Q K^T * scale) V per head, B=2, N=197, 768 = 12 x 64;
1e-4 here), at the sequence lengths and batch sizes the model runs (T = 197,
577, ragged tails, more work items than SMs), with the k / v scales the model
derives from its weights.
"""
import math

import pytest
import torch

from oracle import vit_oracle as orc

pytestmark = pytest.mark.gpu


def pow2_scale(x, limit=8.0):
    """A power-of-two scale as the model would pass (any power of two is exact)."""
    m = float(x.abs().max())
    return 2.0 ** math.floor(math.log2(limit / m)) if m > 0 else 1.0


def run_attn_f16(vlib, q, k, v, scale, k_scale=None, v_scale=None):
    B, T, E = q.shape
    heads = E // 64
    k_scale = k_scale or pow2_scale(k)
    v_scale = v_scale or pow2_scale(v)
    o = torch.full((B, T, E), float("nan"), device=q.device)
    ws = torch.empty(max(1, vlib.lib.vitb200_attention_f16_workspace_bytes(B, T, heads)),
                     dtype=torch.uint8, device=q.device)
    vlib.check(vlib.lib.vitb200_attention_f16(q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                              o.data_ptr(), B, T, heads, E, E, E, E, scale,
                                              k_scale, v_scale, ws.data_ptr(), ws.numel(),
                                              torch.cuda.current_stream().cuda_stream),
               "vitb200_attention_f16")
    return o


# Up to 6 images (head pairs filling under half the SMs) run the one-query-tile
# kernel, larger batches the two-tile kernel: (7, 65), (13, 197), (7, 577) and
# (64, 197) take the latter, ragged tiles included.
@pytest.mark.parametrize("B,T", [(2, 197), (1, 577), (3, 50), (1, 1), (2, 64), (2, 65),
                                 (1, 128), (1, 129), (1, 257), (7, 65), (13, 197), (7, 577),
                                 (64, 197)])
def test_attention_f16_matches_oracle(vlib, cuda, B, T):
    torch.manual_seed(B * 1000 + T)
    q, k, v = (torch.randn(B, T, 768) for _ in range(3))
    out = run_attn_f16(vlib, q.to(cuda), k.to(cuda), v.to(cuda), 0.125)
    torch.testing.assert_close(out.double().cpu(), orc.attention(q, k, v, 0.125), atol=1e-4,
                               rtol=1e-5)


def test_attention_f16_large_logits(vlib, cuda):
    """Large score ranges exercise the online-softmax rescaling."""
    torch.manual_seed(2)
    q, k, v = (torch.randn(2, 197, 768) * 4 for _ in range(3))
    out = run_attn_f16(vlib, q.to(cuda), k.to(cuda), v.to(cuda), 0.125)
    torch.testing.assert_close(out.double().cpu(), orc.attention(q, k, v, 0.125), atol=2e-4,
                               rtol=1e-5)


@pytest.mark.parametrize("mag", [1e-3, 30.0])
def test_attention_f16_magnitudes(vlib, cuda, mag):
    """Small and large activations: the scales keep the split's relative
    accuracy (error measured relative to the output's magnitude)."""
    torch.manual_seed(3)
    q = torch.randn(2, 197, 768) * (0.05 / mag if mag > 1 else 1.0)
    k = torch.randn(2, 197, 768) * mag
    v = torch.randn(2, 197, 768) * mag
    out = run_attn_f16(vlib, q.to(cuda), k.to(cuda), v.to(cuda), 0.125)
    ref = orc.attention(q, k, v, 0.125)
    err = (out.double().cpu() - ref).abs().max().item()
    assert err <= 1e-4 * mag, (err, mag)


def test_attention_f16_matches_tf32_path(vlib, cuda):
    """Both tensor-core attentions agree closely with each other and the oracle."""
    import vit_cuda
    torch.manual_seed(5)
    q, k, v = (torch.randn(4, 197, 768, device=cuda) for _ in range(3))
    a = run_attn_f16(vlib, q, k, v, 0.125)
    b = vit_cuda.flash_attn_2(q, k, v, 0.125)
    ref = orc.attention(q.cpu(), k.cpu(), v.cpu(), 0.125)
    ea = (a.double().cpu() - ref).abs().max().item()
    eb = (b.double().cpu() - ref).abs().max().item()
    assert ea <= 1e-4 and eb <= 1e-4 and ea <= 2 * eb + 1e-6, (ea, eb)


def test_attention_f16_range_error(vlib, cuda):
    """A k scale that takes |k * k_scale| past the split's range is reported
    (device error)."""
    q, k, v = (torch.randn(1, 8, 768, device=cuda) for _ in range(3))
    run_attn_f16(vlib, q, k, v, 0.125, k_scale=2.0 ** 16, v_scale=1.0)
    assert vlib.device_error(clear=True) == 6
