"""Parity at the sizes of BASELINE.json's isolated configurations, against
float64 references computed on the GPU with torch (too large for the CPU
oracle in seconds):

* cfg3 — attention B=256, H=12, N=197, d=64, N(0,1) Q/K/V, scale 1/8, vs float64
  softmax attention (the reference's tests/test_flash_attn.py:10-24 math);
* cfg4 — the ViT-B/16 GEMM set at M = 512*197 = 100,864 rows, N(0,1)
  activations and trunc_normal(0.02) weights: QKV 768->2304, proj 768->768,
  fc1 768->3072 (+bias +erf-GELU), fc2 3072->768 (+bias +residual), and the
  patch-embedding GEMM 768->768, each through the FP16-split path the model uses
  and the TF32x3 path of the per-op API; error no larger than cuBLAS FP32's
  (TF32 off) on the same data, or the reference GEMM tests' 1e-4.
"""
import math

import pytest
import torch
import torch.nn.functional as F

from test_attention_f16_gpu import run_attn_f16
from test_gemm_f16_gpu import run_f16
from test_gemm_gpu import run_gemm

pytestmark = pytest.mark.gpu

M_CFG4 = 512 * 197


def _trunc_normal(n, k, device, gen):
    w = torch.empty(n, k, device=device)
    torch.nn.init.trunc_normal_(w, std=0.02, a=-0.04, b=0.04, generator=gen)
    return w


@pytest.mark.parametrize("name,N,K,epi", [("qkv", 2304, 768, "bias"), ("proj", 768, 768, "bias"),
                                          ("fc1", 3072, 768, "gelu"), ("fc2", 768, 3072, "resid"),
                                          ("patch", 768, 768, "bias")])
def test_cfg4_gemm_set(vlib, cuda, name, N, K, epi):
    gen = torch.Generator(device=cuda).manual_seed(sum(map(ord, name)))
    x = torch.randn(M_CFG4, K, device=cuda, generator=gen)
    w = _trunc_normal(N, K, cuda, gen)
    b = torch.randn(N, device=cuda, generator=gen) * 0.02
    res = torch.randn(M_CFG4, N, device=cuda, generator=gen) if epi == "resid" else None
    e = x.double() @ w.double().t() + b.double()
    if epi == "gelu":
        e = F.gelu(e, approximate="none")
    if epi == "resid":
        e = res.double() + e
    ref32 = x @ w.t() + b
    if epi == "gelu":
        ref32 = F.gelu(ref32, approximate="none")
    if epi == "resid":
        ref32 = res + ref32
    cublas = (ref32.double() - e).abs().max().item()
    bound = max(1.5 * cublas, 1e-4)
    for path, y in (("f16", run_f16(vlib, x, w, b, res, epi)),
                    ("tf32", run_gemm(vlib, x, w, b, res, epi))):
        err = (y.double() - e).abs().max().item()
        assert err <= bound, (name, path, err, cublas)
        del y


def test_cfg3_attention(vlib, cuda):
    gen = torch.Generator(device=cuda).manual_seed(3)
    B, T = 256, 197
    q, k, v = (torch.randn(B, T, 768, device=cuda, generator=gen) for _ in range(3))

    def ref64(q, k, v):
        qh, kh, vh = (t.double().view(B, T, 12, 64).transpose(1, 2) for t in (q, k, v))
        p = torch.softmax(qh @ kh.transpose(-1, -2) * 0.125, dim=-1)
        return (p @ vh).transpose(1, 2).reshape(B, T, 768)

    e = ref64(q, k, v)
    import vit_cuda
    for path, out in (("f16", run_attn_f16(vlib, q, k, v, 0.125)),
                      ("tf32", vit_cuda.flash_attn_2(q, k, v, 0.125))):
        err = (out.double() - e).abs().max().item()
        assert err <= 1e-4, (path, err)
        del out
    # and the torch fp32 SDPA (TF32 off) the configuration names as its comparison
    sdpa = F.scaled_dot_product_attention(q.view(B, T, 12, 64).transpose(1, 2),
                                          k.view(B, T, 12, 64).transpose(1, 2),
                                          v.view(B, T, 12, 64).transpose(1, 2), scale=0.125)
    sdpa = sdpa.transpose(1, 2).reshape(B, T, 768)
    assert (sdpa.double() - e).abs().max().item() <= 1e-4
    assert math.isfinite(e.abs().max().item())
