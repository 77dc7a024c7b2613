"""CPU oracle for the ViT-B/16 forward — TEST INFRASTRUCTURE ONLY.

This module is the parity checker. Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference arm may import it; the product path
(vit_cuda, libvitb200.so) never does.

It restates, in plain PyTorch CPU arithmetic (float64 by default, float32 on
request), the algorithm the reference engine AhmadSaeedZaidi/ViT-Engine-CUDA
runs and checks itself against: timm's `vit_base_patch16_224` eval forward in
FP32 (reference vit_cuda/model.py:8-13, tests/test_end_to_end.py:22-45). timm
itself is a third-party dependency that is absent here (unpinned in the
reference: requirements.txt:3, pyproject.toml:14), so the steps below follow the
reference's own restatement of timm's block order in
scripts/layerwise_compare.py:141-257 and the per-op expected values its tests
construct. Each function cites the reference file:line it follows.

Pinning (see tests/test_oracle_*.py):
  * per-op: against the formulas of the reference's tests (loop-built patch
    vectors, loop-built pos encoding, F.layer_norm, manual attention, ...),
    committed as golden vectors in tests/golden/ops_golden.npz;
  * end to end: against HuggingFace transformers' ViTForImageClassification —
    an independent implementation of the same published ViT-B/16 — run in
    float64 on the same seeded weights, committed as
    tests/golden/vit_e2e_golden.npz (generator: tests/golden/make_golden.py);
  * against the reference's own CUDA kernels compiled from its sources
    (oracle/Makefile -> oracle/_ref/libvitref.so), run on a B200 by
    tests/test_ref_kernels_gpu.py.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

EMBED = 768
HEADS = 12
HEAD_DIM = 64
PATCH = 16


def _t(x, dtype):
    return x.detach().to(device="cpu", dtype=dtype)


# ----------------------------------------------------------------- ops
def im2col(img: torch.Tensor) -> torch.Tensor:
    """[B, C, H, W] -> [B, P, C*256]; patches row-major over the grid, each
    vector in (c, py, px) order (reference tests/test_patch_embed.py:48-56,
    csrc/kernels/patch_embed.cu:29-44, scripts/patch_compare.py:47-53)."""
    B, C, H, W = img.shape
    gh, gw = H // PATCH, W // PATCH
    x = img.reshape(B, C, gh, PATCH, gw, PATCH)
    x = x.permute(0, 2, 4, 1, 3, 5)  # B, gy, gx, c, py, px
    return x.reshape(B, gh * gw, C * PATCH * PATCH)


def patch_embed(img, weight, bias=None, dtype=torch.float64):
    """im2col . W^T (+ bias) (reference csrc/kernels/patch_embed.cu:23-98 plus
    the bias add of csrc/ops/patch_embed_wrapper.cpp:46-48)."""
    img, weight = _t(img, dtype), _t(weight, dtype)
    w2 = weight.reshape(weight.shape[0], -1)
    out = im2col(img) @ w2.T
    if bias is not None:
        out = out + _t(bias, dtype)
    return out


def pos_encoding(patches, cls, pos, dtype=torch.float64):
    """out[b,0] = cls[b] + pos[0]; out[b,i] = patches[b,i-1] + pos[i]
    (reference csrc/kernels/pos_encoding.cu:8-28, tests/test_pos_encoding.py:43-47)."""
    patches, cls, pos = _t(patches, dtype), _t(cls, dtype), _t(pos, dtype)
    B = patches.shape[0]
    cls_b = cls.reshape(-1, patches.shape[-1]).expand(B, -1)
    x = torch.cat([cls_b.unsqueeze(1), patches], dim=1)
    return x + pos.reshape(1, -1, patches.shape[-1])


def layernorm(x, gamma, beta, eps, dtype=torch.float64):
    """Mean, biased variance of (x - mean), (x - mean) / sqrt(var + eps) * g + b
    (reference csrc/kernels/layernorm.cu:44-64)."""
    x, gamma, beta = _t(x, dtype), _t(gamma, dtype), _t(beta, dtype)
    mean = x.mean(dim=-1, keepdim=True)
    d = x - mean
    var = (d * d).mean(dim=-1, keepdim=True)
    return d / torch.sqrt(var + eps) * gamma + beta


def linear(x, w, b=None, dtype=torch.float64):
    """x W^T (+ b), W in PyTorch [out, in] layout (reference csrc/kernels/gemm.cu:12-96)."""
    x, w = _t(x, dtype), _t(w, dtype)
    y = x @ w.T
    if b is not None:
        y = y + _t(b, dtype)
    return y


def gelu_erf(x):
    """0.5 x (1 + erf(x / sqrt 2)) (reference csrc/kernels/gemm.cu:7-10)."""
    return 0.5 * x * (1.0 + torch.erf(x / math.sqrt(2.0)))


def qkv_proj(x, w, b, dtype=torch.float64):
    """Y = x W^T + b split into q, k, v at E-column boundaries
    (reference csrc/ops/qkv_wrapper.cpp:49-52, tests/test_qkv.py:41-44)."""
    y = linear(x, w, b, dtype)
    E = y.shape[-1] // 3
    return y[..., :E], y[..., E:2 * E], y[..., 2 * E:]


def attention(q, k, v, scale, heads=HEADS, dtype=torch.float64):
    """softmax(Q K^T * scale) V per head; q/k/v [B, N, heads*64], head h in
    columns h*64.. (reference tests/test_flash_attn.py:10-24,
    csrc/kernels/attention.cu:50,84)."""
    q, k, v = _t(q, dtype), _t(k, dtype), _t(v, dtype)
    B, N, E = q.shape
    d = E // heads
    qh = q.reshape(B, N, heads, d).transpose(1, 2)
    kh = k.reshape(B, N, heads, d).transpose(1, 2)
    vh = v.reshape(B, N, heads, d).transpose(1, 2)
    s = (qh @ kh.transpose(-2, -1)) * scale
    s = s - s.amax(dim=-1, keepdim=True)
    p = torch.exp(s)
    p = p / p.sum(dim=-1, keepdim=True)
    o = p @ vh
    return o.transpose(1, 2).reshape(B, N, E)


def mlp(x, w1, b1, w2, b2, dtype=torch.float64):
    """(O, H): H = GELU_erf(x W1^T + b1), O = H W2^T + b2
    (reference csrc/kernels/mlp.cu:5-20; the op returns [O, H],
    csrc/ops/mlp_wrapper.cpp:63)."""
    h = gelu_erf(linear(x, w1, b1, dtype))
    return linear(h, w2, b2, dtype), h


def classifier(x, w, b, dtype=torch.float64):
    """logits = x[:, 0, :] W^T + b (reference csrc/kernels/classifier.cu:40-66,
    tests/test_classifier.py:42-43)."""
    x = _t(x, dtype)
    return linear(x[:, 0, :], w, b, dtype)


# --------------------------------------------------------------- model
def block_forward(x, state, idx, eps=1e-6, scale=0.125, dtype=torch.float64):
    """Pre-LN block, reference vit_cuda/model.py:39-60 and
    scripts/layerwise_compare.py:180-250:
    x = x + proj(attn(norm1 x)); x = x + fc2(gelu(fc1(norm2 x)))."""
    p = f"blocks.{idx}."
    x = _t(x, dtype)
    h = layernorm(x, state[p + "norm1.weight"], state[p + "norm1.bias"], eps, dtype)
    q, k, v = qkv_proj(h, state[p + "attn.qkv.weight"], state[p + "attn.qkv.bias"], dtype)
    a = attention(q, k, v, scale, HEADS, dtype)
    x = x + linear(a, state[p + "attn.proj.weight"], state[p + "attn.proj.bias"], dtype)
    h = layernorm(x, state[p + "norm2.weight"], state[p + "norm2.bias"], eps, dtype)
    o, _ = mlp(h, state[p + "mlp.fc1.weight"], state[p + "mlp.fc1.bias"],
               state[p + "mlp.fc2.weight"], state[p + "mlp.fc2.bias"], dtype)
    return x + o


def embed(img, state, dtype=torch.float64):
    """Patch embedding + CLS + positions (reference vit_cuda/model.py:103-118)."""
    patches = patch_embed(img, state["patch_embed.proj.weight"], state["patch_embed.proj.bias"],
                          dtype)
    B = patches.shape[0]
    cls = _t(state["cls_token"], dtype).reshape(1, EMBED).expand(B, -1)
    pos = _t(state["pos_embed"], dtype).reshape(-1, EMBED)
    return pos_encoding(patches, cls, pos, dtype)


def num_blocks(state) -> int:
    n = 0
    while f"blocks.{n}.norm1.weight" in state:
        n += 1
    return n


def vit_forward(img, state, eps=1e-6, scale=0.125, dtype=torch.float64,
                return_intermediates: bool = False):
    """Full forward (reference vit_cuda/model.py:101-126): embed, blocks, final
    LayerNorm, head on the CLS token. With return_intermediates it also returns
    {"embed": x0, "blocks": [x1..x12], "features": cls after the final norm}."""
    x = embed(img, state, dtype)
    inter = {"embed": x, "blocks": []}
    for i in range(num_blocks(state)):
        x = block_forward(x, state, i, eps, scale, dtype)
        inter["blocks"].append(x)
    xn = layernorm(x, state["norm.weight"], state["norm.bias"], eps, dtype)
    inter["features"] = xn[:, 0, :]
    logits = classifier(xn, state["head.weight"], state["head.bias"], dtype)
    return (logits, inter) if return_intermediates else logits


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    """||a - b|| / ||b|| in float64 (per-block metric of the parity bar)."""
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-300))
