"""Operand preparation for the library's two GEMM operand kinds.

TF32 pairs (hi, lo) feed the TF32x3 GEMM; FP16 splits feed the three-product
FP16 GEMM (Ootomo & Yokota, IJHPCA 2022): x ~= hi + lo * 2^-11 with
hi = fp16(x), lo = fp16((x - hi) * 2^11), and weights carry a third plane
hi * 2^11 so that all three tensor-core products share one scale. A weight is
first multiplied by a power of two s that brings its largest magnitude into
[8, 16): the hi * 2^11 plane then stays finite and small weights keep their
low bits; the GEMM multiplies its accumulator by 2^-11 / s (exact).

Activation splits use no scale: every activation the ViT path splits is
bounded in advance by the weights (a LayerNorm output by sqrt(E - 1) * |gamma|
+ |beta|, linear maps of it by the weights' row sums), and `f16_safe_bound`
is the limit such a bound must stay under.
"""
from __future__ import annotations

import math

import torch

from . import _lib

F16_LO_SCALE = 2048.0
# Magnitudes a split may take: |hi| and |hi * 2^11| finite in fp16 (max 65504).
F16_SAFE_BOUND = 32768.0


def f16_weight_scale(w: torch.Tensor) -> float:
    """Power of two s with max|w| * s in [8, 16) (1.0 for an all-zero w)."""
    m = float(w.detach().abs().max().item()) if w.numel() else 0.0
    if not math.isfinite(m):
        raise ValueError("weight holds a non-finite value")
    if m == 0.0:
        return 1.0
    return 2.0 ** (3 - math.floor(math.log2(m)))


def f16_planes(x: torch.Tensor, nplanes: int, scale: float = 1.0, ldp: int | None = None,
               stream=None) -> torch.Tensor:
    """FP16 split of a 2-D fp32 CUDA tensor as a [nplanes][rows][ldp] int16
    tensor (ldp = cols rounded up to 8, zero padded)."""
    if x.dim() != 2 or x.dtype != torch.float32 or not x.is_cuda:
        raise ValueError("f16_planes: expected a 2-D float32 CUDA tensor")
    x = x.contiguous()
    rows, cols = x.shape
    ldp = ldp or (cols + 7) // 8 * 8
    out = torch.empty(nplanes, rows, ldp, dtype=torch.int16, device=x.device)
    s = stream if stream is not None else torch.cuda.current_stream(x.device).cuda_stream
    _lib.check(_lib.lib.vitb200_split_f16(x.data_ptr(), rows, cols, cols, scale, out.data_ptr(),
                                          ldp, nplanes, s), "vitb200_split_f16")
    return out


def f16_weight(w: torch.Tensor) -> tuple[torch.Tensor, float]:
    """W[N][K] -> (planes [3][N][Kp], acc_scale = 2^-11 / s)."""
    s = f16_weight_scale(w)
    return f16_planes(w, 3, s), 1.0 / (F16_LO_SCALE * s)


def f16_combine(planes: torch.Tensor) -> torch.Tensor:
    """hi + lo * 2^-11 of a split, in fp64 (for tests)."""
    h = planes[0].view(torch.float16).double()
    lo = planes[1].view(torch.float16).double()
    return h + lo / F16_LO_SCALE


def layernorm_bound(gamma: torch.Tensor, beta: torch.Tensor) -> float:
    """Largest magnitude a LayerNorm over E = len(gamma) features can output:
    a normalised entry is at most sqrt(E - 1) in magnitude (biased variance),
    so |y| <= sqrt(E - 1) * max|gamma| + max|beta|."""
    e = gamma.numel()
    return math.sqrt(max(e - 1, 0)) * float(gamma.abs().max()) + float(beta.abs().max())


def linear_bound(in_bound: float, w: torch.Tensor, b: torch.Tensor | None) -> float:
    """Bound on |x W^T + b| for inputs bounded by in_bound: in_bound times the
    largest absolute row sum of W, plus max|b|."""
    rows = w.reshape(w.shape[0], -1).double().abs().sum(dim=1)
    out = in_bound * float(rows.max()) if rows.numel() else 0.0
    return out + (float(b.abs().max()) if b is not None and b.numel() else 0.0)


def block_input_bounds(blk, embed_dim: int) -> dict[str, float]:
    """Magnitude bounds of one encoder block's split operands: qkv and fc1
    take LayerNorm outputs; q, k, v (the attention's operands) are linear maps
    of LN1's output; proj takes attention outputs, convex combinations of V
    rows; fc2 takes GELU(fc1 output), at most max(|h|, 0.17)."""
    ln1 = layernorm_bound(blk.norm1_gamma, blk.norm1_beta)
    ln2 = layernorm_bound(blk.norm2_gamma, blk.norm2_beta)
    E = embed_dim
    q = linear_bound(ln1, blk.qkv_weight[:E], blk.qkv_bias[:E])
    k = linear_bound(ln1, blk.qkv_weight[E:2 * E], blk.qkv_bias[E:2 * E])
    v = linear_bound(ln1, blk.qkv_weight[2 * E:3 * E], blk.qkv_bias[2 * E:3 * E])
    h = linear_bound(ln2, blk.fc1_weight, blk.fc1_bias)
    return {"qkv": ln1, "proj": v, "fc1": ln2, "fc2": max(h, 0.2), "q": q, "k": k, "v": v}


def f16_weight_ok(w: torch.Tensor) -> bool:
    """A weight the FP16 split can carry: finite, and not so small that its
    power-of-two scale leaves the fp32 range."""
    m = float(w.detach().abs().max().item()) if w.numel() else 0.0
    return math.isfinite(m) and (m == 0.0 or m >= 2.0 ** -60)
