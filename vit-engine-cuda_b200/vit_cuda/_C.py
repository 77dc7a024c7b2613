"""The eight per-op entry points of the reference's ``vit_cuda._C`` module
(csrc/bindings/binding.cpp:5-23), re-implemented over libvitb200.so.

Each op keeps the reference wrapper's contract (csrc/ops/*_wrapper.cpp): the
inputs must be CUDA float32 tensors on the current device (RuntimeError
otherwise, as ``vit_checks::contig`` / ``check_same_device`` in
csrc/include/cuda_checks.h:21-50 raise), non-contiguous inputs are made
contiguous, outputs are freshly allocated by PyTorch's caching allocator on the
input's device, and the work is launched asynchronously on the current CUDA
stream. Scratch space (TF32 pairs) comes from the caching allocator too, so the
ops can be captured in a CUDA graph.
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch

from . import _lib
from ._lib import lib


# ---------------------------------------------------------------- checks
def _contig(t: torch.Tensor, name: str) -> torch.Tensor:
    # csrc/include/cuda_checks.h:21-25
    if not isinstance(t, torch.Tensor):
        raise RuntimeError(f"{name} must be a tensor")
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if t.dtype != torch.float32:
        raise RuntimeError(f"{name} must be float32")
    return t.contiguous()


def _same_device(tensors: Sequence[torch.Tensor], op: str) -> None:
    # csrc/include/cuda_checks.h:29-50
    if not tensors:
        raise RuntimeError(f"{op}: expected at least one tensor")
    device = None
    for t in tensors:
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise RuntimeError(f"{op}: all inputs must be CUDA tensors")
        if device is None:
            device = t.get_device()
        if t.get_device() != device:
            raise RuntimeError(f"{op}: all inputs must be on the same CUDA device")
    cur = torch.cuda.current_device()
    if device != cur:
        raise RuntimeError(
            f"{op}: inputs are on device {device} but the current CUDA device is {cur} "
            "(run torch.cuda.set_device, or move tensors)")


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


# ---------------------------------------------------------------- ops
def flash_attn_2(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, scale: float) -> torch.Tensor:
    """softmax(Q K^T * scale) V over 12 heads of 64 (csrc/ops/attention_wrapper.cpp:16-52)."""
    _same_device([Q, K, V], "flash_attn_2")
    Qc, Kc, Vc = _contig(Q, "Q"), _contig(K, "K"), _contig(V, "V")
    if Qc.dim() != 3:
        raise RuntimeError("Expected 3D tensor [B, N, 768]")
    if Kc.dim() != 3:
        raise RuntimeError("K must be [B, N, 768]")
    if Vc.dim() != 3:
        raise RuntimeError("V must be [B, N, 768]")
    if Kc.shape != Qc.shape:
        raise RuntimeError("K shape must match Q shape")
    if Vc.shape != Qc.shape:
        raise RuntimeError("V shape must match Q shape")
    B, N, E = Qc.shape
    if E != 768:
        raise RuntimeError("E dimension must be 768")
    O = torch.empty_like(Qc)
    ws = _workspace(lib.vitb200_attention_workspace_bytes(B, N, 12), Qc.device)
    _lib.check(lib.vitb200_attention(Qc.data_ptr(), Kc.data_ptr(), Vc.data_ptr(), O.data_ptr(),
                                     B, N, 12, E, E, E, E, float(scale), ws.data_ptr(),
                                     ws.numel(), _stream()), "flash_attn_2")
    return O


def patch_embed(img: torch.Tensor, weights: torch.Tensor,
                bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """16x16 patch embedding (csrc/ops/patch_embed_wrapper.cpp:13-51): img [B,C,H,W],
    weights [E, C*256] (or the conv's [E, C, 16, 16]) -> [B, P, E] (+ bias)."""
    if not isinstance(img, torch.Tensor) or not img.is_cuda:
        raise RuntimeError("img must be a CUDA tensor")
    if not isinstance(weights, torch.Tensor) or not weights.is_cuda:
        raise RuntimeError("weights must be a CUDA tensor")
    if img.dtype != torch.float32:
        raise RuntimeError("img must be float32")
    if weights.dtype != torch.float32:
        raise RuntimeError("weights must be float32")
    if img.dim() != 4:
        raise RuntimeError("img must be [B,C,H,W]")
    tensors = [img, weights] + ([bias] if bias is not None else [])
    _same_device(tensors, "patch_embed")
    img_c = _contig(img, "img")
    w_c = _contig(weights, "weights")
    B, C, H, W = img_c.shape
    if H % 16 or W % 16 or H < 16 or W < 16:
        raise RuntimeError("img height and width must be positive multiples of 16")
    E = w_c.shape[0]
    w2 = w_c.reshape(E, -1)
    if w2.shape[1] != C * 256:
        raise RuntimeError(f"weights must be [embed_dim, {C * 256}] (C*16*16)")
    b_c = None
    if bias is not None:
        b_c = _contig(bias, "bias").reshape(-1)
        if b_c.numel() != E:
            raise RuntimeError("bias size mismatch")
    P = (H // 16) * (W // 16)
    out = torch.empty((B, P, E), dtype=torch.float32, device=img_c.device)
    ws = _workspace(lib.vitb200_patch_embed_workspace_bytes(B, C, H, W, E), img_c.device)
    _lib.check(lib.vitb200_patch_embed(img_c.data_ptr(), w2.data_ptr(), _ptr(b_c), out.data_ptr(),
                                       B, C, H, W, E, ws.data_ptr(), ws.numel(), _stream()),
               "patch_embed")
    return out


def pos_encoding(patches: torch.Tensor, cls_token: torch.Tensor,
                 pos_embeddings: torch.Tensor) -> torch.Tensor:
    """[cls + pos[0]; patches + pos[1:]] (csrc/ops/pos_encoding_wrapper.cpp:14-47)."""
    _same_device([patches, cls_token, pos_embeddings], "pos_encoding")
    p_c = _contig(patches, "patches")
    c_c = _contig(cls_token, "cls_token")
    pos_c = _contig(pos_embeddings, "pos_embeddings")
    if p_c.dim() != 3:
        raise RuntimeError("patches must be [B,num_patches,embed_dim]")
    B, P, E = p_c.shape
    if c_c.dim() != 2:
        raise RuntimeError("cls_token must be [B,embed_dim]")
    if c_c.shape[0] != B:
        raise RuntimeError("cls_token batch size mismatch")
    if c_c.shape[1] != E:
        raise RuntimeError("cls_token embed dim mismatch")
    if pos_c.dim() != 2:
        raise RuntimeError("pos_embeddings must be [SEQ_LEN,embed_dim]")
    if pos_c.shape[1] != E:
        raise RuntimeError("pos_embeddings embed dim mismatch")
    if pos_c.shape[0] != P + 1:
        raise RuntimeError(
            "pos_embeddings length must equal num_patches + 1 (including CLS token)")
    out = torch.empty((B, P + 1, E), dtype=torch.float32, device=p_c.device)
    _lib.check(lib.vitb200_pos_encoding(p_c.data_ptr(), c_c.data_ptr(), pos_c.data_ptr(),
                                        out.data_ptr(), B, P, E, _stream()), "pos_encoding")
    return out


def mlp_forward(X: torch.Tensor, W1: torch.Tensor, B1: torch.Tensor, W2: torch.Tensor,
                B2: torch.Tensor) -> list:
    """[O, H] with H = GELU_erf(X W1^T + B1), O = H W2^T + B2
    (csrc/ops/mlp_wrapper.cpp:20-64)."""
    _same_device([X, W1, B1, W2, B2], "mlp_forward")
    X_c, W1_c, B1_c = _contig(X, "X"), _contig(W1, "W1"), _contig(B1, "B1")
    W2_c, B2_c = _contig(W2, "W2"), _contig(B2, "B2")
    if X_c.dim() != 3:
        raise RuntimeError("X must be 3D")
    if W1_c.dim() != 2:
        raise RuntimeError("W1 must be 2D")
    if W2_c.dim() != 2:
        raise RuntimeError("W2 must be 2D")
    B, N, E = X_c.shape
    E4 = W1_c.shape[0]
    if W1_c.shape[1] != E:
        raise RuntimeError("W1 shape mismatch")
    if W2_c.shape[0] != E or W2_c.shape[1] != E4:
        raise RuntimeError("W2 shape mismatch")
    if B1_c.numel() != E4:
        raise RuntimeError("B1 size mismatch")
    if B2_c.numel() != E:
        raise RuntimeError("B2 size mismatch")
    H = torch.empty((B, N, E4), dtype=torch.float32, device=X_c.device)
    O = torch.empty((B, N, E), dtype=torch.float32, device=X_c.device)
    M = B * N
    ws = _workspace(lib.vitb200_mlp_workspace_bytes(M, E, E4), X_c.device)
    _lib.check(lib.vitb200_mlp(X_c.data_ptr(), W1_c.data_ptr(), B1_c.data_ptr(), W2_c.data_ptr(),
                               B2_c.data_ptr(), H.data_ptr(), O.data_ptr(), M, E, E4,
                               ws.data_ptr(), ws.numel(), _stream()), "mlp_forward")
    return [O, H]


def layernorm_forward(X: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor,
                      eps: float) -> torch.Tensor:
    """LayerNorm over the last dim, biased variance
    (csrc/ops/layernorm_wrapper.cpp:16-45)."""
    _same_device([X, gamma, beta], "layernorm_forward")
    Xc, gc, bc = _contig(X, "X"), _contig(gamma, "gamma"), _contig(beta, "beta")
    if Xc.dim() != 3:
        raise RuntimeError("X must be [B, N, E]")
    B, N, E = Xc.shape
    if gc.numel() != E:
        raise RuntimeError("gamma size mismatch")
    if bc.numel() != E:
        raise RuntimeError("beta size mismatch")
    Y = torch.empty_like(Xc)
    _lib.check(lib.vitb200_layernorm(Xc.data_ptr(), gc.data_ptr(), bc.data_ptr(), Y.data_ptr(),
                                     B * N, E, float(eps), _stream()), "layernorm_forward")
    return Y


def classifier_forward(X: torch.Tensor, W: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """logits = X[:, 0, :] W^T + bias (csrc/ops/classifier_wrapper.cpp:15-47)."""
    _same_device([X, W, bias], "classifier_forward")
    Xc, Wc, bc = _contig(X, "X"), _contig(W, "W"), _contig(bias, "bias")
    if Xc.dim() != 3:
        raise RuntimeError("X must be [B, SEQ_LEN, E]")
    if Wc.dim() != 2:
        raise RuntimeError("W must be [num_classes, E]")
    if bc.dim() != 1:
        raise RuntimeError("bias must be [num_classes]")
    B, T, E = Xc.shape
    C = Wc.shape[0]
    if Wc.shape[1] != E:
        raise RuntimeError("W second dim must match embed dim")
    if bc.numel() != C:
        raise RuntimeError("bias size mismatch")
    Y = torch.empty((B, C), dtype=torch.float32, device=Xc.device)
    ws = _workspace(lib.vitb200_classifier_workspace_bytes(B, E, C), Xc.device)
    _lib.check(lib.vitb200_classifier(Xc.data_ptr(), Wc.data_ptr(), bc.data_ptr(), Y.data_ptr(),
                                      B, T, E, C, ws.data_ptr(), ws.numel(), _stream()),
               "classifier_forward")
    return Y


def qkv_proj(X: torch.Tensor, W: torch.Tensor, B: torch.Tensor) -> list:
    """[q, k, v] = split of X W^T + B at E-column boundaries
    (csrc/ops/qkv_wrapper.cpp:17-55); each output is contiguous [B, N, E]."""
    qkv = qkv_proj_packed(X, W, B)
    return [qkv[0], qkv[1], qkv[2]]


def qkv_proj_packed(X: torch.Tensor, W: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
    """qkv_proj's q, k, v as one [3, B, N, N_out/3] tensor (planes contiguous)."""
    _same_device([X, W, B], "qkv_proj")
    Xc, Wc, Bc = _contig(X, "X"), _contig(W, "W"), _contig(B, "B")
    if Xc.dim() != 3:
        raise RuntimeError("X must be [B, N, E]")
    Bb, N, E = Xc.shape
    N_out = Wc.shape[0]
    if Wc.dim() != 2 or Wc.shape[1] != E:
        raise RuntimeError("W second dim must match embed dim")
    if Bc.numel() != N_out:
        raise RuntimeError("bias size mismatch")
    if N_out % 3 != 0:
        raise RuntimeError("N_out must be divisible by 3 (for Q, K, V)")
    M = Bb * N
    Es = N_out // 3
    if Es == E and E % 32 == 0:
        # The GEMM epilogue writes q, k and v as three contiguous planes.
        qkv = torch.empty((3, Bb, N, Es), dtype=torch.float32, device=Xc.device)
        ws = _workspace(lib.vitb200_qkv_workspace_bytes(M, E), Xc.device)
        _lib.check(lib.vitb200_qkv(Xc.data_ptr(), Wc.data_ptr(), Bc.data_ptr(), qkv.data_ptr(),
                                   M, E, ws.data_ptr(), ws.numel(), _stream()), "qkv_proj")
        return qkv
    # General N_out: one GEMM into [M, N_out], then the column thirds made
    # contiguous, as the reference wrapper does.
    Y = gemm_bias(Xc.reshape(M, E), Wc, Bc)
    return Y.view(Bb, N, 3, Es).permute(2, 0, 1, 3).contiguous()


def gemm_bias(X: torch.Tensor, W: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
    """Y = X W^T + B for X [N, K] or [B, N, K] (csrc/ops/gemm_wrapper.cpp:16-59)."""
    _same_device([X, W, B], "gemm_bias")
    Xc, Wc, Bc = _contig(X, "X"), _contig(W, "W"), _contig(B, "B")
    if Xc.dim() not in (2, 3):
        raise RuntimeError("X must be [N, K] or [B, N, K]")
    if Wc.dim() != 2:
        raise RuntimeError("W must be [N_out, K]")
    if Bc.dim() != 1:
        raise RuntimeError("B must be [N_out]")
    if Xc.dim() == 3:
        Bb, N, K = Xc.shape
    else:
        Bb, (N, K) = 1, Xc.shape
    N_out = Wc.shape[0]
    if Wc.shape[1] != K:
        raise RuntimeError("W second dim must match K")
    if Bc.numel() != N_out:
        raise RuntimeError("bias size mismatch")
    M = Bb * N
    Y = torch.empty((Bb, N, N_out), dtype=torch.float32, device=Xc.device)
    ws = _workspace(lib.vitb200_gemm_workspace_bytes(M, K, N_out), Xc.device)
    _lib.check(lib.vitb200_gemm(Xc.data_ptr(), Wc.data_ptr(), Bc.data_ptr(), None, Y.data_ptr(),
                                M, K, N_out, _lib.EPI_BIAS, ws.data_ptr(), ws.numel(), _stream()),
               "gemm_bias")
    return Y if Xc.dim() == 3 else Y.view(M, N_out)


__all__ = ["flash_attn_2", "patch_embed", "pos_encoding", "mlp_forward", "layernorm_forward",
           "classifier_forward", "qkv_proj", "gemm_bias"]
