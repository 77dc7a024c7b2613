"""``torch.library`` registration of the vit_cuda ops, so that ``torch.compile``
traces them without graph breaks (the reference studies exactly those breaks
in tests/torch_compile_test.py:106-114).

Every op of ``vit_cuda._C`` (csrc/bindings/binding.cpp:5-23 of the reference)
becomes ``torch.ops.vit_cuda.<op>`` with a fake (shape-only) implementation for
tracing; the CUDA implementation is the ``_C`` function itself. The public
``vit_cuda.<op>`` names call these registered ops; ``vit_cuda._C.<op>`` stays
the direct call (no dispatcher), like the reference's pybind module.

Two adaptations to the custom-op rules (outputs may not alias each other):
``qkv_proj`` is registered as ``qkv_proj_packed`` returning one ``[3, B, N, E]``
tensor, which the public wrapper unbinds into q, k, v; ``mlp_forward`` returns
its two fresh outputs as a tuple and the wrapper makes it the reference's
``[O, H]`` list. The fused forward of a prepared ``ViTCUDA`` is
``vit_cuda::vit_forward(x, model_id, num_classes)``; the model calls it while
being compiled.
"""
from __future__ import annotations

import weakref
from typing import Optional

import torch

from . import _C


# ---------------------------------------------------------------- ops
@torch.library.custom_op("vit_cuda::flash_attn_2", mutates_args=())
def _flash_attn_2(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor,
                  scale: float) -> torch.Tensor:
    return _C.flash_attn_2(Q, K, V, scale)


@_flash_attn_2.register_fake
def _(Q, K, V, scale):
    return Q.new_empty(Q.shape)


@torch.library.custom_op("vit_cuda::patch_embed", mutates_args=())
def _patch_embed(img: torch.Tensor, weights: torch.Tensor,
                 bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    return _C.patch_embed(img, weights, bias)


@_patch_embed.register_fake
def _(img, weights, bias=None):
    B, _, H, W = img.shape
    return img.new_empty((B, (H // 16) * (W // 16), weights.shape[0]))


@torch.library.custom_op("vit_cuda::pos_encoding", mutates_args=())
def _pos_encoding(patches: torch.Tensor, cls_token: torch.Tensor,
                  pos_embeddings: torch.Tensor) -> torch.Tensor:
    return _C.pos_encoding(patches, cls_token, pos_embeddings)


@_pos_encoding.register_fake
def _(patches, cls_token, pos_embeddings):
    B, P, E = patches.shape
    return patches.new_empty((B, P + 1, E))


@torch.library.custom_op("vit_cuda::mlp_forward", mutates_args=())
def _mlp_forward(X: torch.Tensor, W1: torch.Tensor, B1: torch.Tensor, W2: torch.Tensor,
                 B2: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    O, H = _C.mlp_forward(X, W1, B1, W2, B2)
    return O, H


@_mlp_forward.register_fake
def _(X, W1, B1, W2, B2):
    return X.new_empty(X.shape), X.new_empty((*X.shape[:-1], W1.shape[0]))


@torch.library.custom_op("vit_cuda::layernorm_forward", mutates_args=())
def _layernorm_forward(X: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor,
                       eps: float) -> torch.Tensor:
    return _C.layernorm_forward(X, gamma, beta, eps)


@_layernorm_forward.register_fake
def _(X, gamma, beta, eps):
    return X.new_empty(X.shape)


@torch.library.custom_op("vit_cuda::classifier_forward", mutates_args=())
def _classifier_forward(X: torch.Tensor, W: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    return _C.classifier_forward(X, W, bias)


@_classifier_forward.register_fake
def _(X, W, bias):
    return X.new_empty((X.shape[0], W.shape[0]))


@torch.library.custom_op("vit_cuda::qkv_proj_packed", mutates_args=())
def _qkv_proj_packed(X: torch.Tensor, W: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
    return _C.qkv_proj_packed(X, W, B)


@_qkv_proj_packed.register_fake
def _(X, W, B):
    return X.new_empty((3, *X.shape[:-1], W.shape[0] // 3))


@torch.library.custom_op("vit_cuda::gemm_bias", mutates_args=())
def _gemm_bias(X: torch.Tensor, W: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
    return _C.gemm_bias(X, W, B)


@_gemm_bias.register_fake
def _(X, W, B):
    return X.new_empty((*X.shape[:-1], W.shape[0]))


# ---------------------------------------------------------------- whole model
_MODELS: "weakref.WeakValueDictionary[int, object]" = weakref.WeakValueDictionary()
_NEXT_ID = [0]


def register_model(model) -> int:
    """Makes a ViTCUDA reachable from the registered ``vit_forward`` op."""
    _NEXT_ID[0] += 1
    _MODELS[_NEXT_ID[0]] = model
    return _NEXT_ID[0]


@torch.library.custom_op("vit_cuda::vit_forward", mutates_args=())
def _vit_forward(x: torch.Tensor, model_id: int, num_classes: int) -> torch.Tensor:
    model = _MODELS.get(model_id)
    if model is None:
        raise RuntimeError(f"vit_cuda::vit_forward: no live ViTCUDA with id {model_id}")
    return model._forward_impl(x)


@_vit_forward.register_fake
def _(x, model_id, num_classes):
    return x.new_empty((x.shape[0], num_classes))


# ---------------------------------------------------------------- public API
def flash_attn_2(Q, K, V, scale):
    return torch.ops.vit_cuda.flash_attn_2(Q, K, V, scale)


def patch_embed(img, weights, bias=None):
    return torch.ops.vit_cuda.patch_embed(img, weights, bias)


def pos_encoding(patches, cls_token, pos_embeddings):
    return torch.ops.vit_cuda.pos_encoding(patches, cls_token, pos_embeddings)


def mlp_forward(X, W1, B1, W2, B2):
    O, H = torch.ops.vit_cuda.mlp_forward(X, W1, B1, W2, B2)
    return [O, H]


def layernorm_forward(X, gamma, beta, eps):
    return torch.ops.vit_cuda.layernorm_forward(X, gamma, beta, eps)


def classifier_forward(X, W, bias):
    return torch.ops.vit_cuda.classifier_forward(X, W, bias)


def qkv_proj(X, W, B):
    return list(torch.ops.vit_cuda.qkv_proj_packed(X, W, B).unbind(0))


def gemm_bias(X, W, B):
    return torch.ops.vit_cuda.gemm_bias(X, W, B)
