"""vit_cuda — B200-native (sm_100a) ViT-B/16 inference with the reference
project's drop-in surface: the eight ops of ``vit_cuda._C`` re-exported as
``vit_cuda.<op>`` (the reference tests call them that way, e.g.
tests/test_qkv.py:37) and ``vit_cuda.model.ViTCUDA``. The ``vit_cuda.<op>``
names go through ``torch.ops.vit_cuda.<op>`` (registered custom ops that
``torch.compile`` traces); ``vit_cuda._C.<op>`` calls the library directly.
"""
from . import _C
from .library import (classifier_forward, flash_attn_2, gemm_bias, layernorm_forward,
                      mlp_forward, patch_embed, pos_encoding, qkv_proj)
from ._lib import VitB200Error, device_error, set_split_k
from .model import ViTBlockCUDA, ViTCUDA
from .pipeline import StreamedInference
from .preprocess import preprocess

__all__ = [
    "flash_attn_2",
    "patch_embed",
    "pos_encoding",
    "mlp_forward",
    "layernorm_forward",
    "classifier_forward",
    "qkv_proj",
    "gemm_bias",
    "ViTCUDA",
    "ViTBlockCUDA",
    "VitB200Error",
    "device_error",
    "set_split_k",
    "preprocess",
    "StreamedInference",
]
