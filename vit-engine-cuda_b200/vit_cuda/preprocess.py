"""GPU image preprocessing: the step before the forward in the reference
(vit_cuda/model.py:180-188 and scripts/eval_imagenette.py:210-215: torchvision
``Resize(256) -> CenterCrop(224) -> ToTensor -> Normalize(ImageNet mean/std)``),
as one kernel over a batch of decoded 8-bit RGB images (``vitb200_preprocess``).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

IMAGENET_MEAN = (0.485, 0.456, 0.406)
IMAGENET_STD = (0.229, 0.224, 0.225)


def preprocess(images: torch.Tensor, resize: int = 256, crop: int = 224,
               mean=IMAGENET_MEAN, std=IMAGENET_STD) -> torch.Tensor:
    """uint8 RGB images ``[B, H, W, 3]`` (or one ``[H, W, 3]``) on a CUDA device
    -> float32 ``[B, 3, crop, crop]``: the shorter side resized to ``resize``
    (antialiased bilinear), the centred ``crop`` window, ``(x/255 - mean)/std``."""
    if not isinstance(images, torch.Tensor) or not images.is_cuda:
        raise RuntimeError("preprocess: images must be a CUDA tensor")
    if images.dtype != torch.uint8:
        raise RuntimeError("preprocess: images must be uint8")
    if images.dim() == 3:
        images = images.unsqueeze(0)
    if images.dim() != 4 or images.shape[3] != 3:
        raise RuntimeError("preprocess: images must be [B, H, W, 3] (HWC RGB)")
    images = images.contiguous()
    B, H, W, _ = images.shape
    out = torch.empty(B, 3, crop, crop, dtype=torch.float32, device=images.device)
    m = (ctypes.c_float * 3)(*mean)
    s = (ctypes.c_float * 3)(*std)
    with torch.cuda.device(images.device):
        st = _lib.lib.vitb200_preprocess(images.data_ptr(), B, H, W, H * W * 3, resize, crop, m, s,
                                         out.data_ptr(),
                                         torch.cuda.current_stream(images.device).cuda_stream)
    if st == _lib.E_UNSUPPORTED:
        raise RuntimeError(f"preprocess: the image resized to {resize} is smaller than the "
                           f"{crop} crop")
    _lib.check(st, "vitb200_preprocess")
    return out
