"""GPU image preprocessing (vitb200_preprocess / vit_cuda.preprocess) against
(1) torchvision's float tensor path — antialiased bilinear Resize, CenterCrop,
Normalize — which is the same resampling arithmetic in fp32, and (2) the
reference's own PIL pipeline (vit_cuda/model.py:180-188 of the reference
project), committed as tests/golden/preprocess_golden.npz; PIL rounds to 8 bits
between its two resampling passes, so that comparison allows one 8-bit step
after normalisation."""
import os
import sys

import numpy as np
import pytest
import torch
import torchvision.transforms.v2.functional as TF

import vit_cuda
from vit_cuda.preprocess import IMAGENET_MEAN, IMAGENET_STD

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
from make_preprocess_golden import CASES, synthetic_image  # noqa: E402

pytestmark = pytest.mark.gpu


def torchvision_float(images_bhwc: torch.Tensor, resize: int, crop: int) -> torch.Tensor:
    x = images_bhwc.permute(0, 3, 1, 2).double() / 255.0
    x = TF.resize(x, [resize], interpolation=TF.InterpolationMode.BILINEAR, antialias=True)
    x = TF.center_crop(x, [crop, crop])
    return TF.normalize(x, list(IMAGENET_MEAN), list(IMAGENET_STD))


@pytest.mark.parametrize("H,W,resize,crop", [(375, 500, 256, 224), (500, 375, 256, 224),
                                             (256, 256, 256, 224), (224, 301, 256, 224),
                                             (1000, 777, 256, 224), (61, 47, 64, 56)])
def test_preprocess_matches_torchvision(cuda, H, W, resize, crop):
    g = torch.Generator().manual_seed(H * 7 + W)
    imgs = torch.randint(0, 256, (2, H, W, 3), generator=g, dtype=torch.uint8)
    out = vit_cuda.preprocess(imgs.to(cuda), resize, crop)
    ref = torchvision_float(imgs, resize, crop)
    assert out.shape == (2, 3, crop, crop)
    torch.testing.assert_close(out.double().cpu(), ref, atol=1e-4, rtol=0)


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_preprocess_matches_reference_pil_pipeline(cuda, case):
    name, h, w, resize, crop = case
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "preprocess_golden.npz"))
    img = synthetic_image(h, w, CASES.index(case))
    assert int(img.astype(np.int64).sum()) == int(g[f"{name}/image_sum"][0])
    out = vit_cuda.preprocess(torch.from_numpy(img).to(cuda), resize, crop)[0].double().cpu()
    ref = torch.from_numpy(g[f"{name}/out"].astype(np.float64))
    # one 8-bit step after normalisation (1/255/0.224), plus fixture rounding
    assert (out - ref).abs().max().item() <= 0.02


def test_preprocess_feeds_the_model(cuda):
    """Preprocessed batch -> ViTCUDA equals the torchvision-preprocessed batch
    -> ViTCUDA."""
    from vit_cuda.weights import synthetic_state_dict
    state = synthetic_state_dict(seed=0, img_size=224)
    model = vit_cuda.ViTCUDA(state_dict={k: v.to(cuda) for k, v in state.items()}).to(cuda).eval()
    g = torch.Generator().manual_seed(3)
    imgs = torch.randint(0, 256, (3, 333, 444, 3), generator=g, dtype=torch.uint8)
    with torch.no_grad():
        a = model(vit_cuda.preprocess(imgs.to(cuda)))
        b = model(torchvision_float(imgs, 256, 224).float().to(cuda))
    assert (a - b).abs().max().item() <= 1e-3


def test_preprocess_errors(cuda):
    with pytest.raises(RuntimeError, match="uint8"):
        vit_cuda.preprocess(torch.zeros(1, 8, 8, 3, device=cuda))
    with pytest.raises(RuntimeError, match="smaller than"):
        vit_cuda.preprocess(torch.zeros(1, 300, 300, 3, dtype=torch.uint8, device=cuda), 200, 224)
