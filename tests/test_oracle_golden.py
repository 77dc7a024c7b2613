"""Pins the CPU oracle (oracle/vit_oracle.py) before it is trusted as the checker.

1. Per op, against the expected values the reference's own tests construct
   (loop-built patch vectors, loop-built positional rows, F.layer_norm, X W^T + b,
   manual softmax attention, ...), committed in tests/golden/ops_golden.npz.
2. End to end, against HuggingFace transformers' ViT-B/16 run in float64 on the
   same seeded weights and images (tests/golden/vit_e2e_golden.npz), including
   the 384x384 / T=577 configuration.
3. The seeded weight generator has not drifted (its checksum is in the fixture).
"""
import os

import numpy as np
import pytest
import torch

from oracle import vit_oracle as orc
from vit_cuda.weights import state_checksum, synthetic_images, synthetic_state_dict

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def ops_golden():
    return np.load(os.path.join(GOLDEN, "ops_golden.npz"))


@pytest.fixture(scope="module")
def e2e_golden():
    return np.load(os.path.join(GOLDEN, "vit_e2e_golden.npz"))


def check_stats(t, g, prefix, rtol=1e-10):
    a = t.detach().double().cpu().numpy()
    assert tuple(a.shape) == tuple(g[prefix + "/shape"]), prefix
    np.testing.assert_allclose(a.sum(), g[prefix + "/sum"], rtol=rtol, atol=rtol * float(
        g[prefix + "/abssum"]))
    np.testing.assert_allclose(np.linalg.norm(a.ravel()), g[prefix + "/l2"], rtol=rtol)
    np.testing.assert_allclose(a.ravel()[g[prefix + "/idx"]], g[prefix + "/vals"], rtol=rtol,
                               atol=rtol)


def test_patch_embed(ops_golden):
    torch.manual_seed(0)
    img = torch.randn(1, 3, 224, 224)
    w = torch.randn(768, 768)
    check_stats(orc.patch_embed(img, w), ops_golden, "patch_embed")


def test_pos_encoding(ops_golden):
    torch.manual_seed(0)
    pt = torch.randn(1, 196, 768)
    cls = torch.randn(1, 768)
    pos = torch.randn(197, 768)
    check_stats(orc.pos_encoding(pt, cls, pos), ops_golden, "pos_encoding")


def test_layernorm(ops_golden):
    torch.manual_seed(0)
    X = torch.randn(1, 4, 768)
    g = torch.randn(768)
    b = torch.randn(768)
    check_stats(orc.layernorm(X, g, b, 1e-5), ops_golden, "layernorm")


def test_qkv(ops_golden):
    torch.manual_seed(0)
    X = torch.randn(2, 197, 768)
    W = torch.randn(2304, 768)
    B = torch.randn(2304)
    for t, n in zip(orc.qkv_proj(X, W, B), "qkv"):
        check_stats(t, ops_golden, f"qkv_{n}")


def test_gemm_bias(ops_golden):
    torch.manual_seed(0)
    X = torch.randn(8, 768)
    W = torch.randn(3072, 768)
    B = torch.randn(3072)
    check_stats(orc.linear(X, W, B), ops_golden, "gemm_bias")


def test_mlp(ops_golden):
    torch.manual_seed(0)
    X = torch.randn(1, 3, 768)
    W1, B1 = torch.randn(3072, 768), torch.randn(3072)
    W2, B2 = torch.randn(768, 3072), torch.randn(768)
    O, H = orc.mlp(X, W1, B1, W2, B2)
    check_stats(H, ops_golden, "mlp_H")
    check_stats(O, ops_golden, "mlp_O")


def test_classifier(ops_golden):
    torch.manual_seed(0)
    X = torch.randn(2, 197, 768)
    W = torch.randn(10, 768)
    b = torch.randn(10)
    check_stats(orc.classifier(X, W, b), ops_golden, "classifier")


def test_attention(ops_golden):
    torch.manual_seed(0)
    q, k, v = torch.randn(2, 197, 768), torch.randn(2, 197, 768), torch.randn(2, 197, 768)
    check_stats(orc.attention(q, k, v, 0.125), ops_golden, "flash_attn")


@pytest.mark.parametrize("case", ["b2_224", "b1_384"])
def test_end_to_end_vs_transformers(e2e_golden, case):
    size, B, wseed, iseed = (int(v) for v in e2e_golden[f"{case}/meta"])
    state = synthetic_state_dict(seed=wseed, img_size=size)
    np.testing.assert_allclose(state_checksum(state), e2e_golden[f"{case}/weight_checksum"],
                               rtol=1e-12)
    img = synthetic_images(B, size, seed=iseed)
    np.testing.assert_allclose(img.double().abs().sum().item(),
                               e2e_golden[f"{case}/input_checksum"], rtol=1e-12)
    logits, inter = orc.vit_forward(img, state, return_intermediates=True)
    np.testing.assert_allclose(logits.numpy(), e2e_golden[f"{case}/logits"], atol=1e-10)
    np.testing.assert_allclose(inter["features"].numpy(), e2e_golden[f"{case}/features"],
                               atol=1e-10)
    check_stats(inter["embed"], e2e_golden, f"{case}/embed", rtol=1e-9)
    for i, xb in enumerate(inter["blocks"]):
        check_stats(xb, e2e_golden, f"{case}/block{i}", rtol=1e-9)


def test_float32_oracle_close_to_float64():
    """The fp32 oracle (the timed CPU baseline) stays within the parity bar."""
    state = synthetic_state_dict(seed=3, img_size=224, depth=2)
    img = synthetic_images(1, 224, seed=3)
    a = orc.vit_forward(img, state, dtype=torch.float32)
    b = orc.vit_forward(img, state, dtype=torch.float64)
    assert (a.double() - b).abs().max().item() < 1e-4


def test_oracle_matches_torch_functional():
    """Independent cross-check of each restated op against torch.nn.functional."""
    import torch.nn.functional as F
    g = torch.Generator().manual_seed(5)
    x = torch.randn(2, 9, 768, generator=g, dtype=torch.float64)
    w = torch.randn(768, generator=g, dtype=torch.float64)
    b = torch.randn(768, generator=g, dtype=torch.float64)
    torch.testing.assert_close(orc.layernorm(x, w, b, 1e-6), F.layer_norm(x, (768,), w, b, 1e-6))
    torch.testing.assert_close(orc.gelu_erf(x), F.gelu(x, approximate="none"))
    q, k, v = (torch.randn(2, 9, 768, generator=g, dtype=torch.float64) for _ in range(3))
    sdpa = F.scaled_dot_product_attention(
        q.view(2, 9, 12, 64).transpose(1, 2), k.view(2, 9, 12, 64).transpose(1, 2),
        v.view(2, 9, 12, 64).transpose(1, 2), scale=0.125).transpose(1, 2).reshape(2, 9, 768)
    torch.testing.assert_close(orc.attention(q, k, v, 0.125), sdpa)
    img = torch.randn(2, 3, 32, 48, generator=g, dtype=torch.float64)
    cw = torch.randn(768, 3, 16, 16, generator=g, dtype=torch.float64)
    cb = torch.randn(768, generator=g, dtype=torch.float64)
    conv = F.conv2d(img, cw, cb, stride=16).flatten(2).transpose(1, 2)
    torch.testing.assert_close(orc.patch_embed(img, cw, cb), conv)
