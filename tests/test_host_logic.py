"""Host-side logic that needs no GPU: weight generator, sharding arithmetic,
the reference-compatible argument checks of the per-op API, model buffer names."""
import pytest
import torch

import vit_cuda
from vit_cuda import _C
from vit_cuda.parallel import padded_rows, shard_bounds
from vit_cuda.weights import num_tokens, synthetic_images, synthetic_state_dict


def test_synthetic_state_dict_layout():
    sd = synthetic_state_dict(seed=0, img_size=224)
    assert sd["patch_embed.proj.weight"].shape == (768, 3, 16, 16)
    assert sd["pos_embed"].shape == (1, 197, 768)
    assert sd["cls_token"].shape == (1, 1, 768)
    assert sd["blocks.11.attn.qkv.weight"].shape == (2304, 768)
    assert sd["blocks.0.mlp.fc2.weight"].shape == (768, 3072)
    assert sd["head.weight"].shape == (1000, 768)
    w = sd["blocks.3.mlp.fc1.weight"]
    assert abs(w.std().item() - 0.02) < 1e-3 and w.abs().max().item() < 2.0
    assert torch.all(sd["blocks.5.norm2.weight"] == 1) and torch.all(sd["norm.bias"] == 0)
    assert num_tokens(384) == 577
    sd2 = synthetic_state_dict(seed=0, img_size=224)
    assert all(torch.equal(sd[k], sd2[k]) for k in sd)


def test_synthetic_images():
    x = synthetic_images(2, 224, seed=0)
    assert x.shape == (2, 3, 224, 224) and x.dtype == torch.float32
    assert torch.equal(x, synthetic_images(2, 224, seed=0))


@pytest.mark.parametrize("total,world", [(256, 1), (2048, 8), (4096, 8), (5, 2), (3, 4), (0, 2)])
def test_shard_bounds_cover_exactly(total, world):
    seen = []
    for r in range(world):
        s, e = shard_bounds(total, world, r)
        assert 0 <= s <= e <= total
        assert e - s <= padded_rows(total, world)
        seen.extend(range(s, e))
    assert seen == list(range(total))


def test_shard_bounds_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_bounds(10, 2, 2)


def test_ops_reject_cpu_tensors_like_the_reference():
    """csrc/include/cuda_checks.h:21-50 of the reference: non-CUDA inputs raise."""
    x = torch.randn(1, 4, 768)
    g = torch.ones(768)
    with pytest.raises(RuntimeError, match="CUDA"):
        _C.layernorm_forward(x, g, g, 1e-6)
    with pytest.raises(RuntimeError, match="CUDA"):
        _C.gemm_bias(x, torch.randn(8, 768), torch.randn(8))
    with pytest.raises(RuntimeError, match="CUDA"):
        _C.flash_attn_2(x, x, x, 0.125)
    with pytest.raises(RuntimeError, match="CUDA"):
        _C.patch_embed(torch.randn(1, 3, 224, 224), torch.randn(768, 768))


def test_package_surface():
    """vit_cuda.<op> (through the registered torch.ops.vit_cuda ops) and
    vit_cuda._C.<op> (direct) exist for the eight reference ops and raise the
    reference wrappers' RuntimeError for non-CUDA inputs alike."""
    for name in ["flash_attn_2", "patch_embed", "pos_encoding", "mlp_forward",
                 "layernorm_forward", "classifier_forward", "qkv_proj", "gemm_bias"]:
        assert callable(getattr(vit_cuda, name))
        assert callable(getattr(vit_cuda._C, name))
    x = torch.randn(1, 4, 768)
    for mod in (vit_cuda, vit_cuda._C):
        with pytest.raises(RuntimeError, match="CUDA"):
            mod.layernorm_forward(x, torch.ones(768), torch.zeros(768), 1e-6)
        with pytest.raises(RuntimeError, match="CUDA"):
            mod.qkv_proj(x, torch.randn(2304, 768), torch.randn(2304))


def test_model_buffer_names_match_reference():
    """Buffer names of vit_cuda/model.py:23-37,78-91 in the reference."""
    sd = synthetic_state_dict(seed=0, img_size=224, depth=2)
    m = vit_cuda.ViTCUDA(state_dict=sd)
    names = set(dict(m.named_buffers()))
    for n in ["patch_weight", "patch_bias", "cls_token", "pos_embed", "norm_gamma", "norm_beta",
              "head_weight", "head_bias", "blocks.1.qkv_weight", "blocks.0.fc2_bias",
              "blocks.1.norm1_gamma", "blocks.0.norm2_beta", "blocks.1.proj_weight"]:
        assert n in names, n
    assert m.cls_token.shape == (1, 768) and m.pos_embed.shape == (197, 768)
    assert m.img_size == (224, 224) and len(m.blocks) == 2
    with pytest.raises(RuntimeError, match="CUDA"):
        m.prepare()


def test_model_384_geometry():
    sd = synthetic_state_dict(seed=0, img_size=384, depth=1)
    m = vit_cuda.ViTCUDA(state_dict=sd)
    assert m.img_size == (384, 384) and m.pos_embed.shape == (577, 768)


def test_model_requires_state_dict_without_timm():
    with pytest.raises(RuntimeError):
        vit_cuda.ViTCUDA(state_dict=None)


def test_layernorm_bound_is_tight_and_safe():
    """The bound used to choose FP16 operands holds for the worst-case row (one
    outlier among equal entries reaches sqrt(E - 1)) and for random rows."""
    import math
    from vit_cuda.split import layernorm_bound
    E = 768
    g = torch.rand(E, dtype=torch.float64) * 3
    b = torch.randn(E, dtype=torch.float64)
    bound = layernorm_bound(g, b)
    x = torch.zeros(4, E, dtype=torch.float64)
    x[0, 5] = 1.0
    x[1] = torch.randn(E, dtype=torch.float64)
    x[2, :] = 1.0
    x[2, 7] = -1e6
    x[3] = torch.randn(E, dtype=torch.float64) * 1e3
    y = torch.nn.functional.layer_norm(x, (E,), g, b, 1e-6)
    assert float(y.abs().max()) <= bound
    z = torch.nn.functional.layer_norm(x[:1], (E,), None, None, 0.0)
    assert abs(float(z.abs().max()) - math.sqrt(E - 1)) < 1e-9


def test_linear_bound_and_weight_scale():
    import math
    from vit_cuda.split import f16_weight_ok, f16_weight_scale, linear_bound
    w = torch.tensor([[1.0, -2.0], [0.5, 0.25]])
    assert linear_bound(3.0, w, torch.tensor([0.1, -0.4])) == pytest.approx(3.0 * 3.0 + 0.4)
    for m in (1e-5, 0.02, 1.0, 7.9, 8.0, 300.0):
        s = f16_weight_scale(torch.tensor([m, -m / 3]))
        assert 8.0 <= m * s < 16.0 and math.log2(s) == int(math.log2(s))
    assert f16_weight_scale(torch.zeros(3)) == 1.0
    assert not f16_weight_ok(torch.tensor([1e-30]))
    assert not f16_weight_ok(torch.tensor([float("inf")]))
    assert f16_weight_ok(torch.tensor([0.02]))


def test_custom_ops_registered_with_fake_shapes():
    """The ops are registered with torch.library; their fake implementations
    give the reference ops' output shapes without a GPU."""
    from torch._subclasses.fake_tensor import FakeTensorMode
    import vit_cuda  # noqa: F401  (registers torch.ops.vit_cuda.*)
    ops = torch.ops.vit_cuda
    with FakeTensorMode():
        x = torch.empty(2, 197, 768, device="cuda")
        w = torch.empty(768, 768, device="cuda")
        b = torch.empty(768, device="cuda")
        assert ops.flash_attn_2(x, x, x, 0.125).shape == (2, 197, 768)
        img = torch.empty(2, 3, 224, 224, device="cuda")
        assert ops.patch_embed(img, w, b).shape == (2, 196, 768)
        assert ops.pos_encoding(torch.empty(2, 196, 768, device="cuda"),
                                torch.empty(2, 768, device="cuda"),
                                torch.empty(197, 768, device="cuda")).shape == (2, 197, 768)
        o, h = ops.mlp_forward(x, torch.empty(3072, 768, device="cuda"),
                               torch.empty(3072, device="cuda"),
                               torch.empty(768, 3072, device="cuda"), b)
        assert o.shape == (2, 197, 768) and h.shape == (2, 197, 3072)
        assert ops.layernorm_forward(x, b, b, 1e-6).shape == (2, 197, 768)
        assert ops.classifier_forward(x, torch.empty(1000, 768, device="cuda"),
                                      torch.empty(1000, device="cuda")).shape == (2, 1000)
        assert ops.qkv_proj_packed(x, torch.empty(2304, 768, device="cuda"),
                                   torch.empty(2304, device="cuda")).shape == (3, 2, 197, 768)
        assert ops.gemm_bias(x, w, b).shape == (2, 197, 768)
        assert ops.vit_forward(img, 12345, 1000).shape == (2, 1000)
