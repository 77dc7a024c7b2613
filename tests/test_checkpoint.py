"""Checkpoint loading (vit_cuda.checkpoint): timm- and HuggingFace-named state
dicts from safetensors and torch.save files, mapped onto the reference's timm
buffer names (vit_cuda/model.py:23-37,78-91 of the reference project)."""
import os
import sys

import pytest
import torch

from vit_cuda import checkpoint
from vit_cuda.weights import synthetic_state_dict

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))


def _same(a, b):
    assert set(a) == set(b)
    for k in a:
        assert torch.equal(a[k].float(), b[k].float()), k


def test_timm_safetensors_and_torch_save(tmp_path):
    from safetensors.torch import save_file
    sd = synthetic_state_dict(seed=3, img_size=224, depth=2)
    save_file(sd, str(tmp_path / "w.safetensors"))
    _same(checkpoint.load_state_dict(str(tmp_path / "w.safetensors")), sd)
    torch.save({"module." + k: v for k, v in sd.items()}, str(tmp_path / "w.pt"))
    _same(checkpoint.load_state_dict(str(tmp_path / "w.pt")), sd)
    torch.save({"state_dict": sd}, str(tmp_path / "w.ckpt"))
    _same(checkpoint.load_state_dict(str(tmp_path / "w.ckpt")), sd)


def test_huggingface_names_map_to_timm(tmp_path):
    """transformers' own ViTForImageClassification state dict (its real key
    names) loads back to the timm dict it was built from."""
    from make_golden import hf_model
    from safetensors.torch import save_file
    sd = synthetic_state_dict(seed=4, img_size=224)
    hf = hf_model(sd, 224).state_dict()
    save_file({k: v.contiguous() for k, v in hf.items()}, str(tmp_path / "hf.safetensors"))
    _same(checkpoint.load_state_dict(str(tmp_path / "hf.safetensors")), sd)


def test_unknown_layout_rejected(tmp_path):
    torch.save({"foo": torch.zeros(2)}, str(tmp_path / "x.pt"))
    with pytest.raises(ValueError):
        checkpoint.load_state_dict(str(tmp_path / "x.pt"))


def test_load_model_cpu_buffers(tmp_path):
    from safetensors.torch import save_file
    sd = synthetic_state_dict(seed=5, img_size=224, depth=2, num_classes=10)
    save_file(sd, str(tmp_path / "w.safetensors"))
    m = checkpoint.load_model(str(tmp_path / "w.safetensors"), device="cpu")
    assert m.num_classes == 10 and len(m.blocks) == 2
    assert torch.equal(m.blocks[1].qkv_weight, sd["blocks.1.attn.qkv.weight"])
    assert torch.equal(m.pos_embed, sd["pos_embed"].squeeze(0))
