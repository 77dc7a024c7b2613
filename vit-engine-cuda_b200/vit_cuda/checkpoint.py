"""Checkpoint loading for ViTCUDA (the reference loads timm's pretrained
weights through ``timm.create_model(..., pretrained=True)``,
vit_cuda/model.py:67-71, and downloads them with scripts/download_model.py).

* ``load_state_dict(path)`` reads a state dict saved with safetensors or
  ``torch.save`` and returns it in timm's ``vit_base_patch16_*`` layout (the
  buffer names ViTCUDA keeps): timm-named dicts pass through (a leading
  ``module.`` / ``model.`` is dropped), HuggingFace ``ViTForImageClassification``
  dicts are renamed and their separate query / key / value projections
  concatenated into timm's fused ``qkv``.
* ``load_model(path, device)`` builds a ready ViTCUDA from such a file.
* ``save_splits(model, path)`` / ``load_splits(model, path)`` store and restore
  the engine's split weights (FP16 planes or TF32 pairs, their scales and the
  per-GEMM operand choice) — the offline pre-split — keyed by a fingerprint of
  the source weights, so a stale file is refused.
"""
from __future__ import annotations

import hashlib
import os

import torch

_PREFIXES = ("module.", "model.")


def _read(path: str) -> dict[str, torch.Tensor]:
    if path.endswith(".safetensors"):
        from safetensors.torch import load_file
        return load_file(path, device="cpu")
    obj = torch.load(path, map_location="cpu", weights_only=True)
    if isinstance(obj, dict) and "state_dict" in obj and isinstance(obj["state_dict"], dict):
        obj = obj["state_dict"]
    if not isinstance(obj, dict):
        raise ValueError(f"{path}: not a state dict")
    return obj


def hf_to_timm(sd: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
    """HuggingFace ViTForImageClassification names -> timm vit_base_patch16."""
    out = {
        "cls_token": sd["vit.embeddings.cls_token"],
        "pos_embed": sd["vit.embeddings.position_embeddings"],
        "patch_embed.proj.weight": sd["vit.embeddings.patch_embeddings.projection.weight"],
        "patch_embed.proj.bias": sd["vit.embeddings.patch_embeddings.projection.bias"],
        "norm.weight": sd["vit.layernorm.weight"],
        "norm.bias": sd["vit.layernorm.bias"],
        "head.weight": sd["classifier.weight"],
        "head.bias": sd["classifier.bias"],
    }
    i = 0
    while f"vit.encoder.layer.{i}.layernorm_before.weight" in sd:
        h, p = f"vit.encoder.layer.{i}.", f"blocks.{i}."
        att = h + "attention.attention."
        out[p + "attn.qkv.weight"] = torch.cat(
            [sd[att + n + ".weight"] for n in ("query", "key", "value")], dim=0)
        out[p + "attn.qkv.bias"] = torch.cat(
            [sd[att + n + ".bias"] for n in ("query", "key", "value")], dim=0)
        pairs = {"layernorm_before": "norm1", "attention.output.dense": "attn.proj",
                 "layernorm_after": "norm2", "intermediate.dense": "mlp.fc1",
                 "output.dense": "mlp.fc2"}
        for hf, tm in pairs.items():
            out[p + tm + ".weight"] = sd[h + hf + ".weight"]
            out[p + tm + ".bias"] = sd[h + hf + ".bias"]
        i += 1
    if i == 0:
        raise ValueError("no encoder layers found (expected vit.encoder.layer.N.*)")
    return out


def to_timm(sd: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
    """Any supported naming -> timm's, tensors as float32."""
    for pre in _PREFIXES:
        if sd and all(k.startswith(pre) for k in sd):
            sd = {k[len(pre):]: v for k, v in sd.items()}
    if "vit.embeddings.cls_token" in sd:
        sd = hf_to_timm(sd)
    if "patch_embed.proj.weight" not in sd or "blocks.0.attn.qkv.weight" not in sd:
        raise ValueError("unrecognised checkpoint layout (neither timm nor HuggingFace ViT)")
    return {k: v.float().contiguous() for k, v in sd.items()}


def load_state_dict(path: str) -> dict[str, torch.Tensor]:
    return to_timm(_read(path))


def load_model(path: str, device="cuda"):
    """A ViTCUDA with the checkpoint's weights on ``device`` (num_classes from
    the head), weights split and ready."""
    from .model import ViTCUDA
    sd = load_state_dict(path)
    model = ViTCUDA(num_classes=sd["head.weight"].shape[0],
                    state_dict={k: v.to(device) for k, v in sd.items()})
    model = model.to(device).eval()
    if torch.device(device).type == "cuda":
        model.prepare()
    return model


def fingerprint(model) -> str:
    """SHA-256 over the model's buffers (names, shapes and bytes)."""
    h = hashlib.sha256()
    for name, buf in sorted(model.named_buffers()):
        h.update(name.encode())
        h.update(str(tuple(buf.shape)).encode())
        h.update(buf.detach().contiguous().cpu().numpy().tobytes())
    return h.hexdigest()


def save_splits(model, path: str) -> None:
    """Stores the prepared model's split weights (safetensors) with the
    fingerprint of the weights they came from."""
    from safetensors.torch import save_file
    tensors, meta = model.export_splits()
    meta["fingerprint"] = fingerprint(model)
    save_file({k: v.contiguous().cpu() for k, v in tensors.items()}, path, metadata=meta)


def load_splits(model, path: str) -> None:
    """Restores split weights saved by ``save_splits`` into ``model`` (already
    on its CUDA device), skipping the split; refuses a file made from other
    weights."""
    from safetensors import safe_open
    with safe_open(path, framework="pt", device="cpu") as f:
        meta = f.metadata() or {}
        if meta.get("fingerprint") != fingerprint(model):
            raise ValueError(f"{os.path.basename(path)}: split weights were made from other "
                             "weights (fingerprint mismatch)")
        tensors = {k: f.get_tensor(k) for k in f.keys()}
    model.import_splits(tensors, meta)
