"""Seeded random-init ViT-B/16 weights in timm's state-dict layout.

Pretrained checkpoints are not available offline, so every test and benchmark
uses these: trunc_normal(std=0.02, bounds +-2) for the conv / linear weights,
pos_embed and cls_token; LayerNorm weight 1 and bias 0; linear and conv biases
N(0, 0.02). Key names and shapes are those the reference model reads
(vit_cuda/model.py:23-37, 78-91 of the reference project).
"""
from __future__ import annotations

import torch

EMBED = 768
HEADS = 12
MLP = 3072
PATCH = 16


def num_tokens(img_size: int | tuple[int, int]) -> int:
    h, w = (img_size, img_size) if isinstance(img_size, int) else img_size
    return (h // PATCH) * (w // PATCH) + 1


def synthetic_state_dict(seed: int = 0, img_size: int | tuple[int, int] = 224,
                         num_classes: int = 1000, depth: int = 12,
                         in_chans: int = 3, stats: str = "init") -> dict[str, torch.Tensor]:
    """CPU float32 state dict with timm's `vit_base_patch16_*` key names.

    stats="init" (default): timm's initialisation, as above. stats="trained":
    the same draws reshaped to resemble a trained ViT-B/16's statistics (no
    pretrained checkpoint is available offline): LayerNorm gains spread
    log-normally and growing with depth, with a few channels per block at
    5-10; LayerNorm biases N(0, 0.2); linear weights twice as wide, with one
    entry in a hundred four times larger (heavier row sums); positional and
    CLS embeddings ten times larger."""
    if stats not in ("init", "trained"):
        raise ValueError("stats must be 'init' or 'trained'")
    sd = _init_state_dict(seed, img_size, num_classes, depth, in_chans)
    if stats == "trained":
        _reshape_trained(sd, seed, depth)
    return sd


def _reshape_trained(sd: dict[str, torch.Tensor], seed: int, depth: int) -> None:
    g = torch.Generator(device="cpu")
    g.manual_seed(int(seed) + 7919)

    def gains(i):
        gm = torch.exp(torch.randn(EMBED, generator=g) * (0.3 + 0.05 * i))
        idx = torch.randperm(EMBED, generator=g)[:4]
        gm[idx] = 5.0 + 5.0 * torch.rand(4, generator=g)
        return gm

    def heavy(w):
        w = w * 2.0
        mask = torch.rand(w.shape, generator=g) < 0.01
        return torch.where(mask, w * 4.0, w)

    for i in range(depth):
        p = f"blocks.{i}."
        for ln in ("norm1", "norm2"):
            sd[p + ln + ".weight"] = gains(i)
            sd[p + ln + ".bias"] = torch.randn(EMBED, generator=g) * 0.2
        for lin in ("attn.qkv", "attn.proj", "mlp.fc1", "mlp.fc2"):
            sd[p + lin + ".weight"] = heavy(sd[p + lin + ".weight"])
    sd["norm.weight"] = gains(depth)
    sd["norm.bias"] = torch.randn(EMBED, generator=g) * 0.2
    sd["pos_embed"] = sd["pos_embed"] * 10.0
    sd["cls_token"] = sd["cls_token"] * 10.0


def _init_state_dict(seed, img_size, num_classes, depth, in_chans):
    g = torch.Generator(device="cpu")
    g.manual_seed(int(seed))
    T = num_tokens(img_size)

    def tn(*shape):
        t = torch.empty(*shape, dtype=torch.float32)
        torch.nn.init.trunc_normal_(t, mean=0.0, std=0.02, a=-2.0, b=2.0, generator=g)
        return t

    def nb(n):
        return torch.randn(n, generator=g, dtype=torch.float32) * 0.02

    sd: dict[str, torch.Tensor] = {}
    sd["cls_token"] = tn(1, 1, EMBED)
    sd["pos_embed"] = tn(1, T, EMBED)
    sd["patch_embed.proj.weight"] = tn(EMBED, in_chans, PATCH, PATCH)
    sd["patch_embed.proj.bias"] = nb(EMBED)
    for i in range(depth):
        p = f"blocks.{i}."
        sd[p + "norm1.weight"] = torch.ones(EMBED)
        sd[p + "norm1.bias"] = torch.zeros(EMBED)
        sd[p + "attn.qkv.weight"] = tn(3 * EMBED, EMBED)
        sd[p + "attn.qkv.bias"] = nb(3 * EMBED)
        sd[p + "attn.proj.weight"] = tn(EMBED, EMBED)
        sd[p + "attn.proj.bias"] = nb(EMBED)
        sd[p + "norm2.weight"] = torch.ones(EMBED)
        sd[p + "norm2.bias"] = torch.zeros(EMBED)
        sd[p + "mlp.fc1.weight"] = tn(MLP, EMBED)
        sd[p + "mlp.fc1.bias"] = nb(MLP)
        sd[p + "mlp.fc2.weight"] = tn(EMBED, MLP)
        sd[p + "mlp.fc2.bias"] = nb(EMBED)
    sd["norm.weight"] = torch.ones(EMBED)
    sd["norm.bias"] = torch.zeros(EMBED)
    sd["head.weight"] = tn(num_classes, EMBED)
    sd["head.bias"] = nb(num_classes)
    return sd


def synthetic_images(batch: int, img_size: int | tuple[int, int] = 224, seed: int = 0,
                     in_chans: int = 3) -> torch.Tensor:
    """N(0, 1) images [batch, C, H, W] (already-normalised statistics), CPU fp32."""
    h, w = (img_size, img_size) if isinstance(img_size, int) else img_size
    g = torch.Generator(device="cpu")
    g.manual_seed(int(seed))
    return torch.randn(batch, in_chans, h, w, generator=g, dtype=torch.float32)


def state_checksum(sd: dict[str, torch.Tensor]) -> float:
    """Order-independent fingerprint of a state dict (sum of |w| in float64)."""
    return float(sum(t.double().abs().sum().item() for t in sd.values()))
