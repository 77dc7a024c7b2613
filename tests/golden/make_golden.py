"""Generates the golden fixtures that pin the CPU oracle (oracle/vit_oracle.py).

    python tests/golden/make_golden.py          # rewrites tests/golden/*.npz

vit_e2e_golden.npz — for each case (224x224 B=2, 384x384 B=1), the float64
logits, CLS features and per-block checksums of HuggingFace transformers'
ViTForImageClassification, an independent implementation of the published
ViT-B/16 that timm's vit_base_patch16_224 also implements, loaded with the
seeded synthetic weights of vit_cuda.weights.synthetic_state_dict (timm itself
is not installed). The script asserts that the oracle agrees before writing.

ops_golden.npz — per-op expected values built the way the reference's own
tests build them (loop-assembled patch vectors, tests/test_patch_embed.py:48-56;
loop-assembled positional rows, tests/test_pos_encoding.py:43-47;
F.layer_norm at eps 1e-5, tests/test_layernorm.py:43; X W^T + b split at 768,
tests/test_qkv.py:41-44; GPU-style MLP chain, tests/test_mlp.py:54-59; CLS-row
classifier, tests/test_classifier.py:42-43; manual attention,
tests/test_flash_attn.py:10-24), stored as checksums plus sampled entries.
"""
from __future__ import annotations

import math
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "vit-engine-cuda_b200"))
sys.path.insert(0, REPO)

from oracle import vit_oracle as orc  # noqa: E402
from vit_cuda.weights import (state_checksum, synthetic_images,  # noqa: E402
                              synthetic_state_dict)

E2E_CASES = [  # (name, img_size, batch, weight_seed, input_seed)
    ("b2_224", 224, 2, 0, 0),
    ("b1_384", 384, 1, 1, 1),
]
N_SAMPLES = 64


def sample_index(shape, n=N_SAMPLES, seed=1234):
    g = np.random.default_rng(seed)
    total = int(np.prod(shape))
    return np.sort(g.choice(total, size=min(n, total), replace=False))


def stats(t: torch.Tensor, prefix: str, out: dict):
    a = t.detach().double().cpu().numpy()
    out[prefix + "/shape"] = np.array(a.shape)
    out[prefix + "/sum"] = np.array(a.sum())
    out[prefix + "/l2"] = np.array(np.linalg.norm(a.ravel()))
    out[prefix + "/abssum"] = np.array(np.abs(a).sum())
    idx = sample_index(a.shape)
    out[prefix + "/idx"] = idx
    out[prefix + "/vals"] = a.ravel()[idx]


def hf_model(state, img_size):
    from transformers import ViTConfig, ViTForImageClassification
    cfg = ViTConfig(hidden_size=768, num_hidden_layers=12, num_attention_heads=12,
                    intermediate_size=3072, hidden_act="gelu", layer_norm_eps=1e-6,
                    image_size=img_size, patch_size=16, num_channels=3, qkv_bias=True,
                    num_labels=state["head.weight"].shape[0], hidden_dropout_prob=0.0,
                    attention_probs_dropout_prob=0.0)
    cfg._attn_implementation = "eager"
    m = ViTForImageClassification(cfg)
    sd = {
        "vit.embeddings.cls_token": state["cls_token"],
        "vit.embeddings.position_embeddings": state["pos_embed"],
        "vit.embeddings.patch_embeddings.projection.weight": state["patch_embed.proj.weight"],
        "vit.embeddings.patch_embeddings.projection.bias": state["patch_embed.proj.bias"],
        "vit.layernorm.weight": state["norm.weight"],
        "vit.layernorm.bias": state["norm.bias"],
        "classifier.weight": state["head.weight"],
        "classifier.bias": state["head.bias"],
    }
    for i in range(12):
        p, h = f"blocks.{i}.", f"vit.encoder.layer.{i}."
        w, b = state[p + "attn.qkv.weight"], state[p + "attn.qkv.bias"]
        for j, n in enumerate(("query", "key", "value")):
            sd[h + f"attention.attention.{n}.weight"] = w[j * 768:(j + 1) * 768]
            sd[h + f"attention.attention.{n}.bias"] = b[j * 768:(j + 1) * 768]
        sd[h + "attention.output.dense.weight"] = state[p + "attn.proj.weight"]
        sd[h + "attention.output.dense.bias"] = state[p + "attn.proj.bias"]
        sd[h + "intermediate.dense.weight"] = state[p + "mlp.fc1.weight"]
        sd[h + "intermediate.dense.bias"] = state[p + "mlp.fc1.bias"]
        sd[h + "output.dense.weight"] = state[p + "mlp.fc2.weight"]
        sd[h + "output.dense.bias"] = state[p + "mlp.fc2.bias"]
        sd[h + "layernorm_before.weight"] = state[p + "norm1.weight"]
        sd[h + "layernorm_before.bias"] = state[p + "norm1.bias"]
        sd[h + "layernorm_after.weight"] = state[p + "norm2.weight"]
        sd[h + "layernorm_after.bias"] = state[p + "norm2.bias"]
    missing, unexpected = m.load_state_dict(sd, strict=False)
    assert not unexpected and not [k for k in missing if "pooler" not in k], (missing, unexpected)
    return m.double().eval()


def hf_forward(state, img, img_size):
    m = hf_model(state, img_size)
    with torch.no_grad():
        out = m(pixel_values=img.double(), output_hidden_states=True)
        hidden = out.hidden_states  # embeddings, then each block output
        feats = m.vit.layernorm(hidden[-1])[:, 0, :]
    return out.logits.detach(), feats.detach(), [h.detach() for h in hidden]


def make_e2e() -> dict:
    out = {}
    for name, size, B, wseed, iseed in E2E_CASES:
        state = synthetic_state_dict(seed=wseed, img_size=size)
        img = synthetic_images(B, size, seed=iseed)
        logits, feats, hidden = hf_forward(state, img, size)
        o_logits, inter = orc.vit_forward(img, state, return_intermediates=True)
        err = (o_logits - logits).abs().max().item()
        assert err < 1e-9, f"oracle vs transformers logits differ by {err} ({name})"
        for i, hb in enumerate(inter["blocks"]):
            assert orc.rel_l2(hb, hidden[i + 1]) < 1e-12, (name, i)
        out[f"{name}/meta"] = np.array([size, B, wseed, iseed])
        out[f"{name}/weight_checksum"] = np.array(state_checksum(state))
        out[f"{name}/input_checksum"] = np.array(img.double().abs().sum().item())
        out[f"{name}/logits"] = logits.numpy()
        out[f"{name}/features"] = feats.numpy()
        stats(hidden[0], f"{name}/embed", out)
        for i in range(12):
            stats(hidden[i + 1], f"{name}/block{i}", out)
        print(f"{name}: oracle-vs-transformers max|dlogits| = {err:.3e}")
    return out


def make_ops() -> dict:
    out = {}
    d = torch.float64

    # patch_embed, tests/test_patch_embed.py:19-59 construction (B=1, 224, seed 0).
    torch.manual_seed(0)
    img = torch.randn(1, 3, 224, 224)
    w = torch.randn(768, 768)
    patches = []
    for p in range(196):
        row, col = (p // 14) * 16, (p % 14) * 16
        patches.append(img[0, :, row:row + 16, col:col + 16].reshape(-1))
    expected = (torch.stack(patches).double() @ w.double().t()).unsqueeze(0)
    stats(expected, "patch_embed", out)

    # pos_encoding, tests/test_pos_encoding.py:19-50 construction.
    torch.manual_seed(0)
    pt = torch.randn(1, 196, 768)
    cls = torch.randn(1, 768)
    pos = torch.randn(197, 768)
    exp = torch.zeros(1, 197, 768, dtype=d)
    exp[0, 0] = cls[0].double() + pos[0].double()
    for i in range(1, 197):
        exp[0, i] = pt[0, i - 1].double() + pos[i].double()
    stats(exp, "pos_encoding", out)

    # layernorm, tests/test_layernorm.py:19-46 (eps 1e-5).
    torch.manual_seed(0)
    X = torch.randn(1, 4, 768)
    g = torch.randn(768)
    b = torch.randn(768)
    stats(F.layer_norm(X.double(), (768,), g.double(), b.double(), 1e-5), "layernorm", out)

    # qkv, tests/test_qkv.py:19-48.
    torch.manual_seed(0)
    X = torch.randn(2, 197, 768)
    W = torch.randn(2304, 768)
    Bq = torch.randn(2304)
    ref = X.double() @ W.double().t() + Bq.double()
    for j, n in enumerate("qkv"):
        stats(ref[..., j * 768:(j + 1) * 768], f"qkv_{n}", out)

    # gemm_bias, tests/test_qkv.py:51-73.
    torch.manual_seed(0)
    X = torch.randn(8, 768)
    W = torch.randn(3072, 768)
    Bg = torch.randn(3072)
    stats(X.double() @ W.double().t() + Bg.double(), "gemm_bias", out)

    # mlp, tests/test_mlp.py:24-69 (unit-variance weights).
    torch.manual_seed(0)
    X = torch.randn(1, 3, 768)
    W1, B1 = torch.randn(3072, 768), torch.randn(3072)
    W2, B2 = torch.randn(768, 3072), torch.randn(768)
    H = X.double().reshape(3, 768) @ W1.double().t() + B1.double()
    H = 0.5 * H * (1.0 + torch.erf(H / math.sqrt(2)))
    O = H @ W2.double().t() + B2.double()
    stats(H.view(1, 3, 3072), "mlp_H", out)
    stats(O.view(1, 3, 768), "mlp_O", out)

    # classifier, tests/test_classifier.py:19-46.
    torch.manual_seed(0)
    X = torch.randn(2, 197, 768)
    W = torch.randn(10, 768)
    bc = torch.randn(10)
    stats(X[:, 0, :].double() @ W.double().t() + bc.double(), "classifier", out)

    # flash attention, tests/test_flash_attn.py:26-49 (seeded here; the
    # reference test draws unseeded inputs).
    torch.manual_seed(0)
    q = torch.randn(2, 197, 768)
    k = torch.randn(2, 197, 768)
    v = torch.randn(2, 197, 768)
    qh = q.double().view(2, 197, 12, 64).transpose(1, 2)
    kh = k.double().view(2, 197, 12, 64).transpose(1, 2)
    vh = v.double().view(2, 197, 12, 64).transpose(1, 2)
    a = F.softmax(torch.matmul(qh, kh.transpose(-2, -1)) * 0.125, dim=-1)
    o = torch.matmul(a, vh).transpose(1, 2).contiguous().view(2, 197, 768)
    stats(o, "flash_attn", out)
    return out


def main():
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    np.savez_compressed(os.path.join(HERE, "ops_golden.npz"), **make_ops())
    np.savez_compressed(os.path.join(HERE, "vit_e2e_golden.npz"), **make_e2e())
    print("wrote", os.path.join(HERE, "ops_golden.npz"), os.path.join(HERE, "vit_e2e_golden.npz"))


if __name__ == "__main__":
    main()
