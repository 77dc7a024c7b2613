"""The reference project's own CUDA kernels, compiled from its sources for sm_100a
(oracle/Makefile -> oracle/_ref/libvitref.so), run on the B200 next to the CPU
oracle and this engine, on the same inputs.

This pins the oracle to the reference itself. Each reference kernel must agree
with the oracle within the reference's own test tolerances, and the reference's
full forward, composed the way its ViTCUDA does it (vit_cuda/model.py:101-126:
patch_embed + bias, CLS expand, pos_encoding, 12 blocks of LN / qkv / split /
attention / proj / add / LN / MLP / add, LN, classifier), must match the oracle's
logits and this engine's. The reference kernels hardcode 224x224, 197 tokens and
E=768, and need K, N multiples of 4, so only those shapes are used. Skipped when
the library was not built (the reference sources are not on every machine).
"""
import ctypes
import os

import pytest
import torch

from oracle import vit_oracle as orc

pytestmark = pytest.mark.gpu

REF_LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle",
                       "_ref", "libvitref.so")


@pytest.fixture(scope="module")
def ref(cuda):
    if not os.path.exists(REF_LIB):
        pytest.skip("oracle/_ref/libvitref.so not built (needs the reference sources)")
    lib = ctypes.CDLL(REF_LIB)
    P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    sigs = {
        "ref_layernorm": [P, P, P, P, I, I, F, P],
        "ref_gemm": [P, P, P, P, I, I, I, I, P],
        "ref_attention": [P, P, P, P, I, I, F, P],
        "ref_patch_embed": [P, P, P, I, P],
        "ref_pos_encoding": [P, P, P, P, I, P],
        "ref_classifier": [P, P, P, P, I, I, P],
        "ref_mlp": [P, P, P, P, P, P, P, I, I, I, P],
    }
    for n, a in sigs.items():
        getattr(lib, n).argtypes = a
        getattr(lib, n).restype = I
    return lib


def _s():
    return torch.cuda.current_stream().cuda_stream


def _ok(st):
    assert st == 0, f"reference kernel launch failed: {st}"


class RefOps:
    """The reference's per-op wrappers (csrc/ops/*_wrapper.cpp) over its kernels."""

    def __init__(self, lib):
        self.lib = lib

    def layernorm(self, x, g, b, eps):
        y = torch.empty_like(x)
        _ok(self.lib.ref_layernorm(x.data_ptr(), g.data_ptr(), b.data_ptr(), y.data_ptr(),
                                   x.shape[0], x.shape[1], eps, _s()))
        return y

    def gemm(self, x, w, b, mode=1):
        M, K = x.reshape(-1, x.shape[-1]).shape
        N = w.shape[0]
        y = torch.empty(M, N, device=x.device)
        _ok(self.lib.ref_gemm(x.data_ptr(), w.data_ptr(), b.data_ptr() if b is not None else None,
                              y.data_ptr(), M, K, N, mode, _s()))
        return y.view(*x.shape[:-1], N)

    def attention(self, q, k, v, scale):
        o = torch.zeros_like(q)
        _ok(self.lib.ref_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                   q.shape[0], q.shape[1], scale, _s()))
        return o

    def patch_embed(self, img, w, b):
        out = torch.zeros(img.shape[0], 196, 768, device=img.device)
        _ok(self.lib.ref_patch_embed(img.data_ptr(), w.data_ptr(), out.data_ptr(), img.shape[0],
                                     _s()))
        return out + b.view(1, 1, -1) if b is not None else out

    def pos_encoding(self, patches, cls, pos):
        out = torch.zeros(patches.shape[0], 197, 768, device=patches.device)
        _ok(self.lib.ref_pos_encoding(patches.data_ptr(), cls.data_ptr(), pos.data_ptr(),
                                      out.data_ptr(), patches.shape[0], _s()))
        return out

    def classifier(self, x, w, b):
        y = torch.empty(x.shape[0], w.shape[0], device=x.device)
        _ok(self.lib.ref_classifier(x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(),
                                    x.shape[0], w.shape[0], _s()))
        return y

    def mlp(self, x, w1, b1, w2, b2):
        M, E = x.reshape(-1, x.shape[-1]).shape
        E4 = w1.shape[0]
        h = torch.empty(M, E4, device=x.device)
        o = torch.empty(M, E, device=x.device)
        _ok(self.lib.ref_mlp(x.data_ptr(), w1.data_ptr(), b1.data_ptr(), w2.data_ptr(),
                             b2.data_ptr(), h.data_ptr(), o.data_ptr(), M, E, E4, _s()))
        return o.view(*x.shape), h.view(*x.shape[:-1], E4)

    def forward(self, img, sd):
        """The reference ViTCUDA._forward_impl (vit_cuda/model.py:101-126)."""
        g = {k: v for k, v in sd.items()}
        B = img.shape[0]
        x = self.patch_embed(img, g["patch_embed.proj.weight"].reshape(768, -1).contiguous(),
                             g["patch_embed.proj.bias"])
        cls = g["cls_token"].reshape(1, 768).expand(B, -1).contiguous()
        x = self.pos_encoding(x.contiguous(), cls, g["pos_embed"].reshape(-1, 768).contiguous())
        for i in range(12):
            p = f"blocks.{i}."
            res = x
            h = self.layernorm(x, g[p + "norm1.weight"], g[p + "norm1.bias"], 1e-6)
            y = self.gemm(h, g[p + "attn.qkv.weight"], g[p + "attn.qkv.bias"])
            yr = y.view(B, 197, 3, 768)
            q, k, v = (yr.select(2, j).contiguous() for j in range(3))
            a = self.attention(q, k, v, 0.125)
            x = res + self.gemm(a, g[p + "attn.proj.weight"], g[p + "attn.proj.bias"])
            res = x
            h = self.layernorm(x, g[p + "norm2.weight"], g[p + "norm2.bias"], 1e-6)
            o, _ = self.mlp(h, g[p + "mlp.fc1.weight"], g[p + "mlp.fc1.bias"],
                            g[p + "mlp.fc2.weight"], g[p + "mlp.fc2.bias"])
            x = res + o
        x = self.layernorm(x, g["norm.weight"], g["norm.bias"], 1e-6)
        return self.classifier(x, g["head.weight"], g["head.bias"])


def test_reference_ops_agree_with_oracle(ref, cuda):
    r = RefOps(ref)
    torch.manual_seed(0)
    x = torch.randn(1, 4, 768)
    g, b = torch.randn(768), torch.randn(768)
    y = r.layernorm(x.to(cuda), g.to(cuda), b.to(cuda), 1e-5)
    torch.testing.assert_close(y.double().cpu(), orc.layernorm(x, g, b, 1e-5), atol=1e-4, rtol=0)

    X, W, Bv = torch.randn(8, 768), torch.randn(3072, 768), torch.randn(3072)
    y = r.gemm(X.to(cuda), W.to(cuda), Bv.to(cuda))
    torch.testing.assert_close(y.double().cpu(), orc.linear(X, W, Bv), atol=5e-4, rtol=1e-5)

    img, w = torch.randn(1, 3, 224, 224), torch.randn(768, 768)
    y = r.patch_embed(img.to(cuda), w.to(cuda), None)
    torch.testing.assert_close(y.double().cpu(), orc.patch_embed(img, w), atol=1e-4, rtol=1e-5)

    pt, cls, pos = torch.randn(1, 196, 768), torch.randn(1, 768), torch.randn(197, 768)
    y = r.pos_encoding(pt.to(cuda), cls.to(cuda), pos.to(cuda))
    torch.testing.assert_close(y.double().cpu(), orc.pos_encoding(pt, cls, pos), atol=1e-6,
                               rtol=0)

    X, W, b = torch.randn(2, 197, 768), torch.randn(10, 768), torch.randn(10)
    y = r.classifier(X.to(cuda), W.to(cuda), b.to(cuda))
    torch.testing.assert_close(y.double().cpu(), orc.classifier(X, W, b), atol=1e-4, rtol=1e-5)

    X = torch.randn(1, 3, 768)
    W1, B1, W2, B2 = torch.randn(3072, 768), torch.randn(3072), torch.randn(768, 3072), \
        torch.randn(768)
    o, h = r.mlp(X.to(cuda), W1.to(cuda), B1.to(cuda), W2.to(cuda), B2.to(cuda))
    ro, rh = orc.mlp(X, W1, B1, W2, B2)
    torch.testing.assert_close(h.double().cpu(), rh, atol=5e-4, rtol=0)
    torch.testing.assert_close(o.double().cpu(), ro, atol=3e-2, rtol=3e-3)

    q, k, v = (torch.randn(2, 197, 768) for _ in range(3))
    y = r.attention(q.to(cuda), k.to(cuda), v.to(cuda), 0.125)
    # the reference builds with -use_fast_math (__expf): 1e-3, looser than its 1e-4
    torch.testing.assert_close(y.double().cpu(), orc.attention(q, k, v, 0.125), atol=1e-3,
                               rtol=0)


def test_reference_forward_matches_oracle_and_engine(ref, cuda):
    import vit_cuda
    from vit_cuda.weights import synthetic_images, synthetic_state_dict
    state = synthetic_state_dict(seed=0, img_size=224)
    img = synthetic_images(2, 224, seed=0)
    sd = {k: v.to(cuda).contiguous() for k, v in state.items()}
    with torch.no_grad():
        ref_logits = RefOps(ref).forward(img.to(cuda), sd).double().cpu()
        ours = vit_cuda.ViTCUDA(state_dict=sd).to(cuda).eval()(img.to(cuda)).double().cpu()
    oracle = orc.vit_forward(img, state)
    # the reference's own end-to-end bar is 1e-2 against timm (tests/test_end_to_end.py:45)
    assert (ref_logits - oracle).abs().max().item() < 1e-3
    assert (ours - oracle).abs().max().item() < 1e-3
    assert (ours - ref_logits).abs().max().item() < 1e-3
    assert torch.equal(ours.argmax(-1), ref_logits.argmax(-1))
