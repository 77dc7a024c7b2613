"""torch.library registration: torch.library.opcheck on each registered op
(schema, fake implementation, dispatch), and torch.compile(fullgraph=True)
tracing the reference's op-by-op block and the fused model without graph
breaks (the reference's tests/torch_compile_test.py:106-114 studies those
breaks), with results equal to eager."""
import pytest
import torch

import vit_cuda
from vit_cuda.weights import synthetic_state_dict

pytestmark = pytest.mark.gpu


def test_opcheck_all_ops(cuda):
    torch.manual_seed(0)
    x = torch.randn(2, 5, 768, device=cuda)
    w, b = torch.randn(768, 768, device=cuda) * 0.02, torch.randn(768, device=cuda)
    img = torch.randn(2, 3, 32, 48, device=cuda)
    ops = torch.ops.vit_cuda
    cases = [
        (ops.flash_attn_2, (x, x, x, 0.125)),
        (ops.patch_embed, (img, w, b)),
        (ops.pos_encoding, (torch.randn(2, 6, 768, device=cuda), torch.randn(2, 768, device=cuda),
                            torch.randn(7, 768, device=cuda))),
        (ops.mlp_forward, (x, torch.randn(3072, 768, device=cuda) * 0.02,
                           torch.randn(3072, device=cuda), torch.randn(768, 3072, device=cuda) * 0.02,
                           b)),
        (ops.layernorm_forward, (x, torch.ones(768, device=cuda), b, 1e-6)),
        (ops.classifier_forward, (x, torch.randn(10, 768, device=cuda), torch.randn(10, device=cuda))),
        (ops.qkv_proj_packed, (x, torch.randn(2304, 768, device=cuda) * 0.02,
                               torch.randn(2304, device=cuda))),
        (ops.gemm_bias, (x, w, b)),
    ]
    for op, args in cases:
        torch.library.opcheck(op, args, test_utils=("test_schema", "test_faketensor"))


def test_compile_block_fullgraph(cuda):
    """The op-by-op block (registered ops) compiles as one graph."""
    torch._dynamo.reset()
    state = synthetic_state_dict(seed=0, img_size=224, depth=1)
    model = vit_cuda.ViTCUDA(state_dict={k: v.to(cuda) for k, v in state.items()}).to(cuda).eval()
    blk = model.blocks[0]
    x = torch.randn(2, 197, 768, device=cuda)
    eager = blk(x, model.scale, model.eps)
    compiled = torch.compile(lambda t: blk(t, model.scale, model.eps), fullgraph=True)
    torch.testing.assert_close(compiled(x), eager, atol=0, rtol=0)


def test_compile_model_fullgraph(cuda):
    """ViTCUDA under torch.compile(fullgraph=True): one registered op, the
    same kernels, bitwise-equal logits."""
    torch._dynamo.reset()
    state = synthetic_state_dict(seed=1, img_size=224)
    model = vit_cuda.ViTCUDA(state_dict={k: v.to(cuda) for k, v in state.items()}).to(cuda).eval()
    x = torch.randn(3, 3, 224, 224, device=cuda)
    with torch.no_grad():
        eager = model(x)
        compiled = torch.compile(model, fullgraph=True)(x)
    torch.testing.assert_close(compiled, eager, atol=0, rtol=0)


def test_split_weights_save_and_load(cuda, tmp_path):
    """Offline pre-split weights (vit_cuda.checkpoint.save_splits /
    load_splits) reproduce the forward bitwise and are refused for other
    weights."""
    from vit_cuda import checkpoint
    state = synthetic_state_dict(seed=6, img_size=224)
    a = vit_cuda.ViTCUDA(state_dict={k: v.to(cuda) for k, v in state.items()}).to(cuda).eval()
    x = torch.randn(2, 3, 224, 224, device=cuda)
    with torch.no_grad():
        ref = a(x)
    path = str(tmp_path / "splits.safetensors")
    checkpoint.save_splits(a, path)
    b = vit_cuda.ViTCUDA(state_dict={k: v.to(cuda) for k, v in state.items()}).to(cuda).eval()
    checkpoint.load_splits(b, path)
    assert b.gemm_operands == a.gemm_operands
    with torch.no_grad():
        torch.testing.assert_close(b(x), ref, atol=0, rtol=0)
    other = dict(state)
    other["blocks.0.mlp.fc1.weight"] = other["blocks.0.mlp.fc1.weight"] * 2
    c = vit_cuda.ViTCUDA(state_dict={k: v.to(cuda) for k, v in other.items()}).to(cuda).eval()
    with pytest.raises(ValueError, match="fingerprint"):
        checkpoint.load_splits(c, path)


def test_load_model_from_hf_checkpoint(cuda, tmp_path):
    """A HuggingFace-format checkpoint file -> ViTCUDA logits equal to the
    same weights given as a timm state dict."""
    import os
    import sys
    from safetensors.torch import save_file
    from vit_cuda import checkpoint
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
    from make_golden import hf_model
    state = synthetic_state_dict(seed=7, img_size=224)
    save_file({k: v.float().contiguous() for k, v in hf_model(state, 224).state_dict().items()},
              str(tmp_path / "hf.safetensors"))
    m = checkpoint.load_model(str(tmp_path / "hf.safetensors"), device=cuda)
    ref = vit_cuda.ViTCUDA(state_dict={k: v.to(cuda) for k, v in state.items()}).to(cuda).eval()
    x = torch.randn(2, 3, 224, 224, device=cuda)
    with torch.no_grad():
        torch.testing.assert_close(m(x), ref(x), atol=0, rtol=0)
