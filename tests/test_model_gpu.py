"""End-to-end parity of the fused ViT-B/16 forward against the CPU oracle.

Bar (north star): logits max-abs <= 1e-3, per-block relative L2 <= 1e-5
(chained and teacher-forced), 100% top-1 agreement, on seeded N(0,1) images and
seeded random-init weights. Also the reference's own end-to-end checks:
batch>1 (tests/test_end_to_end.py:22-45 of the reference project) and CUDA
graph == eager (tests/test_end_to_end.py:48-68).
"""
import numpy as np
import pytest
import torch

from oracle import vit_oracle as orc
from vit_cuda import ViTCUDA
from vit_cuda.weights import synthetic_images, synthetic_state_dict

pytestmark = pytest.mark.gpu

LOGITS_ATOL = 1e-3
BLOCK_REL_L2 = 1e-5


@pytest.fixture(scope="module")
def case224(cuda):
    state = synthetic_state_dict(seed=0, img_size=224)
    img = synthetic_images(2, 224, seed=0)
    logits, inter = orc.vit_forward(img, state, return_intermediates=True)
    model = ViTCUDA(state_dict={k: v.to(cuda) for k, v in state.items()}).to(cuda).eval()
    return state, img, logits, inter, model


def test_logits_match_oracle(case224, cuda):
    _, img, ref, _, model = case224
    with torch.no_grad():
        out = model(img.to(cuda)).double().cpu()
    err = (out - ref).abs().max().item()
    assert err <= LOGITS_ATOL, err
    assert torch.equal(out.argmax(-1), ref.argmax(-1))


def test_batch8_matches_oracle(case224, cuda):
    """The reference's own end-to-end batch (tests/test_end_to_end.py:22-45 uses
    B=8); M = 8*197 rows selects the CTA-pair GEMM tiles."""
    state, _, _, _, model = case224
    img = synthetic_images(8, 224, seed=5)
    ref = orc.vit_forward(img, state)
    with torch.no_grad():
        out = model(img.to(cuda)).double().cpu()
    assert (out - ref).abs().max().item() <= LOGITS_ATOL
    assert torch.equal(out.argmax(-1), ref.argmax(-1))


def test_logits_match_golden(case224, cuda):
    """The committed transformers-generated golden logits (tests/golden)."""
    _, img, _, _, model = case224
    g = np.load(__file__.replace("test_model_gpu.py", "golden/vit_e2e_golden.npz"))
    with torch.no_grad():
        out = model(img.to(cuda)).double().cpu().numpy()
    assert np.abs(out - g["b2_224/logits"]).max() <= LOGITS_ATOL


def test_blocks_chained(case224, cuda):
    """Per-block relative L2 of the fused path run block by block from its own
    embedding (errors accumulate as in the full forward)."""
    _, img, ref_logits, inter, model = case224
    x = model.embed(img.to(cuda))
    assert orc.rel_l2(x.cpu(), inter["embed"]) <= BLOCK_REL_L2
    worst = 0.0
    for i, ref_block in enumerate(inter["blocks"]):
        x = model.block(i, x)
        worst = max(worst, orc.rel_l2(x.cpu(), ref_block))
    assert worst <= BLOCK_REL_L2, worst
    logits, feats = model.head(x)
    assert (logits.double().cpu() - ref_logits).abs().max().item() <= LOGITS_ATOL
    assert (feats.double().cpu() - inter["features"]).abs().max().item() <= LOGITS_ATOL


def test_blocks_teacher_forced(case224, cuda):
    """Each block fed the oracle's input for that block."""
    _, _, _, inter, model = case224
    inputs = [inter["embed"]] + inter["blocks"][:-1]
    for i, (xin, xout) in enumerate(zip(inputs, inter["blocks"])):
        y = model.block(i, xin.float().to(cuda))
        assert orc.rel_l2(y.cpu(), xout) <= BLOCK_REL_L2, i


def test_op_by_op_block_matches_oracle(case224, cuda):
    """The reference's own block surface, ViTBlockCUDA.forward (reference
    vit_cuda/model.py:39-60: the eight registered ops one by one, residual adds
    in PyTorch), against the oracle's block on the same tokens (B=2, T=197):
    every block fed the oracle's input, relative L2 within the per-block bar."""
    _, _, _, inter, model = case224
    inputs = [inter["embed"]] + inter["blocks"][:-1]
    worst = 0.0
    with torch.no_grad():
        for i, (xin, xout) in enumerate(zip(inputs, inter["blocks"])):
            y = model.blocks[i](xin.float().to(cuda), model.scale, model.eps)
            assert y.shape == xin.shape
            worst = max(worst, orc.rel_l2(y.cpu(), xout))
    assert worst <= BLOCK_REL_L2, worst


def test_forward_features(case224, cuda):
    _, img, _, inter, model = case224
    with torch.no_grad():
        f = model.forward_features(img.to(cuda)).double().cpu()
    assert (f - inter["features"]).abs().max().item() <= LOGITS_ATOL


def test_batch_rows_differ(case224, cuda):
    """Batch > 1 must not collapse rows (the reference's Phase-5 bug class,
    scratch/repro_bug.py:20-27). Small batches split K by how many SMs their
    tile grids fill, so batch-1 rows match the batch-4 rows to FP32 rounding;
    with split-K off they match bitwise (batch invariance)."""
    import vit_cuda
    _, _, _, _, model = case224
    x = synthetic_images(4, 224, seed=7).to(cuda)
    with torch.no_grad():
        out = model(x)
        single = torch.cat([model(x[i:i + 1]) for i in range(4)])
        old = vit_cuda.set_split_k(False)
        try:
            out_unsplit = model(x)
            single_unsplit = torch.cat([model(x[i:i + 1]) for i in range(4)])
        finally:
            vit_cuda.set_split_k(old)
    assert not torch.allclose(out[0], out[1])
    torch.testing.assert_close(out, single, atol=1e-5, rtol=0)
    torch.testing.assert_close(out, out_unsplit, atol=1e-5, rtol=0)
    torch.testing.assert_close(out_unsplit, single_unsplit, atol=0, rtol=0)


def test_batch1_split_k_matches_oracle(case224, cuda):
    """Batch 1 (every block GEMM split over K) against the oracle; split-K
    sums partials in a fixed order, so repeated forwards agree bitwise."""
    state, img, ref, _, model = case224
    x = img[:1].to(cuda)
    with torch.no_grad():
        a = model(x).clone()
        b = model(x)
    assert (a.double().cpu() - ref[:1]).abs().max().item() <= LOGITS_ATOL
    assert torch.equal(a.argmax(-1).cpu(), ref[:1].argmax(-1))
    torch.testing.assert_close(a, b, atol=0, rtol=0)


def test_concurrent_streams_match_serial(case224, cuda):
    """Batch-1 forwards on two streams at once (split-K clusters of both in
    flight together) give the serial results bitwise."""
    _, _, _, _, model = case224
    xs = [synthetic_images(1, 224, seed=30 + i).to(cuda) for i in range(2)]
    with torch.no_grad():
        serial = [model(x).clone() for x in xs]
        streams = [torch.cuda.Stream(cuda) for _ in xs]
        torch.cuda.synchronize(cuda)
        outs = [[], []]
        for _ in range(4):
            for k, (s, x) in enumerate(zip(streams, xs)):
                with torch.cuda.stream(s):
                    outs[k].append(model(x))
        torch.cuda.synchronize(cuda)
    for k in range(2):
        for o in outs[k]:
            torch.testing.assert_close(o, serial[k], atol=0, rtol=0)


def test_graph_matches_eager(cuda):
    state = synthetic_state_dict(seed=1, img_size=224)
    torch.manual_seed(1)
    x = torch.randn(4, 3, 224, 224, device=cuda)
    model = ViTCUDA(state_dict={k: v.to(cuda) for k, v in state.items()}).to(cuda).eval()
    with torch.no_grad():
        eager = model(x).clone()
    model.capture_graph(x, num_warmup=3)
    with torch.no_grad():
        graph = model(x)
    torch.testing.assert_close(graph, eager, atol=0, rtol=0)
    x2 = torch.randn(4, 3, 224, 224, device=cuda)
    with torch.no_grad():
        g2 = model(x2).clone()
    model.release_graph()
    with torch.no_grad():
        e2 = model(x2)
    torch.testing.assert_close(g2, e2, atol=0, rtol=0)


def test_384_tokens577(case384, cuda):
    """384x384 input, T = 577 (the reference's kernels hardcode 224/197)."""
    _, img, ref, _, model = case384
    with torch.no_grad():
        out = model(img.to(cuda)).double().cpu()
    assert (out - ref).abs().max().item() <= LOGITS_ATOL
    assert torch.equal(out.argmax(-1), ref.argmax(-1))


@pytest.fixture(scope="module")
def case384(cuda):
    state = synthetic_state_dict(seed=1, img_size=384)
    img = synthetic_images(1, 384, seed=1)
    logits, inter = orc.vit_forward(img, state, return_intermediates=True)
    model = ViTCUDA(state_dict={k: v.to(cuda) for k, v in state.items()}).to(cuda).eval()
    return state, img, logits, inter, model


def test_384_blocks_chained_and_teacher_forced(case384, cuda):
    """384x384, T = 577 (five query tiles, ten key tiles): per-block relative
    L2 of the fused path, run block by block from its own embedding (chained)
    and with each block fed the oracle's input (teacher-forced)."""
    _, img, ref_logits, inter, model = case384
    x = model.embed(img.to(cuda))
    assert orc.rel_l2(x.cpu(), inter["embed"]) <= BLOCK_REL_L2
    chained = 0.0
    for i, ref_block in enumerate(inter["blocks"]):
        x = model.block(i, x)
        chained = max(chained, orc.rel_l2(x.cpu(), ref_block))
    assert chained <= BLOCK_REL_L2, chained
    logits, _ = model.head(x)
    assert (logits.double().cpu() - ref_logits).abs().max().item() <= LOGITS_ATOL
    inputs = [inter["embed"]] + inter["blocks"][:-1]
    forced = 0.0
    for i, (xin, xout) in enumerate(zip(inputs, inter["blocks"])):
        forced = max(forced, orc.rel_l2(model.block(i, xin.float().to(cuda)).cpu(), xout))
    assert forced <= BLOCK_REL_L2, forced


def test_cfg5_shard_batch512_384(case384, cuda):
    """BASELINE configs[4]'s per-GPU shard: 512 images at 384x384 (T = 577,
    295,424 token rows) in one forward. Three images of the batch (first,
    middle, last) against the oracle; the same images alone in a batch of 7
    give bitwise the same logits (the per-image arithmetic does not depend on
    the batch from 7 images up), so every shard of the 4096-image batch
    computes what one GPU would."""
    state, _, _, _, model = case384
    x = synthetic_images(512, 384, seed=4096)
    rows = [0, 255, 511]
    with torch.no_grad():
        out = model(x.to(cuda)).double().cpu()
        small = model(x[rows + [1, 2, 3, 4]].to(cuda)).double().cpu()
    assert out.shape == (512, 1000) and torch.isfinite(out).all()
    torch.testing.assert_close(out[rows], small[:3], atol=0, rtol=0)
    ref = orc.vit_forward(x[rows], state)
    assert (out[rows] - ref).abs().max().item() <= LOGITS_ATOL
    assert torch.equal(out[rows].argmax(-1), ref.argmax(-1))


def test_operand_choice(case224, cuda):
    """Random-init ViT-B/16 weights bound every block GEMM input far below the
    FP16 split's range, so all 48 GEMMs and the 12 attentions run on FP16
    splits by default."""
    _, _, _, _, model = case224
    model.prepare()
    assert model.patch_operands == "f16"
    assert len(model.gemm_operands) == 12
    assert all(k == "f16" for blk in model.gemm_operands for k in blk.values())


def test_tf32_operands_match_oracle(case224, cuda):
    state, img, ref, _, _ = case224
    model = ViTCUDA(state_dict={k: v.to(cuda) for k, v in state.items()},
                    operands="tf32").to(cuda).eval()
    model.prepare()
    assert model.patch_operands == "tf32"
    assert all(k == "tf32" for blk in model.gemm_operands for k in blk.values())
    with torch.no_grad():
        out = model(img.to(cuda)).double().cpu()
    assert (out - ref).abs().max().item() <= LOGITS_ATOL
    assert torch.equal(out.argmax(-1), ref.argmax(-1))


def test_out_of_range_block_falls_back_to_tf32(cuda):
    """A LayerNorm gain large enough that the fc1 / fc2 inputs could leave the
    FP16 split's range moves those GEMMs (only) onto TF32 pairs; results still
    match the oracle."""
    state = synthetic_state_dict(seed=2, img_size=224)
    state["blocks.11.norm2.weight"] = state["blocks.11.norm2.weight"] * 3000.0
    img = synthetic_images(2, 224, seed=2)
    ref = orc.vit_forward(img, state)
    model = ViTCUDA(state_dict={k: v.to(cuda) for k, v in state.items()}).to(cuda).eval()
    model.prepare()
    assert model.gemm_operands[11] == {"qkv": "f16", "proj": "f16", "fc1": "tf32", "fc2": "tf32",
                                       "attn": "f16"}
    assert all(k == "f16" for blk in model.gemm_operands[:11] for k in blk.values())
    with torch.no_grad():
        out = model(img.to(cuda)).double().cpu()
    assert (out - ref).abs().max().item() <= LOGITS_ATOL * max(1.0, ref.abs().max().item())
    assert torch.equal(out.argmax(-1), ref.argmax(-1))


def test_streamed_inference_matches_eager(cuda):
    """Host-resident batches through vit_cuda.StreamedInference (copy of batch
    i+1 overlapping the forward of batch i) give the eager logits bitwise."""
    import vit_cuda
    state = synthetic_state_dict(seed=3, img_size=224)
    model = ViTCUDA(state_dict={k: v.to(cuda) for k, v in state.items()}).to(cuda).eval()
    batches = [synthetic_images(3, 224, seed=20 + i).pin_memory() for i in range(5)]
    run = vit_cuda.StreamedInference(model, (3, 3, 224, 224))
    outs = [run(x) for x in batches]
    torch.cuda.current_stream().synchronize()
    with torch.no_grad():
        for x, o in zip(batches, outs):
            torch.testing.assert_close(o, model(x.to(cuda)).cpu(), atol=0, rtol=0)


def test_streamed_inference_host_buffer_reuse(cuda):
    """One pinned host buffer refilled between calls: after waiting on
    input_copied() the buffer may be overwritten, and each call's logits are
    those of the images it held when it was called."""
    import vit_cuda
    state = synthetic_state_dict(seed=3, img_size=224)
    model = ViTCUDA(state_dict={k: v.to(cuda) for k, v in state.items()}).to(cuda).eval()
    batches = [synthetic_images(2, 224, seed=60 + i) for i in range(4)]
    host = torch.empty(2, 3, 224, 224).pin_memory()
    run = vit_cuda.StreamedInference(model, (2, 3, 224, 224))
    assert run.input_copied() is None
    outs = []
    for b in batches:
        host.copy_(b)
        outs.append(run(host, torch.empty(2, 1000).pin_memory()))
        run.input_copied().synchronize()
    torch.cuda.current_stream().synchronize()
    with torch.no_grad():
        for b, o in zip(batches, outs):
            torch.testing.assert_close(o, model(b.to(cuda)).cpu(), atol=0, rtol=0)


def test_batch_invariance_from_seven_images(case224, cuda):
    """From 7 images up (224²) every kernel's per-image arithmetic is the same
    whatever the batch (CTA-pair GEMM tiles from 1024 token rows, the two-tile
    attention, the fused final LayerNorm + head), so an image's logits are
    bitwise the same alone in a batch of 7 and inside a batch of 16; they match
    the oracle."""
    state, _, _, _, model = case224
    x = synthetic_images(16, 224, seed=11)
    with torch.no_grad():
        big = model(x.to(cuda)).double().cpu()
        small = model(x[:7].to(cuda)).double().cpu()
    torch.testing.assert_close(big[:7], small, atol=0, rtol=0)
    ref = orc.vit_forward(x[:2], state)
    assert (small[:2] - ref).abs().max().item() <= LOGITS_ATOL


def test_concurrent_host_threads_match_serial(case224, cuda):
    """Two host threads call the forward at once, each on its own stream (ctypes
    releases the GIL, so the library is entered concurrently): results equal
    the serial ones bitwise."""
    import threading
    _, _, _, _, model = case224
    xs = [synthetic_images(1, 224, seed=40 + i).to(cuda) for i in range(2)]
    with torch.no_grad():
        serial = [model(x).clone() for x in xs]
    outs = [[], []]
    errors = []

    def worker(k):
        try:
            torch.cuda.set_device(cuda)
            s = torch.cuda.Stream(cuda)
            with torch.no_grad(), torch.cuda.stream(s):
                for _ in range(5):
                    outs[k].append(model(xs[k]))
            s.synchronize()
        except Exception as e:  # reported below
            errors.append(e)

    threads = [threading.Thread(target=worker, args=(k,)) for k in range(2)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    assert not errors, errors
    for k in range(2):
        assert len(outs[k]) == 5
        for o in outs[k]:
            torch.testing.assert_close(o, serial[k], atol=0, rtol=0)


@pytest.mark.parametrize("num_classes,batch", [(10, 3), (7, 9), (1, 1)])
def test_odd_class_counts(cuda, num_classes, batch):
    """The fused final LayerNorm + head with class counts that leave a block's
    warps idle (8 classes and 8 images per block) and batches past one block of
    images; logits and features against the oracle."""
    state = synthetic_state_dict(seed=12, img_size=224, depth=1, num_classes=num_classes)
    img = synthetic_images(batch, 224, seed=12)
    ref, inter = orc.vit_forward(img, state, return_intermediates=True)
    model = ViTCUDA(num_classes=num_classes,
                    state_dict={k: v.to(cuda) for k, v in state.items()}).to(cuda).eval()
    with torch.no_grad():
        out = model(img.to(cuda)).double().cpu()
        feats = model.forward_features(img.to(cuda)).double().cpu()
        x = model.block(0, model.embed(img.to(cuda)))
        logits, hfeats = model.head(x)
    assert out.shape == (batch, num_classes)
    assert (out - ref).abs().max().item() <= LOGITS_ATOL
    assert (feats - inter["features"]).abs().max().item() <= LOGITS_ATOL
    torch.testing.assert_close(logits.double().cpu(), out, atol=0, rtol=0)
    # forward_features runs the LayerNorm kernel, head() the fused one (same row routine)
    torch.testing.assert_close(hfeats.double().cpu(), feats, atol=1e-6, rtol=0)


def test_trained_like_weights(cuda):
    """Weights with trained-like statistics (LayerNorm gains spread to 5-10,
    twice-wider weights with heavy rows, larger positional embeddings): the
    worst-case input bounds stay inside the FP16 split's range (block 11's
    largest, the attention's v, is ~1.4e4 against 3.3e4), so every block GEMM
    and attention keeps the FP16 path, and the forward still meets the parity
    bar, block by block and on the logits."""
    from vit_cuda.split import F16_SAFE_BOUND, block_input_bounds
    state = synthetic_state_dict(seed=0, img_size=224, stats="trained")
    img = synthetic_images(2, 224, seed=0)
    ref, inter = orc.vit_forward(img, state, return_intermediates=True)
    model = ViTCUDA(state_dict={k: v.to(cuda) for k, v in state.items()}).to(cuda).eval()
    model.prepare()
    worst = max(max(block_input_bounds(b, 768).values()) for b in model.blocks)
    assert worst < F16_SAFE_BOUND
    assert all(k == "f16" for blk in model.gemm_operands for k in blk.values())
    x = model.embed(img.to(cuda))
    chained = 0.0
    for i, ref_block in enumerate(inter["blocks"]):
        x = model.block(i, x)
        chained = max(chained, orc.rel_l2(x.cpu(), ref_block))
    assert chained <= BLOCK_REL_L2, chained
    with torch.no_grad():
        out = model(img.to(cuda)).double().cpu()
    assert (out - ref).abs().max().item() <= LOGITS_ATOL * max(1.0, ref.abs().max().item())
    assert torch.equal(out.argmax(-1), ref.argmax(-1))


def test_out_of_range_pixel_reported(case224, cuda):
    """The patch GEMM runs on FP16 splits of the pixels, which must stay below
    32768 in magnitude: a pixel beyond that is reported through the device
    error word (code 6) rather than producing silent garbage; with
    operands="tf32" the same image runs on TF32 pairs and matches the oracle."""
    import vit_cuda
    state, _, _, _, model = case224
    img = synthetic_images(1, 224, seed=9)
    img[0, 1, 100, 37] = 40000.0
    with torch.no_grad():
        model(img.to(cuda))
    assert vit_cuda.device_error(clear=True) == 6
    m32 = ViTCUDA(state_dict={k: v.to(cuda) for k, v in state.items()},
                  operands="tf32").to(cuda).eval()
    with torch.no_grad():
        out = m32(img.to(cuda)).double().cpu()
    assert vit_cuda.device_error(clear=True) == 0
    ref = orc.vit_forward(img, state)
    assert (out - ref).abs().max().item() <= LOGITS_ATOL * max(1.0, ref.abs().max().item())


def test_nan_pixel_reported(case224, cuda):
    """A NaN pixel among finite ones is reported like an out-of-range one
    (code 6): the range check does not rely on fmaxf, which drops NaN."""
    import vit_cuda
    _, _, _, _, model = case224
    img = synthetic_images(1, 224, seed=10)
    img[0, 2, 17, 201] = float("nan")
    with torch.no_grad():
        model(img.to(cuda))
    assert vit_cuda.device_error(clear=True) == 6


def test_folded_layernorm_matches_unfolded_and_oracle(case224, cuda):
    """Below 1024 token rows the LayerNorms before qkv and fc1 run inside those
    GEMMs (vitb200_vit_params.ln_fold): the GEMM multiplies the FP16 split of x
    by W * diag(gamma) and applies rstd * (acc - mean * c) + d with the row
    statistics the previous residual GEMM wrote. Both forms meet the parity
    bars per block (chained) and on the logits, and they differ (the fold ran)
    only at FP32 rounding level. (test_blocks_chained / _teacher_forced check
    the folded path per block: the model folds at this batch.)"""
    state, img, ref, inter, model = case224
    assert model.ln_folded
    plain = ViTCUDA(state_dict={k: v.to(cuda) for k, v in state.items()},
                    ln_fold=False).to(cuda).eval()
    assert not plain.ln_folded
    with torch.no_grad():
        a = model(img.to(cuda)).double().cpu()
        b = plain(img.to(cuda)).double().cpu()
    for out in (a, b):
        assert (out - ref).abs().max().item() <= LOGITS_ATOL
        assert torch.equal(out.argmax(-1), ref.argmax(-1))
    assert not torch.equal(a, b)
    assert (a - b).abs().max().item() <= 1e-4
    x = plain.embed(img.to(cuda))
    for i, ref_block in enumerate(inter["blocks"]):
        x = plain.block(i, x)
        assert orc.rel_l2(x.cpu(), ref_block) <= BLOCK_REL_L2, i


def test_folded_layernorm_range_reported(cuda):
    """With the LayerNorms folded, the GEMMs read the FP16 split of the
    residual stream itself, which must stay below 32768 in magnitude: a
    residual stream past that (patch weights scaled by 2^20) is reported
    through the device error word (code 6); unfolded, the same model runs and
    matches the oracle."""
    import vit_cuda
    state = synthetic_state_dict(seed=3, img_size=224, depth=2)
    state["patch_embed.proj.weight"] = state["patch_embed.proj.weight"] * 2.0 ** 20
    img = synthetic_images(1, 224, seed=4)
    dev_state = {k: v.to(cuda) for k, v in state.items()}
    folded = ViTCUDA(state_dict=dev_state).to(cuda).eval()
    assert folded.ln_folded
    with torch.no_grad():
        folded(img.to(cuda))
    assert vit_cuda.device_error(clear=True) == 6
    plain = ViTCUDA(state_dict=dev_state, ln_fold=False).to(cuda).eval()
    with torch.no_grad():
        out = plain(img.to(cuda)).double().cpu()
    assert vit_cuda.device_error(clear=True) == 0
    ref = orc.vit_forward(img, state)
    assert (out - ref).abs().max().item() <= LOGITS_ATOL * max(1.0, ref.abs().max().item())


def test_folded_layernorm_with_tf32_attention(cuda):
    """Folded LayerNorms with one block's attention on TF32 pairs: its q rows of
    the qkv weight scaled by 2^12 take q's bound past the FP16 split's range
    (attention -> TF32) while every GEMM input stays inside it (all four GEMMs
    FP16, so the fold applies). Batch 1 (below 1024 token rows) against the
    oracle."""
    state = synthetic_state_dict(seed=6, img_size=224, depth=3)
    w = state["blocks.1.attn.qkv.weight"].clone()
    w[:768] *= 2.0 ** 12
    state["blocks.1.attn.qkv.weight"] = w
    img = synthetic_images(1, 224, seed=6)
    ref = orc.vit_forward(img, state)
    model = ViTCUDA(state_dict={k: v.to(cuda) for k, v in state.items()}).to(cuda).eval()
    model.prepare()
    assert model.gemm_operands[1] == {"qkv": "f16", "proj": "f16", "fc1": "f16", "fc2": "f16",
                                      "attn": "tf32"}
    assert model.ln_folded
    with torch.no_grad():
        out = model(img.to(cuda)).double().cpu()
    assert (out - ref).abs().max().item() <= LOGITS_ATOL * max(1.0, ref.abs().max().item())
    assert torch.equal(out.argmax(-1), ref.argmax(-1))
