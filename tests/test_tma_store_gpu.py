"""The GEMM epilogues' TMA tensor stores (fc1's FP16-split H, the QKV
epilogue's q and k splits, an fp32 result replacing its residual) change only
how bytes reach memory, never the arithmetic: the forward's logits and an
in-place residual GEMM are bitwise the same as with every result written by
per-lane stores. The switch (VITB200_TMA_STORE=0) is read once per process, so
the per-lane run happens in a child process on the same inputs."""
import os
import subprocess
import sys
import textwrap

import pytest
import torch

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = textwrap.dedent("""
    import sys, torch
    sys.path.insert(0, {pkg!r}); sys.path.insert(0, {repo!r})
    from tma_store_case import compute
    torch.save(compute(torch.device("cuda", 0)), {out!r})
""")


def _case_module(tmp_path):
    """Writes the shared computation as a module both processes import."""
    src = textwrap.dedent("""
        import torch
        from vit_cuda import _lib
        from vit_cuda.model import ViTCUDA
        from vit_cuda.split import f16_planes, f16_weight
        from vit_cuda.weights import synthetic_images, synthetic_state_dict

        def compute(dev):
            torch.backends.cuda.matmul.allow_tf32 = False
            state = synthetic_state_dict(seed=7, img_size=224, depth=2)
            model = ViTCUDA(state_dict={k: v.to(dev) for k, v in state.items()}).to(dev).eval()
            out = {}
            with torch.no_grad():
                for batch in (1, 8):   # split-K owners at batch 1; CTA-pair tiles at batch 8
                    x = synthetic_images(batch, 224, seed=batch).to(dev)
                    out[f"logits{batch}"] = model(x).cpu()
            # x += W x' + b in place (the residual is the output), FP16 splits
            g = torch.Generator(device=dev).manual_seed(3)
            a = torch.randn(300, 768, device=dev, generator=g)
            w = torch.randn(768, 768, device=dev, generator=g) * 0.03
            b = torch.randn(768, device=dev, generator=g)
            y = torch.randn(300, 768, device=dev, generator=g)
            ap = f16_planes(a, 2)
            wp, acc = f16_weight(w)
            s = torch.cuda.current_stream().cuda_stream
            _lib.check(_lib.lib.vitb200_gemm_f16(ap.data_ptr(), wp.data_ptr(), acc, b.data_ptr(),
                                                 y.data_ptr(), y.data_ptr(), 768, None, 300,
                                                 ap.shape[-1], 768, 3, s), "vitb200_gemm_f16")
            out["resid_inplace"] = y.cpu()
            torch.cuda.synchronize()
            assert _lib.device_error() == 0
            return out
    """)
    (tmp_path / "tma_store_case.py").write_text(src)
    return str(tmp_path)


def test_tma_stores_bitwise_equal_per_lane_stores(cuda, tmp_path):
    case_dir = _case_module(tmp_path)
    sys.path.insert(0, case_dir)
    try:
        from tma_store_case import compute
        ours = compute(cuda)
    finally:
        sys.path.remove(case_dir)
    out = str(tmp_path / "per_lane.pt")
    env = dict(os.environ, VITB200_TMA_STORE="0",
               PYTHONPATH=os.pathsep.join([case_dir, os.environ.get("PYTHONPATH", "")]))
    script = CHILD.format(pkg=os.path.join(REPO, "vit-engine-cuda_b200"), repo=REPO, out=out)
    r = subprocess.run([sys.executable, "-c", script], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    theirs = torch.load(out)
    assert set(ours) == set(theirs)
    for k in ours:
        assert torch.equal(ours[k], theirs[k]), k
