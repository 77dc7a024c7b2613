"""Failure reporting without a GPU fault: every wait in the library's kernels is
bounded (1 s of %globaltimer); a wait that runs out records a code in the
device error word, the kernel returns, and the context stays usable. Here a
wait that nothing satisfies runs out on purpose (a fresh mbarrier nobody
arrives on), through the same bounded-wait helpers the GEMM, attention and
split-K kernels use."""
import time

import pytest
import torch

from test_gemm_gpu import check_fp32_parity, run_gemm

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind,code", [(0, 1), (1, 7)])
def test_bounded_wait_reports_and_returns(vlib, cuda, kind, code):
    assert vlib.device_error(clear=True) == 0
    t0 = time.perf_counter()
    vlib.check(vlib.lib.vitb200_check_wait_timeout(kind, torch.cuda.current_stream().cuda_stream),
               "vitb200_check_wait_timeout")
    assert vlib.device_error(clear=True) == code
    assert 0.9 < time.perf_counter() - t0 < 30.0
    # the context still computes correctly (a split-K launch and an unsplit one)
    torch.manual_seed(9)
    for m in (197, 2048):
        x = torch.randn(m, 768, device=cuda)
        w = torch.randn(768, 768, device=cuda) * 0.05
        b = torch.randn(768, device=cuda)
        check_fp32_parity(run_gemm(vlib, x, w, b, None, "bias"), x, w, b, None, "bias")
    assert vlib.device_error(clear=True) == 0


def test_bad_kind_rejected(vlib, cuda):
    assert vlib.lib.vitb200_check_wait_timeout(2, None) != 0
