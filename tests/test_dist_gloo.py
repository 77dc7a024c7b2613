"""Data-parallel sharding and the logits all-gather (vit_cuda/parallel.py) on two
CPU processes with the gloo backend: the gathered logits must equal a single
process's, for even and uneven batches, and a rank that fails before the
collective must make the other rank's collective fail (not hang)."""
import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import vit_oracle
from vit_cuda.parallel import DataParallelViT, gather_rows, shard_bounds
from vit_cuda.weights import synthetic_images, synthetic_state_dict


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tiny_model():
    state = synthetic_state_dict(seed=4, img_size=32, depth=1, num_classes=7)
    return lambda x: vit_oracle.vit_forward(x, state, dtype=torch.float64)


def _worker(rank, world, port, batch, mode, queue):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=timedelta(seconds=20))
        torch.set_num_threads(1)
        if mode == "fail" and rank == 1:
            raise RuntimeError("injected failure on rank 1 before the all-gather")
        images = synthetic_images(batch, 32, seed=9)
        out = DataParallelViT(_tiny_model())(images)
        queue.put((rank, "ok", out.numpy()))  # pickled by value
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent, which decides
        queue.put((rank, "error", f"{type(e).__name__}: {e}\n{traceback.format_exc()[-400:]}"))


def _run(world, batch, mode="normal"):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, batch, mode, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, status, payload = q.get(timeout=120)
        results[rank] = (status, payload)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


@pytest.mark.parametrize("batch", [4, 5])
def test_gather_equals_single_process(batch):
    images = synthetic_images(batch, 32, seed=9)
    expected = _tiny_model()(images)
    res = _run(2, batch)
    for rank in range(2):
        status, out = res[rank]
        assert status == "ok", out
        # the CPU stand-in model's BLAS blocking depends on the slice size, so
        # compare at float64 round-off (the GPU engine is bitwise, tested on GPU)
        torch.testing.assert_close(torch.from_numpy(out), expected, atol=1e-12, rtol=1e-12)


def test_failed_rank_surfaces_as_error():
    res = _run(2, 4, mode="fail")
    assert res[1][0] == "error" and "injected" in res[1][1]
    assert res[0][0] == "error", "rank 0 should see its collective fail, not hang"


def test_gather_rows_single_process_is_identity():
    x = torch.randn(3, 5)
    assert gather_rows(x, 3) is x
    assert shard_bounds(7, 3, 2) == (5, 7)
