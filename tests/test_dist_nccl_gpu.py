"""Data parallelism on two GPUs over NCCL (vit_cuda/parallel.py): each rank
runs its slice of the batch through the fused forward and one all-gather
assembles the logits. With at least 7 images per rank every kernel's
per-image arithmetic matches the single-GPU run of the whole batch, so the
gathered logits equal it bit for bit; an uneven split (15 images: 8 + 7)
included. Skipped with fewer than two GPUs. The process group has a short
timeout, and the parent kills any child still alive after its join."""
import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, batch, queue):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60), device_id=dev)
        from vit_cuda import ViTCUDA
        from vit_cuda.parallel import DataParallelViT
        from vit_cuda.weights import synthetic_images, synthetic_state_dict
        state = synthetic_state_dict(seed=5, img_size=224, depth=2)
        model = ViTCUDA(state_dict={k: v.to(dev) for k, v in state.items()}).to(dev).eval()
        x = synthetic_images(batch, 224, seed=6).to(dev)
        with torch.no_grad():
            gathered = DataParallelViT(model)(x)
            torch.cuda.synchronize()
            single = model(x) if rank == 0 else None
        dist.barrier()
        dist.destroy_process_group()
        if rank == 0:  # numpy: pickled by value (the child exits after this)
            queue.put((rank, "ok", (gathered.cpu().numpy(), single.cpu().numpy())))
        else:
            queue.put((rank, "ok", None))
    except Exception as e:  # reported to the parent
        queue.put((rank, "error", f"{type(e).__name__}: {e}\n{traceback.format_exc()[-600:]}"))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("batch", [16, 15])
def test_two_gpu_gather_equals_single_gpu(batch):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, batch, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(2):
            rank, status, payload = q.get(timeout=300)
            results[rank] = (status, payload)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(2):
        assert results[r][0] == "ok", results[r][1]
    gathered, single = (torch.from_numpy(a) for a in results[0][1])
    assert gathered.shape == (batch, 1000)
    torch.testing.assert_close(gathered, single, atol=0, rtol=0)
