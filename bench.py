#!/usr/bin/env python
"""ViT-B/16 FP32-parity inference benchmark (images/sec @ bs256 per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...    (N > 1)

A step is one forward of `batch` images per GPU (224x224 default: T=197) with
seeded N(0,1) inputs and seeded random-init ViT-B/16 weights (synthetic data,
no checkpoints offline). Weak scaling: every rank runs its own batch; for N > 1
the logits are all-gathered with NCCL inside the step. Rank 0 prints one JSON
line.

  value     images/s over all ranks, inputs resident in HBM, CUDA events, max
            over ranks. Inputs (154 MB/GPU at bs256) exceed L2 (126 MB).
  e2e       the same through the public API (vit_cuda.StreamedInference over
            ViTCUDA) with every step's images copied host(pinned)->device and its
            logits read back to pinned host memory inside the timed region; the
            copy of step i+1 runs on a copy stream during the forward of step i.
  roofline  the fc1 GEMM of this workload (FP16-split operands, bias + GELU,
            FP16-split output: the model's fc1 launch) timed alone with CUDA
            events on its stream; achieved = FP16 tensor-pipe FLOP/s
            (3 x 2MNK / t) against the measured dense bf16/fp16 peak
            (MEASURED_PEAKS.json, burst: the kernel is timed alone).
  tf32x3    the same forward with every GEMM on TF32 pairs (TF32x3), the
            north star's formulation, for comparison.
  cpu_baseline  the CPU oracle (a PyTorch fp32 restatement of the reference
            path) on the host cores, rank 0 at N=1, on a bounded sample.

--impl reference times the reference path's CPU implementation (the oracle
port; the reference project itself has no CPU path and its timm dependency is
absent) on the same config and prints the same line with "impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "vit-engine-cuda_b200")
for _p in (PKG, REPO):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "ViT-B/16 images/sec @bs256 on 1/2/4/8 B200 (FP32 parity)"
UNIT = "images/s"
CONFIGS = {
    # name: (images per GPU per step, image size)
    "bs256_224": (256, 224),   # bs256 on one B200
    "bs512_384": (512, 384),   # BASELINE configs[4] per-GPU shard (B=4096 over 8 GPUs)
    "bs1_224": (1, 224),       # BASELINE configs[0] shape (batch-1 latency studies)
}
GFLOP_PER_IMG = {224: 35.1277, 384: 110.9687}
# Block GEMMs as the model launches them: (N, K, epilogue, FP16-split output).
ROOFLINE_GEMMS = {"qkv": (2304, 768, "bias", False), "proj": (768, 768, "resid", False),
                  "fc1": (3072, 768, "gelu", True), "fc2": (768, 3072, "resid", False)}
SMI_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="bs256_224")
    ap.add_argument("--cpu-sample", type=int, default=2, help="images per CPU sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-p50", action="store_true")
    ap.add_argument("--cpu-p50-runs", type=int, default=20,
                    help="single-image CPU oracle forwards behind the CPU p50 latency")
    ap.add_argument("--mode", choices=["full", "roofline", "peaks", "forward"], default="full",
                    help="roofline: time only the dominant GEMM launch (for ncu captures); "
                         "peaks: measure cuBLAS TF32 / bf16 / fp16 GEMM throughput; "
                         "forward: only model forwards of --batch images (for profilers)")
    ap.add_argument("--batch", type=int, default=None, help="override images per GPU")
    ap.add_argument("--weights", choices=["init", "trained"], default="init",
                    help="synthetic weight statistics: timm's initialisation (default) or "
                         "trained-like (wider LayerNorm gains, heavier weight rows)")
    ap.add_argument("--kernel", choices=sorted(ROOFLINE_GEMMS) + ["attention", "attention_tf32",
                                                                 "patch"], default="fc1",
                    help="roofline mode: which block GEMM (FP16 splits), the FP16-split "
                         "attention, or the per-op TF32x3 attention / patch GEMM to time")
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def emit(obj):
    print(json.dumps(obj), flush=True)


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples every 50 ms, read on a thread with their arrival
    times; ``start()`` waits for the first sample (the tool takes a moment to
    come up) and marks the timed region's start, ``stop()`` its end, and only
    samples inside the region count."""

    def __init__(self, device_index: int):
        self.proc = None
        self.samples = []  # (monotonic time, fields)
        self.t0 = self.t1 = None
        self.first = threading.Event()
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={SMI_FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(device_index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return
        self.reader = threading.Thread(target=self._read, daemon=True)
        self.reader.start()

    def _read(self):
        for ln in self.proc.stdout:
            if ln.strip():
                self.samples.append((time.monotonic(), [c.strip() for c in ln.split(",")]))
                self.first.set()

    def start(self):
        if self.proc is not None:
            self.first.wait(timeout=15)
        self.t0 = time.monotonic()

    def stop(self):
        self.t1 = time.monotonic()
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"],
                    "samples": 0}
        time.sleep(0.1)  # the sample taken at the region's end
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            self.proc.wait()
        self.reader.join(timeout=5)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for t, r in list(self.samples):
            if len(r) < 9 or not (self.t0 <= t <= self.t1 + 0.06):
                continue
            try:
                sm.append(float(r[1]))
                smax = float(r[2])
            except ValueError:
                continue
            for name, val in zip(names, r[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------- helpers
def max_over_ranks(v: float, world: int, dev) -> float:
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        dist.barrier()


L2_BYTES = 126 * 1024 * 1024


def timed(fn, steps, world, dev, flush=None):
    """CUDA-event time of `steps` calls of fn on the current stream, bracketed by
    a barrier and a synchronize on both sides; max over ranks (ms). With
    `flush` (a device buffer larger than L2), L2 is flushed by writing it
    before every step, outside the timed intervals: each step then has its own
    pair of events and the step times are summed (a synchronize after each
    flush keeps copies issued on other streams inside their step's interval)."""
    stream = torch.cuda.current_stream()
    barrier(world)
    torch.cuda.synchronize()
    if flush is None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        total = e0.elapsed_time(e1)
    else:
        events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(steps)]
        for e0, e1 in events:
            flush.zero_()
            torch.cuda.synchronize()  # nothing (a copy on another stream) starts before e0
            e0.record(stream)
            fn()
            e1.record(stream)
        torch.cuda.synchronize()
        total = sum(e0.elapsed_time(e1) for e0, e1 in events)
    barrier(world)
    return max_over_ranks(total, world, dev)


def gemm_roofline(dev, M: int, name: str = "fc1", reps: int = 10):
    """Times one block GEMM as the model launches it (FP16-split operands; fc1:
    bias + GELU with FP16-split output; proj / fc2: bias + residual; qkv: bias)
    alone; returns ms per launch."""
    from vit_cuda import _lib
    from vit_cuda.split import f16_planes, f16_weight
    lib = _lib.lib
    N, K, epi, split_out = ROOFLINE_GEMMS[name]
    code = {"bias": _lib.EPI_BIAS, "gelu": _lib.EPI_BIAS_GELU, "resid": _lib.EPI_BIAS_RESID}[epi]
    s = torch.cuda.current_stream().cuda_stream
    a = torch.randn(M, K, device=dev)
    w = torch.randn(N, K, device=dev) * 0.02
    bias = torch.randn(N, device=dev) * 0.02
    ap = f16_planes(a, 2)
    wp, acc_scale = f16_weight(w)
    del a
    out = torch.empty(2, M, N, dtype=torch.int16, device=dev) if split_out else None
    y = None if split_out else torch.randn(M, N, device=dev)

    def launch():
        _lib.check(lib.vitb200_gemm_f16(ap.data_ptr(), wp.data_ptr(), acc_scale, bias.data_ptr(),
                                        y.data_ptr() if epi == "resid" else None,
                                        y.data_ptr() if y is not None else None, N,
                                        out.data_ptr() if out is not None else None, M, K, N,
                                        code, s), "gemm")

    for _ in range(3):
        launch()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        launch()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    del ap, wp, out, y
    return ms


def measured_tensor_peak():
    """Dense bf16 (= fp16) tensor TFLOP/s from MEASURED_PEAKS.json (burst),
    else the pool's fallback figure."""
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            v = float(json.load(f)["bf16_tflops"])
        return v, "MEASURED_PEAKS.json bf16_tflops (cuBLAS bf16 8192^3, burst; of measured)"
    except (OSError, ValueError, KeyError):
        return 1590.0, "fallback 1.59 PFLOP/s bf16 (of fallback)"


def ncu_traffic(name: str):
    """DRAM bytes per launch from the committed ncu summary, if present."""
    path = os.path.join(REPO, "profiles", name)
    try:
        with open(path) as f:
            return json.load(f).get("dram_bytes_per_launch")
    except (OSError, ValueError):
        return None


def cpu_oracle_rate(img_size: int, sample: int, min_seconds: float = 10.0, max_reps: int = 20):
    """Images/s of the CPU oracle (fp32) on `sample` images, repeated for at
    least min_seconds (one repetition minimum)."""
    from oracle import vit_oracle
    from vit_cuda.weights import synthetic_images, synthetic_state_dict
    torch.set_num_threads(os.cpu_count() or 1)
    state = synthetic_state_dict(seed=0, img_size=img_size)
    img = synthetic_images(sample, img_size, seed=0)
    with torch.no_grad():
        vit_oracle.vit_forward(img[:1], state, dtype=torch.float32)  # warm-up
        t0 = time.perf_counter()
        reps = 0
        while reps < max_reps:
            vit_oracle.vit_forward(img, state, dtype=torch.float32)
            reps += 1
            if time.perf_counter() - t0 >= min_seconds:
                break
        dt = time.perf_counter() - t0
    return sample * reps / dt, reps, torch.get_num_threads()


def cpu_oracle_p50_bs1(img_size: int, runs: int = 20) -> float:
    """Median milliseconds of `runs` single-image CPU oracle forwards (fp32,
    all host threads) after one warm-up."""
    from oracle import vit_oracle
    from vit_cuda.weights import synthetic_images, synthetic_state_dict
    torch.set_num_threads(os.cpu_count() or 1)
    state = synthetic_state_dict(seed=0, img_size=img_size)
    img = synthetic_images(1, img_size, seed=0)
    times = []
    with torch.no_grad():
        vit_oracle.vit_forward(img, state, dtype=torch.float32)
        for _ in range(runs):
            t0 = time.perf_counter()
            vit_oracle.vit_forward(img, state, dtype=torch.float32)
            times.append((time.perf_counter() - t0) * 1e3)
    return statistics.median(times)


def input_bytes(batch: int, img: int) -> int:
    """Bytes of one step's images on one GPU ([batch, 3, img, img] fp32)."""
    return batch * 3 * img * img * 4


def flush_bytes(batch: int, img: int) -> int:
    """L2 flush buffer of a step whose input fits in L2 (twice L2), else 0."""
    return 2 * L2_BYTES if input_bytes(batch, img) < L2_BYTES else 0


def workload_config(name: str, world: int, weights: str = "init") -> dict:
    """The `config` both arms report for workload `name` on `world` GPUs."""
    batch, img = CONFIGS[name]
    h2d = input_bytes(batch, img)
    fb = flush_bytes(batch, img)
    model = ("ViT-B/16 (random init, seed 0)" if weights == "init" else
             "ViT-B/16 (random init reshaped to trained-like statistics, seed 0)")
    return {"workload": name, "model": model,
            "global_batch": batch * world, "img_size": img, "seq_len": (img // 16) ** 2 + 1,
            "parallelism": f"dp{world}" if world > 1 else "single GPU",
            "l2": ("inputs larger than L2 (%.0f MB per GPU per step)" % (h2d / 1e6) if fb == 0
                   else "L2 flushed before every timed step (%.0f MB written, outside the "
                        "per-step CUDA events); input %.1f MB per GPU per step"
                        % (fb / 1e6, h2d / 1e6)),
            "gflop_per_image": GFLOP_PER_IMG.get(img)}


# ----------------------------------------------------------------- arms
def run_reference(args):
    rank, _, world = dist_env()
    if rank != 0:
        return
    batch, img = CONFIGS[args.config]
    from oracle import vit_oracle
    from vit_cuda.weights import synthetic_images, synthetic_state_dict
    torch.set_num_threads(os.cpu_count() or 1)
    state = synthetic_state_dict(seed=0, img_size=img, stats=args.weights)
    x = synthetic_images(args.cpu_sample, img, seed=0)
    with torch.no_grad():
        for _ in range(args.warmup):
            vit_oracle.vit_forward(x, state, dtype=torch.float32)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            vit_oracle.vit_forward(x, state, dtype=torch.float32)
        dt = time.perf_counter() - t0
    rate = args.cpu_sample * args.steps / dt
    sample = (f"{args.cpu_sample} images per step of the {args.config} workload "
              f"({img}x{img}, fp32), CPU oracle port of the reference path")
    config = workload_config(args.config, world, args.weights)
    config["cpu_sample"] = (f"each step times {args.cpu_sample} of the {batch * world} images "
                            f"on the host cores ({torch.get_num_threads()} threads)")
    emit({
        "impl": "reference", "metric": METRIC, "value": rate, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config,
        "cpu_baseline": {"value": rate, "unit": UNIT, "cores": torch.get_num_threads(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": rate, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "p50_bs1_ms": {"cpu_ms": cpu_oracle_p50_bs1(img, args.cpu_p50_runs),
                       "runs": args.cpu_p50_runs},
    })


def run_ours(args):
    rank, local_rank, world = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    assert torch.cuda.is_available(), "bench.py needs CUDA devices"
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)

    import vit_cuda
    from vit_cuda import _lib
    from vit_cuda.parallel import gather_rows
    from vit_cuda.weights import synthetic_images, synthetic_state_dict

    batch, img = CONFIGS[args.config]
    T = (img // 16) ** 2 + 1
    total = batch * world
    state = synthetic_state_dict(seed=0, img_size=img, stats=args.weights)
    model = vit_cuda.ViTCUDA(state_dict={k: v.to(dev) for k, v in state.items()}).to(dev).eval()
    model.prepare()
    operands = sorted({k for blk in model.gemm_operands for k in blk.values()})
    x_host = synthetic_images(batch, img, seed=1000 + rank)
    x_dev = x_host.to(dev)
    # A step whose input fits in L2 gets L2 flushed before it (outside the timing).
    fb = flush_bytes(batch, img)
    flush_buf = torch.empty(fb // 4, dtype=torch.float32, device=dev) if fb else None

    def step_device():
        logits = model._forward_impl(x_dev)
        if world > 1:
            gather_rows(logits, total)

    x_pin = x_host.pin_memory()
    out_pin = torch.empty((total, model.num_classes), dtype=torch.float32).pin_memory()
    # Public API for host-resident batches: each step copies its own batch
    # host->device (on a copy stream, overlapping the previous step's forward)
    # and its logits device->host, all inside the timed region.
    streamed = vit_cuda.StreamedInference(
        model, tuple(x_host.shape),
        fn=(lambda t: gather_rows(model(t), total)) if world > 1 else None)

    def step_e2e():
        streamed(x_pin, out_pin)

    with torch.no_grad():
        for _ in range(args.warmup):
            step_device()
            step_e2e()
        torch.cuda.synchronize()
        clocks = ClockSampler(torch.cuda.current_device() if "CUDA_VISIBLE_DEVICES" not in
                              os.environ else local_rank)
        clocks.start()
        n0 = _lib.lib.vitb200_launch_count()
        ms = timed(step_device, args.steps, world, dev, flush=flush_buf)
        launches = _lib.lib.vitb200_launch_count() - n0
        clk = clocks.stop()
        ms_e2e = timed(step_e2e, args.steps, world, dev, flush=flush_buf)
        # The north star's formulation: every GEMM on TF32 pairs (TF32x3).
        model_tf32 = vit_cuda.ViTCUDA(state_dict={k: v.to(dev) for k, v in state.items()},
                                      operands="tf32").to(dev).eval()
        model_tf32.prepare()

        def step_tf32():
            logits = model_tf32._forward_impl(x_dev)
            if world > 1:
                gather_rows(logits, total)

        for _ in range(args.warmup):
            step_tf32()
        ms_tf32 = timed(step_tf32, args.steps, world, dev, flush=flush_buf)
        del model_tf32
    assert _lib.device_error() == 0, "a kernel reported a device error"

    value = total * args.steps / (ms * 1e-3)
    e2e_value = total * args.steps / (ms_e2e * 1e-3)
    h2d = x_host.numel() * 4
    d2h = total * model.num_classes * 4
    del x_dev

    # Roofline of the fc1 GEMM (FP16-split operands), the model's largest GEMM.
    M = batch * T
    gemm_ms = gemm_roofline(dev, M, "fc1")
    alg_flops = 2.0 * M * 3072 * 768
    peak, peak_src = measured_tensor_peak()
    achieved = 3 * alg_flops / (gemm_ms * 1e-3) / 1e12
    traffic = ncu_traffic(f"gemm_f16x3_fc1_{args.config}.json")
    roofline = {
        "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
        "frac": achieved / peak, "traffic": traffic,
        "kernel": f"gemm f16x3 fc1 M={M} N=3072 K=768 (+bias+GELU, FP16-split out)",
        "kernel_ms": gemm_ms, "algorithmic_tflops": alg_flops / (gemm_ms * 1e-3) / 1e12,
        "peak_source": peak_src + "; achieved counts the 3 FP16 tensor products per "
                       "algorithmic multiply-add",
    }

    result = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args.config, world, args.weights),
        "block_gemm_operands": "+".join(operands),
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": ms_e2e / args.steps},
        "gpu_launches": int(launches),
        "tf32x3": {"value": total * args.steps / (ms_tf32 * 1e-3), "unit": UNIT,
                   "ms_per_step": ms_tf32 / args.steps,
                   "note": "same forward, every GEMM on TF32 pairs (TF32x3)"},
        "roofline": roofline,
        "clocks": clk,
        "model_tflops": GFLOP_PER_IMG.get(img, 0) * value / 1e3,
    }

    if world == 1 and rank == 0 and not args.no_p50:
        result["p50_bs1_ms"] = p50_bs1(state, img, dev)
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        rate, reps, cores = cpu_oracle_rate(img, args.cpu_sample)
        result["cpu_baseline"] = {
            "value": rate, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{args.cpu_sample} images x {reps} reps of the {args.config} workload "
                      "(CPU oracle port of the reference path, fp32)",
            "p50_bs1_ms": cpu_oracle_p50_bs1(img, args.cpu_p50_runs)}
    if rank == 0:
        emit(result)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def p50_bs1(state, img, dev, iters: int = 200) -> dict:
    """Batch-1 latency: CUDA-graph replays (the reference's capture_graph path)
    and eager calls, CUDA events per call, median."""
    import vit_cuda
    model = vit_cuda.ViTCUDA(state_dict={k: v.to(dev) for k, v in state.items()}).to(dev).eval()
    x = torch.randn(1, 3, img, img, device=dev)

    def lat(fn):
        ts = []
        for _ in range(10):
            fn()
        torch.cuda.synchronize()
        for _ in range(iters):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        return statistics.median(ts)

    with torch.no_grad():
        eager = lat(lambda: model(x))
        model.capture_graph(x, num_warmup=3)
        graph = lat(lambda: model(x))
        model.release_graph()
    return {"graph_ms": graph, "eager_ms": eager}


def attention_roofline(dev, B: int, T: int, reps: int = 10):
    """Times the FP16-split attention (vitb200_attention_f16: splits of q, k,
    V^T, then the attention kernel) on [B, T, 768] inputs; returns ms per call."""
    from vit_cuda import _lib
    lib = _lib.lib
    s = torch.cuda.current_stream().cuda_stream
    q, k, v = (torch.randn(B, T, 768, device=dev) for _ in range(3))
    o = torch.empty_like(q)
    ws = torch.empty(lib.vitb200_attention_f16_workspace_bytes(B, T, 12), dtype=torch.uint8,
                     device=dev)

    def launch():
        _lib.check(lib.vitb200_attention_f16(q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                             o.data_ptr(), B, T, 12, 768, 768, 768, 768, 0.125,
                                             1.0, 1.0, ws.data_ptr(), ws.numel(), s), "attention")

    for _ in range(3):
        launch()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        launch()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def per_op_roofline(dev, B: int, T: int, kernel: str, reps: int = 10):
    """Times a per-op TF32x3 entry point as a user calls it (its operand splits
    included): vit_cuda._C.flash_attn_2 on [B, T, 768] q, k, v, or
    vit_cuda._C.gemm_bias for the patch projection (768 -> 768 over B*T rows);
    returns ms per call."""
    from vit_cuda import _C
    if kernel == "attention_tf32":
        q, k, v = (torch.randn(B, T, 768, device=dev) for _ in range(3))

        def launch():
            _C.flash_attn_2(q, k, v, 0.125)
    else:
        x = torch.randn(B * T, 768, device=dev)
        w = torch.randn(768, 768, device=dev) * 0.02
        b = torch.randn(768, device=dev) * 0.02

        def launch():
            _C.gemm_bias(x, w, b)
    for _ in range(3):
        launch()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        launch()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def run_roofline_only(args):
    """The dominant kernel alone (fc1 shape for `batch` images), a small case
    for profilers; prints one JSON line with its CUDA-event time."""
    torch.backends.cuda.matmul.allow_tf32 = False
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    batch, img = CONFIGS[args.config]
    if args.batch:
        batch = args.batch
    T = (img // 16) ** 2 + 1
    M = batch * T
    if args.kernel in ("attention_tf32", "patch"):
        ms = per_op_roofline(dev, batch, T, args.kernel, reps=max(1, args.steps))
        flop = (4.0 * batch * 12 * T * T * 64 if args.kernel == "attention_tf32"
                else 2.0 * M * 768 * 768)
        emit({"mode": "roofline", "kernel": f"per-op TF32x3 {args.kernel} (splits included)",
              "B": batch, "T": T, "M": M, "call_ms": ms,
              "algorithmic_tflops": flop / (ms * 1e-3) / 1e12})
        return
    if args.kernel == "attention":
        ms = attention_roofline(dev, batch, T, reps=max(1, args.steps))
        emit({"mode": "roofline", "kernel": "attention f16 (splits + attention_f16_kernel)",
              "B": batch, "T": T, "heads": 12, "call_ms": ms,
              "algorithmic_tflops": 4.0 * batch * 12 * T * T * 64 / (ms * 1e-3) / 1e12})
        return
    N, K = ROOFLINE_GEMMS[args.kernel][:2]
    ms = gemm_roofline(dev, M, args.kernel, reps=max(1, args.steps))
    emit({"mode": "roofline", "kernel": f"gemm f16x3 {args.kernel}", "M": M, "N": N, "K": K,
          "kernel_ms": ms, "f16_pipe_tflops": 3 * 2.0 * M * N * K / (ms * 1e-3) / 1e12})


def run_forward_only(args):
    """`warmup` + `steps` forwards of the model on `batch` images of the
    config's size, nothing else (a small case for profilers); prints one JSON
    line with the median CUDA-event time per forward."""
    torch.backends.cuda.matmul.allow_tf32 = False
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    import vit_cuda
    from vit_cuda.weights import synthetic_images, synthetic_state_dict
    batch, img = CONFIGS[args.config]
    if args.batch:
        batch = args.batch
    state = synthetic_state_dict(seed=0, img_size=img, stats=args.weights)
    model = vit_cuda.ViTCUDA(state_dict={k: v.to(dev) for k, v in state.items()}).to(dev).eval()
    x = synthetic_images(batch, img, seed=1).to(dev)
    times = []
    with torch.no_grad():
        for i in range(args.warmup + args.steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            model(x)
            e1.record()
            torch.cuda.synchronize()
            if i >= args.warmup:
                times.append(e0.elapsed_time(e1))
    from vit_cuda import _lib
    assert _lib.device_error() == 0, "a kernel reported a device error"
    emit({"mode": "forward", "workload": args.config, "batch": batch,
          "ms_per_forward": statistics.median(times) if times else None})


def run_peaks():
    """Dense tensor throughput of cuBLAS (torch.matmul) at 8192^3 on this GPU:
    TF32 (fp32 inputs with TF32 allowed), bf16 and fp16; burst = best of 10
    launches, sustained = back-to-back launches for about 3 s (power capped).
    TF32 is the north star's formulation (TF32x3 costs three TF32 products per
    multiply); the repository's kernels run FP16 products."""
    dev = torch.device("cuda", 0)
    n = 8192
    flops = 2.0 * n ** 3
    out = {"mode": "peaks", "shape": f"{n}^3"}

    def measure(dtype, tf32, seconds):
        torch.backends.cuda.matmul.allow_tf32 = tf32
        a = torch.randn(n, n, device=dev).to(dtype)
        b = torch.randn(n, n, device=dev).to(dtype)
        for _ in range(3):
            a @ b
        torch.cuda.synchronize()
        best = float("inf")
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            a @ b
            e1.record()
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1))
        burst = flops / (best * 1e-3) / 1e12
        reps = max(1, int(seconds / (best * 1e-3)))
        clocks = ClockSampler(0)
        clocks.start()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            a @ b
        e1.record()
        torch.cuda.synchronize()
        clk = clocks.stop()
        sustained = flops * reps / (e0.elapsed_time(e1) * 1e-3) / 1e12
        torch.backends.cuda.matmul.allow_tf32 = False
        return burst, sustained, clk

    for name, dtype, tf32 in (("tf32", torch.float32, True), ("bf16", torch.bfloat16, False),
                              ("fp16", torch.float16, False)):
        burst, sustained, clk = measure(dtype, tf32, 3.0)
        out[f"{name}_tflops"] = burst
        out[f"{name}_tflops_sustained"] = sustained
        out[f"{name}_clocks_sustained"] = clk
    emit(out)


def main():
    args = parse_args()
    if args.mode == "peaks":
        run_peaks()
        return
    if args.mode == "roofline":
        run_roofline_only(args)
        return
    if args.mode == "forward":
        run_forward_only(args)
        return
    if args.batch:
        CONFIGS[args.config] = (args.batch, CONFIGS[args.config][1])
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
