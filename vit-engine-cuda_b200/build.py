"""Builds libvitb200.so (the sm_100a kernels + C ABI) in-tree with nvcc.

    python vit-engine-cuda_b200/build.py [--force] [--jobs N]

The library lands next to the Python package (vit_cuda/libvitb200.so) so that it
travels with the source tree; it links the CUDA runtime statically and resolves
the driver's tensor-map encoder at run time, so it loads on a machine without a
GPU (the kernels themselves need an sm_100a device).
"""
from __future__ import annotations

import argparse
import os
import re
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(REPO, "include")
OUT_DIR = os.path.join(HERE, "vit_cuda")
LIB = os.path.join(OUT_DIR, "libvitb200.so")
OBJ_DIR = os.path.join(HERE, "_build")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr", "-Xptxas", "-v",
    # No -use_fast_math: the parity kernels rely on IEEE division, sqrt, expf, erff.
]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found")
    return path


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs.append(os.path.join(INCLUDE, "vitb200.h"))
    return hs


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(f) <= t for f in sources() + headers() + [__file__])


def compile_one(src: str) -> tuple[str, str]:
    obj = os.path.join(OBJ_DIR, os.path.basename(src).replace(".cu", ".o"))
    cmd = [nvcc(), *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


# Kernels that move registers between warpgroups with setmaxnreg, and the
# per-thread register count their split assumes. csrc/attention_f16.cu and
# csrc/attention_f16_tile.cu: 384 threads launched at 168. csrc/gemm_tcgen05.cu: the last template argument
# (EPI, the number of epilogue warpgroups) sets it: 2 -> 384 threads at 168,
# 3 -> 512 threads at 128, 4 -> 640 threads at 96 (EpiCfg there). A kernel compiled to any other count
# could make setmaxnreg.inc wait forever.
def expected_registers(mangled: str) -> int | None:
    if "attention_f16_kernel" in mangled or "attention_f16_tile_kernel" in mangled:
        return 168
    m = re.search(r"gemm_tf32x3_kernelI(.*?)EEv", mangled)
    if m:
        epi = int(re.findall(r"Li(\d+)E", m.group(1) + "E")[-1])
        return {2: 168, 3: 128, 4: 96}[epi]
    return None


def check_register_split(ptxas_log: str) -> None:
    current, expected = None, None
    for line in ptxas_log.splitlines():
        if "Compiling entry function" in line:
            current = line.split("'")[1] if "'" in line else line
            expected = expected_registers(current)
        elif expected is not None and "Used" in line and "registers" in line:
            used = int(line.split("Used")[1].split("registers")[0])
            if used != expected:
                raise RuntimeError(
                    f"{current} compiled to {used} registers per thread; its setmaxnreg split "
                    f"requires exactly {expected}")
            current, expected = None, None


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    os.makedirs(OBJ_DIR, exist_ok=True)
    srcs = sources()
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    with ThreadPoolExecutor(max_workers=jobs) as ex:
        results = list(ex.map(compile_one, srcs))
    for _, log in results:
        check_register_split(log)
        if verbose:
            sys.stderr.write(log)
    objs = [o for o, _ in results]
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/smem usage")
    a = ap.parse_args()
    print(build(force=a.force, jobs=a.jobs, verbose=a.verbose))


if __name__ == "__main__":
    main()
