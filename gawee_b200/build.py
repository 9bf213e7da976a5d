"""Build libgawee_cuda.so in-tree with nvcc for sm_100a.

    python -m gawee_b200.build [--force] [--jobs N]

Objects go to gawee_b200/_build/, the library to gawee_b200/libgawee_cuda.so,
and the native command-line tools to gawee_b200/bin/.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libgawee_cuda.so")
BIN = os.path.join(HERE, "bin")

SOURCES = [
    "kernels/memory_ops.cu",
    "kernels/conv_gemm_tc.cu",
    "kernels/conv_gemm_tma.cu",
    "kernels/attention_tc.cu",
    "kernels/noalloc_gemm.cu",
    "kernels/tc_probe.cu",
    "host/ir.cpp",
    "host/plan.cpp",
    "host/runtime.cpp",
]
TOOLS = {
    "gawee-cuda-runner": "tools/gawee_cuda_runner.cpp",
}
HEADERS = ["kernels/kernels.h", "kernels/program.cuh", "kernels/tc_common.cuh", "host/ir.h", "host/plan.h", "host/launch.h", "host/npy.h"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
                     "-diag-suppress", "128,177", "-I" + os.path.join(ROOT, "include"), "-I/usr/include"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _newest_header() -> float:
    hs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "gawee_cuda.h")]
    return max(os.path.getmtime(h) for h in hs if os.path.exists(h))


def _compile(src: str, force: bool, hdr_time: float) -> str:
    path = os.path.join(CSRC, src)
    obj = os.path.join(OBJ, src.replace("/", "_") + ".o")
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(path), hdr_time):
        return obj
    cmd = [nvcc()] + NVCC_FLAGS + ["-c", path, "-o", obj]
    if src.endswith(".cpp"):
        cmd = [nvcc(), "-x", "cu"] + NVCC_FLAGS + ["-c", path, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {src}\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False, jobs: int = 8, verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    hdr_time = _newest_header()
    with ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, hdr_time), SOURCES))
    newest_obj = max(os.path.getmtime(o) for o in objs)
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < newest_obj:
        cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs + ["-ldl", "-lrt", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed\n{r.stdout}\n{r.stderr}")
    os.makedirs(BIN, exist_ok=True)
    for name, src in TOOLS.items():
        path = os.path.join(CSRC, src)
        out = os.path.join(BIN, name)
        if not os.path.exists(path):
            continue
        if force or not os.path.exists(out) or os.path.getmtime(out) < max(os.path.getmtime(path),
                                                                            os.path.getmtime(LIB)):
            cmd = ["g++", "-std=c++17", "-O2", "-I" + os.path.join(ROOT, "include"), path,
                   os.path.join(CSRC, "host", "ir.cpp"), "-o", out,
                   "-L" + HERE, "-lgawee_cuda", "-Wl,-rpath,$ORIGIN/.."]
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"tool build failed: {name}\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(LIB)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=8)
    a = ap.parse_args(argv)
    build(a.force, a.jobs, verbose=True)


if __name__ == "__main__":
    sys.exit(main())
