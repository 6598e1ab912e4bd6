"""Builds libmoe_cuda.so in-tree for sm_100a (nvcc cross-compiles without a GPU).

    python -m flash_deepseek_b200.build [--force]
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
ROOT = os.path.dirname(HERE)
OUT = os.path.join(HERE, "libmoe_cuda.so")
SOURCES = ["moe_kernels.cu", "moe_experts.cu", "moe_experts_tc.cu", "moe_prefill.cu", "moe_ep.cu", "moe_api.cu",
           "moe_noalloc.cu", "moe_dense.cu", "moe_sample.cu"]
HEADERS = ["moe_common.cuh", "moe_internal.h", "moe_nccl.h", "moe_umma.cuh", "moe_wait.h"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "-diag-suppress", "177,550", f"-I{os.path.join(ROOT, 'include')}"]
# extra nvcc flags (e.g. -D overrides of tuning constants for a side-by-side build)
FLAGS += os.environ.get("MOE_NVCC_EXTRA", "").split()


def _stale() -> bool:
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS] + [os.path.join(ROOT, "include", "moe_cuda.h")]
    return any(os.path.getmtime(p) > t for p in deps)


def _obj(src: str) -> str:
    return os.path.join(CSRC, "_build", src.replace(".cu", ".o"))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return OUT
    os.makedirs(os.path.join(CSRC, "_build"), exist_ok=True)

    def compile_one(src):
        cmd = [NVCC, *ARCH, *FLAGS, "-c", os.path.join(CSRC, src), "-o", _obj(src)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if verbose:
            sys.stderr.write(r.stderr)
        return src

    with ThreadPoolExecutor(len(SOURCES)) as ex:
        list(ex.map(compile_one, SOURCES))
    link = [NVCC, *ARCH, "-shared", "-o", OUT + ".tmp", *[_obj(s) for s in SOURCES], "-ldl",
            "-Xlinker", "-rpath,$ORIGIN"]
    r = subprocess.run(link, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
