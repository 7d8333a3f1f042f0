"""Build liblai_kernels.so in-tree for sm_100a (nvcc, no JIT cache).

    python local-ai-server_b200/build.py [--force] [--ptxas-v]

Each csrc/*.cu / *.cpp is compiled to _build/*.o (rebuilt when the source or a
header is newer), then linked into local-ai-server_b200/liblai_kernels.so with the
CUDA runtime linked statically, so the library loads beside any torch build.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "liblai_kernels.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
              "-I", os.path.join(REPO, "include")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build liblai_kernels.so")


def _headers() -> list[str]:
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(REPO, "include", "*.h"))


def _stale(obj: str, src: str, deps: list[str]) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(p) > t for p in [src, *deps])


def _compile(src: str, obj: str, extra: list[str]) -> tuple[str, str]:
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    return src, r.stderr


def build(force: bool = False, ptxas_verbose: bool = False, quiet: bool = True) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    deps = _headers()
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    objs, jobs = [], []
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        for src in srcs:
            obj = os.path.join(OUT_DIR, os.path.basename(src) + ".o")
            objs.append(obj)
            if force or ptxas_verbose or _stale(obj, src, deps):
                jobs.append(ex.submit(_compile, src, obj, extra))
        for j in cf.as_completed(jobs):
            src, log = j.result()
            if log and (ptxas_verbose or not quiet):
                print(f"--- {os.path.basename(src)}\n{log}", file=sys.stderr)
    if force or jobs or not os.path.exists(LIB) or any(
            os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, ptxas_verbose=a.ptxas_v, quiet=False))
