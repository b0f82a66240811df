"""Build ``libmh3_b200.so`` (the C-ABI library) in-tree with nvcc for sm_100a.

    python -m minimaxh3_b200.build          # incremental
    python -m minimaxh3_b200.build --force  # rebuild everything

Each ``csrc/*.cu`` is compiled to ``_build/<name>.o`` (skipped when newer
than its sources and headers), then linked into
``minimaxh3_b200/libmh3_b200.so`` with the static CUDA runtime, so the
library has no link dependency on libcuda or on torch.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO_DIR, "include")
BUILD_DIR = os.path.join(REPO_DIR, "_build")
LIB_PATH = os.path.join(PKG_DIR, "libmh3_b200.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-O3,-fvisibility=hidden",
    "-I" + INCLUDE,
    "-I" + CSRC,
    "-DMH3_BUILDING_LIB",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put it on PATH)")


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return hs


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(nvcc: str, src: str, obj: str, verbose_ptxas: bool) -> str:
    cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-c", src, "-o", obj]
    if verbose_ptxas:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return r.stdout + r.stderr


def build(force: bool = False, verbose_ptxas: bool = False, jobs: int | None = None) -> str:
    """Compile every CUDA source for sm_100a and link the shared library."""
    nvcc = nvcc_path()
    os.makedirs(BUILD_DIR, exist_ok=True)
    headers = _headers()
    srcs = _sources()
    objs = []
    todo = []
    for src in srcs:
        obj = os.path.join(BUILD_DIR, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or _stale(obj, [src, *headers]):
            todo.append((src, obj))
    logs = []
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(len(todo), os.cpu_count() or 1)) as ex:
            futs = [ex.submit(_compile, nvcc, s, o, verbose_ptxas) for s, o in todo]
            for f in futs:
                logs.append(f.result())
    if force or todo or _stale(LIB_PATH, objs):
        tmp = LIB_PATH + ".tmp"
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", tmp, *objs, "-cudart", "static", "-lrt", "-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB_PATH)
    return "".join(logs)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    args = ap.parse_args(argv)
    out = build(force=args.force, verbose_ptxas=args.ptxas_verbose)
    if out:
        sys.stdout.write(out)
    print(LIB_PATH)


if __name__ == "__main__":
    main()
