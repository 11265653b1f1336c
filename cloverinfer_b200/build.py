"""Build libclover_b200.so (sm_100a) in-tree with nvcc.

    python -m cloverinfer_b200.build            # build if sources changed
    python -m cloverinfer_b200.build --force    # rebuild

The library is written to ``cloverinfer_b200/_lib/libclover_b200.so``; it is
git-ignored but travels with the working tree.  Each ``.cu`` file compiles to
its own object in parallel, then nvcc links the shared library with the CUDA
runtime linked statically (the library exports only the ``clover_b200_*``
C ABI of ``include/clover_b200.h``).
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OUT_DIR = os.path.join(PKG, "_lib")
LIB_NAME = "libclover_b200.so"
LIB_PATH = os.path.join(OUT_DIR, LIB_NAME)
STAMP = os.path.join(OUT_DIR, "build.stamp")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr"]


def nvcc_path() -> str:
    cand = [shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"]
    for c in cand:
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libclover_b200")


def sources() -> list:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _digest() -> str:
    h = hashlib.sha256()
    files = sources() + [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC))
                         if f.endswith((".cuh", ".h"))]
    files += [os.path.join(INCLUDE, f) for f in sorted(os.listdir(INCLUDE))]
    for f in files:
        h.update(f.encode())
        with open(f, "rb") as fh:
            h.update(fh.read())
    h.update(" ".join(ARCH_FLAGS + NVCC_FLAGS).encode())
    return h.hexdigest()


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH) or not os.path.exists(STAMP):
        return False
    with open(STAMP) as f:
        return f.read().strip() == _digest()


def _compile(nvcc: str, src: str, obj: str, extra: list) -> None:
    cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, *extra, "-I", INCLUDE, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    if "-Xptxas" in extra:
        sys.stderr.write(r.stderr)


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    """Compile every CUDA source for sm_100a and link the shared library."""
    if not force and up_to_date():
        return LIB_PATH
    nvcc = nvcc_path()
    os.makedirs(OUT_DIR, exist_ok=True)
    objs = []
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        futs = []
        for src in sources():
            obj = os.path.join(OUT_DIR, os.path.basename(src)[:-3] + ".o")
            objs.append(obj)
            futs.append(ex.submit(_compile, nvcc, src, obj, extra))
        for f in futs:
            f.result()
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", tmp, *objs, "-cudart", "static"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB_PATH)
    with open(STAMP, "w") as f:
        f.write(_digest())
    return LIB_PATH


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force or a.ptxas_verbose, verbose_ptxas=a.ptxas_verbose))
