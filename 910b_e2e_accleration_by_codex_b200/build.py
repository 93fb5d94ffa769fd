"""Build the in-tree CUDA library ``libgdn_b200.so`` for sm_100a with nvcc.

Every ``csrc/*.cu`` file is compiled to an object under ``_build/`` at the repo root
(rebuilt when it or any ``csrc/*.cuh`` / ``include/*.h`` header is newer), then linked
into ``libgdn_b200.so`` next to this file.  nvcc cross-compiles, so this runs on a
machine without a GPU.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG_DIR, "libgdn_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-fvisibility=hidden", f"-I{os.path.join(ROOT, 'include')}"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the GDN CUDA library cannot be built")


def _newest_header() -> float:
    hs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def _compile(nvcc: str, src: str, obj: str, ptxas_verbose: bool) -> str:
    cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj]
    if ptxas_verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    return r.stderr


def build(verbose: bool = False, ptxas_verbose: bool = False, force: bool = False) -> str:
    """Compile csrc/*.cu for sm_100a and link libgdn_b200.so; returns the library path."""
    nvcc = nvcc_path()
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdr_t = _newest_header()
    jobs = []
    objs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if force or ptxas_verbose or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), hdr_t):
            jobs.append((s, o))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            futs = {ex.submit(_compile, nvcc, s, o, ptxas_verbose): s for s, o in jobs}
            for f in cf.as_completed(futs):
                log = f.result()
                if verbose and log:
                    print(f"[{os.path.basename(futs[f])}]\n{log}", file=sys.stderr)
    lib_t = os.path.getmtime(LIB) if os.path.exists(LIB) else 0.0
    if jobs or lib_t < max(os.path.getmtime(o) for o in objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc, *ARCH, "-shared", "-o", tmp, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    if verbose:
        print(f"built {LIB}", file=sys.stderr)
    return LIB


if __name__ == "__main__":
    build(verbose=True, ptxas_verbose="-v" in sys.argv, force="-f" in sys.argv)
