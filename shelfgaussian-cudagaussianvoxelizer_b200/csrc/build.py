"""Build libg2v.so (the C-ABI library) for sm_100a with nvcc.

    python shelfgaussian-cudagaussianvoxelizer_b200/csrc/build.py [--force]

Objects go to csrc/_build/, the library to CudaGaussianVoxelizer/libg2v.so next to the Python
package that loads it.  g2v_prep.cu is compiled with --use_fast_math (the reference's flag) so that
its box arithmetic rounds like the reference build; everything else uses IEEE division/sqrt.
cudart is linked statically, so the library does not depend on the CUDA runtime that torch ships.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
REPO = os.path.dirname(PKG)
INCLUDE = os.path.join(REPO, "include")
OBJ_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(PKG, "CudaGaussianVoxelizer", "libg2v.so")

SOURCES = {
    "g2v_api.cu": [],
    "g2v_prep.cu": ["--use_fast_math"],
    "g2v_scan.cu": [],
    "g2v_csr.cu": [],
    "g2v_splat.cu": [],
    "g2v_grad.cu": [],
    "g2v_profile.cu": [],
    "g2v_static.cu": [],
    "g2v_splat_tc.cu": [],
    "g2v_grad_tc.cu": [],
    "g2v_spass_tc.cu": [],
    "g2v_selftest.cu": [],
    "g2v_loss.cu": [],
    "g2v_cov.cu": [],
}
HEADERS_TC = ["g2v_tc.cuh"]
HEADERS = [os.path.join(HERE, "g2v_internal.cuh"), os.path.join(HERE, "g2v_tc.cuh"), os.path.join(HERE, "g2v_cov.cuh"),
           os.path.join(INCLUDE, "g2v.h")]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
          "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", HERE]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra_flags=()) -> str:
    os.makedirs(OBJ_DIR, exist_ok=True)
    nv = nvcc()
    jobs = []
    objs = []
    for src, flags in SOURCES.items():
        path = os.path.join(HERE, src)
        obj = os.path.join(OBJ_DIR, src.replace(".cu", ".o"))
        objs.append(obj)
        if force or _stale(obj, [path, *HEADERS, __file__]):
            cmd = [nv, *ARCH, *COMMON, *flags, *extra_flags, "-c", path, "-o", obj]
            jobs.append((src, cmd))

    def run(job):
        src, cmd = job
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
        return src, r.stderr

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for src, err in ex.map(run, jobs):
            if verbose and err.strip():
                print(err, file=sys.stderr)
    if force or jobs or _stale(LIB, objs):
        tmp = LIB + f".tmp{os.getpid()}"
        cmd = [nv, *ARCH, "-shared", "-o", tmp, *objs, "-Xlinker", "--no-undefined"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers / spills per kernel")
    a = ap.parse_args()
    extra = ["-Xptxas", "-v"] if a.ptxas_info else []
    print(build(force=a.force or a.ptxas_info, verbose=a.verbose or a.ptxas_info, extra_flags=extra))
