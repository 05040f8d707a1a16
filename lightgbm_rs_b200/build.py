"""Build the in-tree shared library lightgbm_rs_b200/liblgbm_b200.so for sm_100a.

Incremental: objects under lightgbm_rs_b200/_build/ are rebuilt when a source or
header is newer. Usage: python -m lightgbm_rs_b200.build [--force]
"""

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "liblgbm_b200.so")
NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
HOST_CXX = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else (shutil.which("g++") or "g++")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", f"-I{INCLUDE}", f"-I{CSRC}"]
# --fmad=false: f64 expressions round exactly as the reference (no a*b+c contraction).
NVCC_FLAGS = ARCH + COMMON + ["--fmad=false", "-lineinfo", "-Xcompiler", "-fPIC",
                              "-Xcompiler", "-ffp-contract=off", "-ccbin", HOST_CXX]
CXX_FLAGS = COMMON + ["-fPIC", "-ffp-contract=off", "-Wall"]


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(obj, src, deps):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(p) > t for p in [src] + deps)


def _compile(src, obj, extra=()):
    if src.endswith(".cu"):
        cmd = [NVCC] + NVCC_FLAGS + list(extra) + ["-c", src, "-o", obj]
    else:
        cmd = [HOST_CXX] + CXX_FLAGS + list(extra) + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r.stderr


def build(force=False, verbose=False, ptxas_info=False):
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    deps = _headers()
    jobs = []
    objs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s) + ".o")
        objs.append(o)
        if force or ptxas_info or _stale(o, s, deps):
            jobs.append((s, o))
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    with cf.ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        futs = {ex.submit(_compile, s, o, extra if s.endswith(".cu") else ()): s for s, o in jobs}
        for f in cf.as_completed(futs):
            msg = f.result()
            if verbose and msg:
                print(f"[{os.path.basename(futs[f])}]\n{msg}")
    if force or jobs or not os.path.exists(LIB) or any(
            os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        tmp = LIB + ".tmp"
        cmd = [NVCC] + ARCH + ["-shared", "-o", tmp] + objs + ["-ccbin", HOST_CXX]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    lib = build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas" in sys.argv)
    print(lib)
