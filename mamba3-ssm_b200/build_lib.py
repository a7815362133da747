"""Build libmamba3_b200.so (the C-ABI library) in-tree for sm_100a.

    python mamba3-ssm_b200/build_lib.py [--force] [--jobs N]

Each csrc/*.cu is compiled with nvcc (-gencode arch=compute_100a,code=sm_100a) into
_build/, then linked with the static CUDA runtime into mamba3_ssm/libmamba3_b200.so, so the
library has no dependency on a libcudart of a particular version. Rebuilds only what is out
of date (object older than its source or than any header under csrc/ or include/).
"""

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "mamba3_ssm", "libmamba3_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills"]


def _nvcc():
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; set NVCC or put the CUDA toolkit on PATH")
    return cand


def _newest_header():
    hs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def _compile(nvcc, src, obj, verbose):
    cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, "-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stderr}")
    return r.stderr


def build(force=False, jobs=None, verbose=False):
    nvcc = _nvcc()
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdr = _newest_header()
    todo = []
    objs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if force or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), hdr):
            todo.append((s, o))
    logs = []
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as ex:
            futs = [ex.submit(_compile, nvcc, s, o, verbose) for s, o in todo]
            for f in futs:
                logs.append(f.result())
    if todo or not os.path.exists(LIB):
        tmp = LIB + ".tmp"
        cmd = [nvcc, *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB, "".join(logs)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--verbose", action="store_true", help="print ptxas register / spill report")
    a = ap.parse_args()
    lib, log = build(a.force, a.jobs, a.verbose)
    if log:
        sys.stderr.write(log)
    print(lib)
