"""Build and call the fp32 C restatement of the reference's SISO scan loop (scan_ref.c).

Test infrastructure and CPU baseline only. ``build()`` compiles ``oracle/scan_ref.c`` with
gcc (-O3 -march=x86-64-v3 -fopenmp) into ``oracle/build/libm3ref.so``; ``siso_fwd`` runs it
on contiguous float32 numpy arrays with all host threads by default.
"""

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "scan_ref.c")
LIB = os.path.join(HERE, "build", "libm3ref.so")
_lib = None


def build(force=False):
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    tmp = LIB + ".tmp"
    cmd = ["gcc", "-O3", "-march=x86-64-v3", "-fopenmp", "-shared", "-fPIC", "-o", tmp, SRC, "-lm"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    os.replace(tmp, LIB)
    return LIB


def load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(LIB)
        fp = ctypes.POINTER(ctypes.c_float)
        lib.m3_ref_siso_fwd.argtypes = [fp] * 8 + [ctypes.c_int] * 6
        lib.m3_ref_siso_fwd.restype = ctypes.c_int
        lib.m3_ref_max_threads.restype = ctypes.c_int
        _lib = lib
    return _lib


def max_threads():
    """Host cores this process may run on (torchrun sets OMP_NUM_THREADS=1 for its ranks;
    the CPU baseline uses every core it is allowed to)."""
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:
        n = os.cpu_count() or 1
    return max(n, load().m3_ref_max_threads())


def siso_fwd(x, B, C, ADT, DT, trap, D, nthreads=0):
    """y = the reference SISO loop (fp32) for x (B,L,H,P), B/C (B,L,H,D), scalars (B,L,H)."""
    lib = load()
    arrs = [np.ascontiguousarray(a, dtype=np.float32) for a in (x, B, C, ADT, DT, trap, D)]
    Bn, L, H, P = arrs[0].shape
    Ds = arrs[1].shape[-1]
    y = np.empty((Bn, L, H, P), dtype=np.float32)
    fp = ctypes.POINTER(ctypes.c_float)
    ptrs = [a.ctypes.data_as(fp) for a in arrs] + [y.ctypes.data_as(fp)]
    rc = lib.m3_ref_siso_fwd(*ptrs, Bn, L, H, P, Ds, int(nthreads))
    if rc:
        raise MemoryError("scan_ref: allocation failed")
    return y
