"""ctypes binding of libmamba3_b200.so (declared in include/mamba3_b200.h).

The library is built in-tree by ``mamba3-ssm_b200/build_lib.py`` and loaded from this
directory. There is deliberately no fallback: if the library is missing or a call fails,
a RuntimeError is raised with the library's own error text.
"""

import ctypes
import os
import struct

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmamba3_b200.so")
MAX_DIMS = 6

M3_FLOAT32, M3_BFLOAT16, M3_FLOAT16 = 0, 1, 2
M3_OK, M3_ERR_INVALID_ARGUMENT, M3_ERR_UNSUPPORTED, M3_ERR_CUDA, M3_ERR_WORKSPACE = 0, 1, 2, 3, 4
M3_INT64 = 3
_DTYPE_CODE = {torch.float32: M3_FLOAT32, torch.bfloat16: M3_BFLOAT16, torch.float16: M3_FLOAT16,
               torch.int64: M3_INT64}
_STATUS = {1: "invalid argument", 2: "unsupported", 3: "CUDA error", 4: "workspace"}


class M3Tensor(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("ndim", ctypes.c_int32),
        ("shape", ctypes.c_int64 * MAX_DIMS),
        ("stride", ctypes.c_int64 * MAX_DIMS),
    ]


class M3LayerDims(ctypes.Structure):
    _fields_ = [
        ("d_model", ctypes.c_int32),
        ("d_inner", ctypes.c_int32),
        ("nheads", ctypes.c_int32),
        ("headdim", ctypes.c_int32),
        ("d_state", ctypes.c_int32),
        ("ngroups", ctypes.c_int32),
        ("mimo_rank", ctypes.c_int32),
        ("num_rope_angles", ctypes.c_int32),
        ("rope_split", ctypes.c_int32),
        ("A_floor", ctypes.c_float),
        ("norm_eps", ctypes.c_float),
    ]


# tensor arguments are passed as plain addresses of m3_tensor records (see pack())
_P = ctypes.c_void_p
_REC = struct.Struct("<qii" + "q" * MAX_DIMS + "q" * MAX_DIMS)
assert _REC.size == ctypes.sizeof(M3Tensor)
_SIGS = {
    "m3_abi_version": ([], ctypes.c_int),
    "m3_last_error_string": ([], ctypes.c_char_p),
    "m3_siso_scan_fwd": ([_P] * 12 + [ctypes.c_void_p], ctypes.c_int),
    "m3_siso_scan_bwd_workspace_size": ([ctypes.c_int64] * 5, ctypes.c_size_t),
    "m3_siso_scan_bwd": ([_P] * 19 + [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p], ctypes.c_int),
    "m3_siso_scan_bwd_noalloc": ([_P] * 19 + [ctypes.c_void_p], ctypes.c_int),
    "m3_siso_scan_kstates_size": ([ctypes.c_int64] * 5 + [ctypes.c_int, ctypes.c_int], ctypes.c_size_t),
    "m3_siso_scan_bwd_kstates_workspace_size": ([ctypes.c_int64] * 3, ctypes.c_size_t),
    "m3_siso_scan_fwd_kstates": ([_P] * 12 + [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p], ctypes.c_int),
    "m3_siso_scan_bwd_kstates": ([_P] * 19 + [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t,
                                              ctypes.c_void_p], ctypes.c_int),
    "m3_mimo_scan_fwd": ([_P] * 14 + [ctypes.c_void_p], ctypes.c_int),
    "m3_mimo_scan_fwd_workspace_size": ([ctypes.c_int64] * 4, ctypes.c_size_t),
    "m3_mimo_scan_fwd_ws": ([_P] * 14 + [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p], ctypes.c_int),
    "m3_mimo_scan_bwd_workspace_size": ([ctypes.c_int64] * 6, ctypes.c_size_t),
    "m3_mimo_scan_bwd": ([_P] * 23 + [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p], ctypes.c_int),
    "m3_mimo_scan_bwd_ws_workspace_size": ([ctypes.c_int64] * 6, ctypes.c_size_t),
    "m3_mimo_scan_bwd_ws": ([_P] * 23 + [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t,
                                         ctypes.c_void_p], ctypes.c_int),
    "m3_siso_step": ([ctypes.c_void_p] + [_P] * 14 + [ctypes.c_void_p], ctypes.c_int),
    "m3_mimo_step": ([ctypes.c_void_p] + [_P] * 16 + [ctypes.c_void_p], ctypes.c_int),
    "m3_rmsnorm": ([_P, _P, _P, ctypes.c_float, _P, _P, ctypes.c_void_p], ctypes.c_int),
    "m3_device_timeouts": ([ctypes.c_int, ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    "m3_layer_prologue": ([ctypes.c_void_p] + [_P] * 13 + [ctypes.c_void_p], ctypes.c_int),
    "m3_silu_gate": ([_P] * 3 + [ctypes.c_void_p], ctypes.c_int),
    "m3_mimo_layer_scan_fwd": ([ctypes.c_void_p] + [_P] * 14 + [ctypes.c_int32] + [_P] * 3 +
                               [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p], ctypes.c_int),
    "m3_layer_prologue_bwd_workspace_size": ([ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64], ctypes.c_size_t),
    "m3_layer_prologue_bwd": ([ctypes.c_void_p] + [_P] * 19 + [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p],
                              ctypes.c_int),
    "m3_silu_gate_bwd": ([_P] * 5 + [ctypes.c_void_p], ctypes.c_int),
    "m3_argmax_rows": ([_P, _P, ctypes.c_void_p], ctypes.c_int),
}

_lib = None


def load():
    """Load the library once and attach the C signatures."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"{LIB_PATH} is not built; run `python mamba3-ssm_b200/build_lib.py` (nvcc, sm_100a). "
            "There is no CPU or PyTorch fallback.")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (args, res) in _SIGS.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    if lib.m3_abi_version() != 1:
        raise RuntimeError("libmamba3_b200.so ABI version mismatch")
    _lib = lib
    return lib


def exported_symbols():
    return list(_SIGS)


def tensor(t):
    """m3_tensor view of a torch tensor (None -> absent optional argument)."""
    m = M3Tensor()
    if t is None:
        m.data = None
        m.ndim = 0
        return m
    if t.dim() > MAX_DIMS:
        raise ValueError("tensor has too many dimensions for the C ABI")
    code = _DTYPE_CODE.get(t.dtype)
    if code is None:
        raise TypeError(f"dtype {t.dtype} is not supported by libmamba3_b200")
    n = t.dim()
    m.data = t.data_ptr() or (1 if t.numel() == 0 else 0)
    m.dtype = code
    m.ndim = n
    m.shape[:n] = t.shape
    m.stride[:n] = t.stride()
    return m


class Packed:
    """m3_tensor records of several tensors in one buffer (built with struct, which is
    several times cheaper than filling ctypes structures). ``ptrs[i]`` is the address
    of record i, or None for an absent optional argument; the object must stay alive
    until the call returns."""

    __slots__ = ("buf", "ptrs")

    def __init__(self, ts):
        n = len(ts)
        self.buf = ctypes.create_string_buffer(_REC.size * n)
        base = ctypes.addressof(self.buf)
        ptrs = []
        for i, t in enumerate(ts):
            if t is None:
                ptrs.append(None)
                continue
            code = _DTYPE_CODE.get(t.dtype)
            if code is None:
                raise TypeError(f"dtype {t.dtype} is not supported by libmamba3_b200")
            nd = t.dim()
            if nd > MAX_DIMS:
                raise ValueError("tensor has too many dimensions for the C ABI")
            pad = (0,) * (MAX_DIMS - nd)
            ptr = t.data_ptr() or (1 if t.numel() == 0 else 0)
            _REC.pack_into(self.buf, _REC.size * i, ptr, code, nd, *t.shape, *pad, *t.stride(), *pad)
            ptrs.append(base + _REC.size * i)
        self.ptrs = ptrs


def pack(*ts):
    return Packed(ts)


def ref(m):
    return ctypes.byref(m) if m is not None else None


def check(rc, what):
    if rc != 0:
        msg = load().m3_last_error_string().decode(errors="replace")
        raise RuntimeError(f"{what} failed ({_STATUS.get(rc, rc)}): {msg}")


def stream_of(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def device_timeouts(reset=False, device=None):
    """Nonzero once a bounded inter-warp wait of a kernel on this device gave up (outputs
    of that launch are invalid). Synchronises the device."""
    lib = load()
    v = ctypes.c_int(0)
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        check(lib.m3_device_timeouts(1 if reset else 0, ctypes.byref(v)), "m3_device_timeouts")
    return v.value
