"""CPU-only checks of the boundary: the C-ABI library loads without a GPU, exports every
entry point include/mamba3_b200.h declares, rejects bad arguments on the host, and the
Python drop-in keeps the reference's parameter names, shapes and init order."""

import ctypes
import os
import re

import numpy as np
import pytest
import torch

from conftest import ROOT, load_golden

HEADER = os.path.join(ROOT, "include", "mamba3_b200.h")


def _declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|const char\*)\s+(m3_\w+)\s*\(", src, re.M)))


@pytest.fixture(scope="module")
def lib():
    from mamba3_ssm import _lib
    return _lib.load()


def test_library_exports_every_declared_symbol(lib):
    from mamba3_ssm import _lib
    names = _declared()
    assert len(names) >= 10
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) <= set(_lib.exported_symbols()) | {"m3_abi_version", "m3_last_error_string"}
    assert lib.m3_abi_version() == 1


def test_workspace_size_queries(lib):
    from mamba3_ssm import _lib
    # CUDA-core backward: one float per position
    assert lib.m3_siso_scan_bwd_workspace_size(2, 100, 3, 32, 64) == 4 * 2 * 100 * 3
    # headdim 64 / d_state 128 may take the chunked path: room for the chunk states
    # (bf16 128 x 64 per 128-step chunk, rounded to 256 bytes), three floats per position
    # and four per (unit, chunk) (the chunk-boundary dot products of dADT)
    assert lib.m3_siso_scan_bwd_workspace_size(2, 100, 3, 64, 128) == (2 * 3 * 1 * 128 * 64 * 2 + 12 * 2 * 100 * 3
                                                                        + 16 * 2 * 3 * 1)
    bf = _lib.M3_BFLOAT16
    assert lib.m3_siso_scan_kstates_size(2, 300, 3, 64, 128, bf, bf) == 2 * 3 * 3 * 128 * 64 * 2
    assert lib.m3_siso_scan_kstates_size(2, 300, 3, 64, 128, _lib.M3_FLOAT32, bf) == 0
    assert lib.m3_siso_scan_kstates_size(2, 300, 3, 32, 128, bf, bf) == 0
    assert lib.m3_siso_scan_kstates_size(2, 300, 3, 64, 64, bf, bf) == 2 * 3 * 3 * 128 * 64 * 2
    assert lib.m3_siso_scan_kstates_size(2, 300, 3, 64, 32, bf, bf) == 0
    assert lib.m3_siso_scan_kstates_size(2, 0, 3, 64, 128, bf, bf) == 0
    assert lib.m3_siso_scan_bwd_kstates_workspace_size(2, 300, 3) == 12 * 2 * 300 * 3 + 16 * 2 * 3 * 3
    assert lib.m3_mimo_scan_bwd_workspace_size(2, 100, 3, 32, 64, 4) > 0


def test_host_validation_errors(lib):
    from mamba3_ssm import _lib
    null = _lib.M3Tensor()
    rc = lib.m3_siso_scan_fwd(*([ctypes.byref(null)] * 12), None)
    assert rc == 1
    assert b"x: missing" in lib.m3_last_error_string()
    x = _lib.M3Tensor()
    x.data = 16
    x.ndim = 3
    rc = lib.m3_siso_scan_fwd(ctypes.byref(x), *([ctypes.byref(null)] * 11), None)
    assert rc == 1 and b"x: expected" in lib.m3_last_error_string()
    dims = _lib.M3LayerDims()
    rc = lib.m3_siso_step(ctypes.byref(dims), *([ctypes.byref(null)] * 14), None)
    assert rc == 1 and b"dims" in lib.m3_last_error_string()


def _view(shape, code, data=16):
    """A descriptor of a contiguous tensor at a fake address (never dereferenced: every case
    below fails, or finishes, on the host before any device access)."""
    from mamba3_ssm import _lib
    m = _lib.M3Tensor()
    m.data, m.dtype, m.ndim = data, code, len(shape)
    st = 1
    for i in range(len(shape) - 1, -1, -1):
        m.shape[i], m.stride[i] = shape[i], st
        st *= max(shape[i], 1)
    return m


def test_mimo_layer_scan_and_prologue_host_validation(lib):
    """m3_mimo_layer_scan_fwd and m3_layer_prologue reject bad arguments on the host: no
    dims, inconsistent dims, a gate flag other than 0 / 1, B_proj without C_proj, and more
    than one B / C group (M3_ERR_UNSUPPORTED); an empty sequence without states is a no-op."""
    from mamba3_ssm import _lib
    f32, bf = _lib.M3_FLOAT32, _lib.M3_BFLOAT16
    B, L, H, P, D, R, S = 2, 0, 4, 8, 16, 2, 4
    dp = 2 * H * P + 2 * D * R + 3 * H + S

    def dims(G=1):
        d = _lib.M3LayerDims()
        d.d_model, d.d_inner, d.nheads, d.headdim, d.d_state = H * P // 2, H * P, H, P, D
        d.ngroups, d.mimo_rank, d.num_rope_angles, d.rope_split = G, R, S, 2 * S
        d.A_floor, d.norm_eps = 1e-4, 1e-5
        return d

    def args(G=1):
        dpg = 2 * H * P + 2 * D * R * G + 3 * H + S
        ins = [_view((B, L, dpg), bf), _view((B, L, H), f32), _view((B, L, H), f32), _view((B, L, H), f32),
               _view((B, L, H, S), f32), _view((H, R, D), f32), _view((H, R, D), f32), _view((D,), f32),
               _view((D,), f32), _view((H,), f32), _view((H, R, P), f32), _view((H, R, P), f32)]
        return ins

    null = _lib.M3Tensor()

    def call(d, ins, gate):
        refs = [ctypes.byref(t) for t in ins] + [ctypes.byref(null)] * 2
        out = _view((B, L, H, P), bf)
        return lib.m3_mimo_layer_scan_fwd(d, *refs, gate, ctypes.byref(out), ctypes.byref(null), ctypes.byref(null),
                                          None, 0, None)

    assert call(None, args(), 1) == _lib.M3_ERR_INVALID_ARGUMENT
    assert b"dims: missing" in lib.m3_last_error_string()
    assert call(ctypes.byref(_lib.M3LayerDims()), args(), 1) == _lib.M3_ERR_INVALID_ARGUMENT
    assert b"inconsistent" in lib.m3_last_error_string()
    assert call(ctypes.byref(dims()), args(), 2) == _lib.M3_ERR_INVALID_ARGUMENT
    assert b"gate" in lib.m3_last_error_string()
    bad = args()
    bad[5] = _view((H, R, D + 1), f32)
    assert call(ctypes.byref(dims()), bad, 1) == _lib.M3_ERR_INVALID_ARGUMENT
    assert b"B_bias" in lib.m3_last_error_string()
    assert call(ctypes.byref(dims(G=H)), args(G=H), 1) == _lib.M3_ERR_UNSUPPORTED
    assert b"one B / C group" in lib.m3_last_error_string()
    assert call(ctypes.byref(dims()), args(), 1) == _lib.M3_OK  # empty sequence, no states

    # the prologue: B_proj and C_proj both present or both absent
    zx = _view((B, L, dp), bf)
    bc = _view((B, L, R, H, D), bf)
    sc = [_view((B, L, H), f32) for _ in range(3)] + [_view((B, L, H, S), f32)]
    pars = [_view((H,), f32), _view((H, R, D), f32), _view((H, R, D), f32), _view((D,), f32), _view((D,), f32)]
    rc = lib.m3_layer_prologue(ctypes.byref(dims()), ctypes.byref(zx), *[ctypes.byref(t) for t in pars],
                               ctypes.byref(null), ctypes.byref(bc), ctypes.byref(null),
                               *[ctypes.byref(t) for t in sc], None)
    assert rc == _lib.M3_ERR_INVALID_ARGUMENT and b"C_proj: missing" in lib.m3_last_error_string()
    rc = lib.m3_layer_prologue(ctypes.byref(dims()), ctypes.byref(zx), *[ctypes.byref(t) for t in pars],
                               ctypes.byref(null), ctypes.byref(null), ctypes.byref(null),
                               *[ctypes.byref(t) for t in sc], None)
    assert rc == _lib.M3_OK  # scalars and angles only, empty sequence


def test_cpu_tensors_are_rejected():
    from mamba3_ssm import ssm_scan_siso, ssm_scan_mimo
    x = torch.randn(1, 4, 2, 8)
    B = torch.randn(1, 4, 2, 16)
    s = torch.randn(1, 4, 2)
    with pytest.raises(RuntimeError, match="no CPU path"):
        ssm_scan_siso(x, B, B, s, s, s, torch.ones(2))
    with pytest.raises(RuntimeError, match="no CPU path"):
        ssm_scan_mimo(x, B.unsqueeze(2), B.unsqueeze(2), s, s, s, torch.ones(2), torch.ones(2, 1, 8),
                      torch.ones(2, 1, 8))


@pytest.mark.parametrize("name", ["layer_c1_siso_f32", "layer_siso_f32_grad", "layer_siso_rope1_f32",
                                  "layer_mimo_f32_grad", "layer_c2_mimo_bf16", "layer_siso_bf16"])
def test_layer_init_matches_reference(name):
    """Same seed -> bit-identical parameters and state_dict keys (layer.py:107-162)."""
    from mamba3_ssm import Mamba3
    g = load_golden(name)
    cfg = {k[4:]: g[k].item() for k in g if k.startswith("cfg.")}
    seed = {"layer_c1_siso_f32": 0, "layer_siso_f32_grad": 7, "layer_siso_rope1_f32": 8,
            "layer_mimo_f32_grad": 9, "layer_c2_mimo_bf16": 0, "layer_siso_bf16": 3}[name]
    torch.manual_seed(seed)
    m = Mamba3(**cfg)
    if str(g["dtype"]) == "bfloat16":
        m = m.to(torch.bfloat16)
    sd = m.state_dict()
    assert sorted(sd) == sorted(k[2:] for k in g if k.startswith("w."))
    for k, v in sd.items():
        assert np.array_equal(v.float().numpy(), g["w." + k]), k


def test_lm_init_matches_reference():
    from mamba3_ssm import MambaConfig, MambaLMHeadModel
    g = load_golden("lm_mimo_f32")
    ssm = {k[4:]: g[k].item() for k in g if k.startswith("ssm.")}
    cfg = MambaConfig(d_model=int(g["cfg.d_model"]), n_layer=int(g["cfg.n_layer"]),
                      vocab_size=int(g["cfg.vocab_size"]), ssm_cfg=ssm)
    torch.manual_seed(6)
    m = MambaLMHeadModel(cfg)
    sd = m.state_dict()
    assert m.vocab_size == 296  # padded to a multiple of 8 (block.py:61-66)
    for k, v in sd.items():
        assert np.array_equal(v.numpy(), g["w." + k]), k


def test_allocate_inference_cache_shapes():
    from mamba3_ssm import Mamba3
    m = Mamba3(d_model=1536, d_state=64, headdim=64, is_mimo=True, mimo_rank=4)
    a, s, b = m.allocate_inference_cache(256)
    assert a.shape == (256, 48, 16) and s.shape == (256, 48, 64) and b.shape == (256, 48, 64)
    assert a.dtype == s.dtype == b.dtype == torch.float32
    m = Mamba3(d_model=128, d_state=32, headdim=32)
    a, s, b = m.allocate_inference_cache(3)
    assert s.shape == (3, 8, 32, 32) and b.shape == s.shape and a.shape == (3, 8, 8)
