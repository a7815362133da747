"""Chunked prefill (not in the reference, whose generate loop calls step() once per prompt
token): Mamba3.forward(u, cache=..., return_cache=True), MambaLMHeadModel.prefill and
DecodeGraph.prefill return the decode cache of the prompt from the chunked scans. Checked
against the reference's own step() caches and step logits (golden fixtures), against
stepping through the prompt here, in two chunks against one, and for greedy decoding that
continues from the prefilled cache. Tolerances: rel 1e-4 fp32, 2e-2 bf16."""

import numpy as np
import pytest
import torch

from conftest import load_golden, rel_err
from test_gpu_layer import _layer, _lm, _t

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _np(t):
    return t.detach().float().cpu().numpy()


@pytest.fixture(autouse=True)
def _no_kernel_timeouts():
    yield
    from mamba3_ssm import _lib as L
    assert L.device_timeouts(reset=True) == 0


@pytest.mark.parametrize("grad", [False, True], ids=["fused", "autograd"])
@pytest.mark.parametrize("name", ["layer_c1_siso_f32", "layer_siso_f32_grad", "layer_mimo_f32_grad",
                                  "layer_c2_mimo_bf16", "layer_siso_bf16", "layer_siso_rope1_f32"])
def test_layer_forward_returns_step_cache(name, grad):
    g = load_golden(name)
    m = _layer(g)
    tol = 2e-2 if str(g["dtype"]) == "bfloat16" else 1e-4
    n = g["step_y"].shape[1]
    u = _t(g, "u")[:, :n].contiguous()
    with torch.set_grad_enabled(grad):
        out, (a, s, b) = m(u.requires_grad_(grad), return_cache=True)
        assert rel_err(_np(out), g["step_y"]) < tol
        assert rel_err(_np(s), g["step_ssm"]) < tol
        assert rel_err(_np(b), g["step_bx"]) < tol
        assert rel_err(_np(a), g["step_angle"]) < tol
        # the same prompt in two pieces, the second continuing from the first one's cache
        k = n // 2 + 1
        o1, c1 = m(u[:, :k], return_cache=True)
        o2, (a2, s2, b2) = m(u[:, k:], cache=c1, return_cache=True)
    assert rel_err(_np(torch.cat([o1, o2], 1)), g["step_y"]) < tol
    assert rel_err(_np(s2), g["step_ssm"]) < tol
    assert rel_err(_np(b2), g["step_bx"]) < tol
    assert rel_err(_np(a2), g["step_angle"]) < tol
    assert [t.dtype for t in (a2, s2, b2)] == [torch.float32] * 3


@pytest.mark.parametrize("name", ["lm_siso_f32", "lm_mimo_f32", "lm_mimo_bf16"])
def test_lm_prefill_matches_reference_steps(name):
    g = load_golden(name)
    m = _lm(g)
    tol = 2e-2 if str(g["dtype"]) == "bfloat16" else 1e-4
    ids = torch.from_numpy(g["ids"]).to(DEV)
    n = g["step_logits"].shape[1]
    with torch.no_grad():
        lg, cache = m.prefill(ids[:, :n])
        assert rel_err(_np(lg), g["step_logits"]) < tol
        for i, (a, s, b) in enumerate(cache):
            assert rel_err(_np(s), g[f"cache{i}.ssm"]) < tol
            assert rel_err(_np(b), g[f"cache{i}.bx"]) < tol
            assert rel_err(_np(a), g[f"cache{i}.angle"]) < tol
        # chunked: two prefills, then step() continues from the cache like the reference
        k = n // 2
        lg1, c1 = m.prefill(ids[:, :k])
        lg2, c2 = m.prefill(ids[:, k:n], c1)
        assert rel_err(_np(torch.cat([lg1, lg2], 1)), g["step_logits"]) < tol
        out, c3 = m.step(ids[:, n], c2)
        cache_s = m.allocate_inference_cache(ids.shape[0])
        for t in range(n + 1):
            out_s, cache_s = m.step(ids[:, t], cache_s)
        assert rel_err(_np(out), _np(out_s)) < tol
        for (a, s, b), (a_, s_, b_) in zip(c3, cache_s):
            assert rel_err(_np(s), _np(s_)) < tol
            assert rel_err(_np(a), _np(a_)) < tol


@pytest.mark.parametrize("name", ["lm_siso_f32", "lm_mimo_f32"])
def test_decode_graph_prefill_then_greedy(name):
    """DecodeGraph.prefill (chunked scans into the graph's static cache) followed by greedy
    replays gives the tokens of step(): fp32 models, so ties are not an issue."""
    g = load_golden(name)
    m = _lm(g)
    ids = torch.from_numpy(g["ids"]).to(DEV)
    n = g["step_logits"].shape[1]
    dg = m.decode_graph(ids.shape[0], greedy=True)
    last = dg.prefill(ids[:, :n])
    assert rel_err(_np(last), g["step_logits"][:, -1]) < 1e-4
    with torch.no_grad():
        cache = m.allocate_inference_cache(ids.shape[0])
        for t in range(n):
            out, cache = m.step(ids[:, t], cache)
        tok = out.argmax(-1)
        assert torch.equal(dg.tokens, tok)
        for _ in range(5):
            out, cache = m.step(tok, cache)
            tok = out.argmax(-1)
            assert torch.equal(dg.next(), tok)
