"""Residual block and language model with the interface of the reference's
``mamba3_ssm/block.py``: MambaBlock (:20-29), MLPBlock (:32-43) and MambaLMHeadModel
(:46-139: forward, allocate_inference_cache, step). Parameter names match, so
reference checkpoints load with ``load_state_dict``."""

from typing import List, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .config import MambaConfig
from .layer import Mamba3
from .ops import RMSNorm, argmax_rows, rmsnorm


class MambaBlock(nn.Module):
    """x + Mamba3(RMSNorm(x))."""

    def __init__(self, d_model: int, ssm_cfg: dict, device=None, dtype=None):
        super().__init__()
        self.norm = RMSNorm(d_model)
        self.mixer = Mamba3(d_model=d_model, **ssm_cfg, device=device, dtype=dtype)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return x + self.mixer(self.norm(x))


class MLPBlock(nn.Module):
    """SwiGLU feed-forward used when d_intermediate > 0 (plain PyTorch: not on the scan path)."""

    def __init__(self, d_model: int, d_intermediate: int, device=None, dtype=None):
        super().__init__()
        f = {"device": device, "dtype": dtype}
        self.fc1 = nn.Linear(d_model, 2 * d_intermediate, bias=False, **f)
        self.fc2 = nn.Linear(d_intermediate, d_model, bias=False, **f)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        gate, val = self.fc1(x).chunk(2, dim=-1)
        return self.fc2(F.silu(gate) * val)


class MambaLMHeadModel(nn.Module):
    """Embedding -> n_layer x MambaBlock [+ MLPBlock] -> RMSNorm -> LM head (tied)."""

    def __init__(self, config: MambaConfig, device=None, dtype=None):
        f = {"device": device, "dtype": dtype}
        super().__init__()
        self.config = config
        v = config.vocab_size
        r = v % config.pad_vocab_size_multiple
        if r:
            v += config.pad_vocab_size_multiple - r
        self.vocab_size = v
        self.embedding = nn.Embedding(v, config.d_model, **f)
        self.layers = nn.ModuleList([MambaBlock(config.d_model, config.ssm_cfg, **f) for _ in range(config.n_layer)])
        if config.d_intermediate > 0:
            self.mlp_norms = nn.ModuleList([RMSNorm(config.d_model) for _ in range(config.n_layer)])
            self.mlp_layers = nn.ModuleList([MLPBlock(config.d_model, config.d_intermediate, **f)
                                             for _ in range(config.n_layer)])
        else:
            self.mlp_norms = None
            self.mlp_layers = None
        self.norm_f = RMSNorm(config.d_model)
        self.lm_head = nn.Linear(config.d_model, v, bias=False, **f)
        if device is not None:
            for mod in [self.norm_f] + [blk.norm for blk in self.layers]:
                mod.weight = nn.Parameter(mod.weight.data.to(device))
        if config.tie_embeddings:
            self.lm_head.weight = self.embedding.weight

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        x = self.embedding(input_ids)
        for i, block in enumerate(self.layers):
            x = block(x)
            if self.mlp_layers is not None:
                x = x + self.mlp_layers[i](self.mlp_norms[i](x))
        return self.lm_head(self.norm_f(x))

    def allocate_inference_cache(self, batch_size: int) -> List[Tuple[torch.Tensor, ...]]:
        return [blk.mixer.allocate_inference_cache(batch_size) for blk in self.layers]

    def prefill(self, input_ids: torch.Tensor, cache=None):
        """Run a whole prompt (B, L) through the chunked scans and return (logits (B, L, V),
        cache), the decode cache after the last token (a list of (angle, ssm, bx_prev) per
        layer, as allocate_inference_cache lays it out), ready for step(). Continues from
        ``cache`` when given (chunked prefill of a long prompt). Not in the reference, whose
        generate loop prefills one step() per prompt token; the result is that of stepping
        through the prompt."""
        x = self.embedding(input_ids)
        new_cache = []
        for i, block in enumerate(self.layers):
            out, c = block.mixer(block.norm(x), cache=None if cache is None else cache[i], return_cache=True)
            x = x + out
            new_cache.append(c)
            if self.mlp_layers is not None:
                x = x + self.mlp_layers[i](self.mlp_norms[i](x))
        return self.lm_head(self.norm_f(x)), new_cache

    def _norms_after(self, i):
        """The norm that follows layer i's mixer residual add: the MLP norm of layer i,
        the next block's norm, or norm_f."""
        if self.mlp_layers is not None:
            return self.mlp_norms[i]
        return self.layers[i + 1].norm if i + 1 < len(self.layers) else self.norm_f

    def step(self, input_ids: torch.Tensor, cache: List[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]]):
        if input_ids.dim() == 1:
            input_ids = input_ids.unsqueeze(-1)
        x = self.embedding(input_ids).squeeze(1)
        new_cache = []
        h = self.layers[0].norm(x) if self.layers else self.norm_f(x)
        for i, block in enumerate(self.layers):
            out, a, s, b = block.mixer.step(h, *cache[i])
            new_cache.append((a, s, b))
            # x = x + out, then the next norm, in one kernel
            nrm = self._norms_after(i)
            x_new = torch.empty_like(x)
            h = rmsnorm(x, nrm.weight, nrm.eps, residual=out, residual_out=x_new)
            x = x_new
            if self.mlp_layers is not None:
                nxt = self.layers[i + 1].norm if i + 1 < len(self.layers) else self.norm_f
                x_new = torch.empty_like(x)
                h = rmsnorm(x, nxt.weight, nxt.eps, residual=self.mlp_layers[i](h), residual_out=x_new)
                x = x_new
        return self.lm_head(h), new_cache

    # ------------------------------------------------------------------------------
    def decode_graph(self, batch_size: int, greedy: bool = True) -> "DecodeGraph":
        """A CUDA-graph decode loop for this model at a fixed batch size (see DecodeGraph).
        Not part of the reference interface; step() keeps the reference's semantics."""
        return DecodeGraph(self, batch_size, greedy)


class DecodeGraph:
    """Replays one whole decode step (embedding, every layer's norm / in_proj / fused step
    kernel / out_proj / residual, norm_f, lm_head and, with ``greedy``, the argmax) as one
    CUDA graph. The decode cache lives in static tensors updated in place; ``logits`` and
    ``tokens`` are static buffers overwritten by every call.

        g = model.decode_graph(batch)          # captures on the current device
        g.prefill(prompt)                      # whole prompt through the chunked scans
        for _ in range(n): tok = g.next()      # greedy: the argmax becomes the next input
    (``g.reset()`` then ``g.feed(t)`` per prompt token also works, like step().)
    """

    def __init__(self, model: "MambaLMHeadModel", batch_size: int, greedy: bool = True):
        dev = model.embedding.weight.device
        if dev.type != "cuda":
            raise RuntimeError("DecodeGraph needs the model on a CUDA device")
        self.model = model
        self.greedy = greedy
        self.tokens = torch.zeros(batch_size, dtype=torch.long, device=dev)
        self.cache = model.allocate_inference_cache(batch_size)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side), torch.no_grad():
            for _ in range(2):  # warm the caching allocator and the libraries outside the graph
                self._body()
        torch.cuda.current_stream(dev).wait_stream(side)
        self.reset()
        self.graph = torch.cuda.CUDAGraph()
        with torch.no_grad(), torch.cuda.graph(self.graph, capture_error_mode="relaxed"):
            self.logits = self._body()
        self.reset()

    def _body(self):
        m = self.model
        x = m.embedding(self.tokens)
        h = m.layers[0].norm(x) if m.layers else m.norm_f(x)
        for i, blk in enumerate(m.layers):
            out = blk.mixer.step_inplace(h, *self.cache[i])
            nrm = m._norms_after(i)
            h = rmsnorm(x, nrm.weight, nrm.eps, residual=out, residual_out=x)  # x += out; norm
            if m.mlp_layers is not None:
                nxt = m.layers[i + 1].norm if i + 1 < len(m.layers) else m.norm_f
                h = rmsnorm(x, nxt.weight, nxt.eps, residual=m.mlp_layers[i](h), residual_out=x)
        logits = m.lm_head(h)
        if self.greedy:
            argmax_rows(logits, out=self.tokens)
        return logits

    def reset(self):
        for a, s, b in self.cache:
            a.zero_()
            s.zero_()
            b.zero_()

    def prefill(self, prompt: torch.Tensor) -> torch.Tensor:
        """Replace the cache by that of the prompt (B, L), computed by MambaLMHeadModel.prefill
        (chunked scans, not one replay per token), and return the last position's logits
        (B, V); with ``greedy`` the next input token is their argmax."""
        with torch.no_grad():
            logits, cache = self.model.prefill(prompt.reshape(self.tokens.shape[0], -1))
            for dst, src in zip(self.cache, cache):
                for d, s_ in zip(dst, src):
                    d.copy_(s_)
            last = logits[:, -1]
            if self.greedy:
                argmax_rows(last, out=self.tokens)
        return last

    def feed(self, tokens: torch.Tensor) -> torch.Tensor:
        """One step on the given tokens (B,) or (B, 1); returns the static logits."""
        self.tokens.copy_(tokens.reshape(-1))
        self.graph.replay()
        return self.logits

    def next(self) -> torch.Tensor:
        """One greedy step on the previous step's argmax; returns the static token buffer."""
        self.graph.replay()
        return self.tokens
