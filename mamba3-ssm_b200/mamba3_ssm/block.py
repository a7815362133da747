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
from .ops import RMSNorm


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

    def step(self, input_ids: torch.Tensor, cache: List[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]]):
        if input_ids.dim() == 1:
            input_ids = input_ids.unsqueeze(-1)
        x = self.embedding(input_ids).squeeze(1)
        new_cache = []
        for i, block in enumerate(self.layers):
            out, a, s, b = block.mixer.step(block.norm(x), *cache[i])
            x = x + out
            new_cache.append((a, s, b))
            if self.mlp_layers is not None:
                x = x + self.mlp_layers[i](self.mlp_norms[i](x))
        return self.lm_head(self.norm_f(x)), new_cache
