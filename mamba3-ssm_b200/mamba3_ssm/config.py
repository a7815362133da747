"""Model configuration dataclasses with the fields of the reference's
``mamba3_ssm/config.py`` (SSMConfig :11-45, MambaConfig :47-61), so that configs and
checkpoints written for the reference load unchanged."""

from dataclasses import dataclass, field
from typing import Any, Dict, List


@dataclass
class SSMConfig:
    d_state: int = 128
    expand: int = 2
    headdim: int = 64
    ngroups: int = 1
    rope_fraction: float = 0.5
    dt_min: float = 0.001
    dt_max: float = 0.1
    dt_init_floor: float = 1e-4
    A_floor: float = 1e-4
    is_mimo: bool = False
    mimo_rank: int = 4

    def to_dict(self) -> Dict[str, Any]:
        return dict(self.__dict__)


@dataclass
class MambaConfig:
    d_model: int = 2560
    d_intermediate: int = 0
    n_layer: int = 64
    vocab_size: int = 50277
    ssm_cfg: Dict[str, Any] = field(default_factory=dict)
    rms_norm: bool = True
    residual_in_fp32: bool = True
    fused_add_norm: bool = True
    pad_vocab_size_multiple: int = 8
    tie_embeddings: bool = True
    attn_layer_idx: List[int] = field(default_factory=list)
    attn_cfg: Dict[str, Any] = field(default_factory=dict)
