"""B200 (sm_100a) build of the Mamba-3 selective-scan hot path.

Drop-in for the scan path of the reference package ``mamba3_ssm`` (v0.2.1): the same
module and class names (ops.ssm_scan_siso / ssm_scan_mimo, Mamba3, MambaLMHeadModel,
MambaBlock, RMSNorm, apply_rope, MambaConfig, SSMConfig), with the scans, their backward
and the decode step running as hand-written CUDA kernels behind the C ABI of
libmamba3_b200.so. There is no CPU path.
"""

from .config import MambaConfig, SSMConfig
from .layer import Mamba3
from .block import MambaLMHeadModel, MambaBlock, DecodeGraph
from .ops import RMSNorm, apply_rope, ssm_scan_siso, ssm_scan_mimo

__all__ = [
    "MambaConfig",
    "SSMConfig",
    "Mamba3",
    "MambaLMHeadModel",
    "MambaBlock",
    "DecodeGraph",
    "RMSNorm",
    "apply_rope",
    "ssm_scan_siso",
    "ssm_scan_mimo",
]
