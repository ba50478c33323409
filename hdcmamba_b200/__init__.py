"""hdcmamba_b200: HdcMamba-9v3's layer forward on NVIDIA B200 (sm_100a).

Same exports as the reference package ``hdcmamba`` (hdcmamba/__init__.py:1-13).
"""
from .model import (
    FusedNormConv1dFunction,
    HdcMamba9v3Block,
    HdcMamba9v3Model,
    fused_norm_conv1d_trainable,
)

__all__ = [
    "HdcMamba9v3Block",
    "HdcMamba9v3Model",
    "FusedNormConv1dFunction",
    "fused_norm_conv1d_trainable",
]
