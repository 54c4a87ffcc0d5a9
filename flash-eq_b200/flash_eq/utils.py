"""Small helpers shared by the layers (flash_eq/utils.py:8-27 in the reference)."""
from __future__ import annotations

import torch
import torch.nn as nn


def init_linear_weights(module: nn.Module) -> None:
    """Xavier-uniform weights and zero bias for every nn.Linear (use with Module.apply)."""
    if isinstance(module, nn.Linear):
        nn.init.xavier_uniform_(module.weight)
        if module.bias is not None:
            nn.init.zeros_(module.bias)


def get_epsilon(dtype: torch.dtype) -> float:
    """Numerical floor per dtype: 1e-5 for 16-bit floats, 1e-8 otherwise."""
    return 1e-5 if dtype in (torch.float16, torch.bfloat16) else 1e-8
