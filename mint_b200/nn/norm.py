"""RMSNorm module with zero-initialized ``scale`` used as ``(1 + scale)`` (mint/nn/norm.py:5-25)."""

from __future__ import annotations

import torch
from torch import nn

from mint_b200.ops.norm import rmsnorm


class RMSNorm(nn.Module):
    def __init__(self, emb_dim: int, eps: float = 1e-6, *, bias: bool = False) -> None:
        super().__init__()
        self.eps = eps
        self.scale = nn.Parameter(torch.zeros(emb_dim))
        self.shift = nn.Parameter(torch.zeros(emb_dim)) if bias else None

    def reset_parameters(self) -> None:
        nn.init.zeros_(self.scale)
        if self.shift is not None:
            nn.init.zeros_(self.shift)

    def forward(self, x: torch.Tensor, out_dtype: torch.dtype | None = None) -> torch.Tensor:
        return rmsnorm(x, self.scale, self.eps, self.shift, out_dtype=out_dtype or x.dtype)
