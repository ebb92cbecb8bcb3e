"""LoRA adapters (mint/sft/peft/lora.py:9-58): ``y = W x + (alpha/r) * B(A(dropout(x)))`` with A
kaiming-uniform and B zero, targets matched by substring (default ``wq``, ``wv``), every non-LoRA
parameter frozen. The frozen base GEMM and the two low-rank GEMMs run through the framework's
linear op (bf16 tcgen05 GEMM on CUDA)."""

from __future__ import annotations

import math
from typing import Any

import torch
from torch import nn

from mint_b200.nn.base import compute_dtype
from mint_b200.ops.linear import linear
from mint_b200.sft.peft.base import Adapter


class LoRALinear(nn.Module):
    def __init__(self, base_layer: nn.Linear, r: int = 8, alpha: int = 16, dropout: float = 0.05) -> None:
        super().__init__()
        self.base_layer = base_layer
        self.scaling = alpha / r
        base_layer.weight.requires_grad = False
        if base_layer.bias is not None:
            base_layer.bias.requires_grad = False
        dev, dt = base_layer.weight.device, base_layer.weight.dtype
        self.lora_A = nn.Linear(base_layer.in_features, r, bias=False, device=dev, dtype=dt)
        self.lora_B = nn.Linear(r, base_layer.out_features, bias=False, device=dev, dtype=dt)
        self.dropout = nn.Dropout(dropout)
        nn.init.kaiming_uniform_(self.lora_A.weight, a=math.sqrt(5))
        nn.init.zeros_(self.lora_B.weight)

    @property
    def weight(self) -> torch.Tensor:
        return self.base_layer.weight

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        dt = compute_dtype(x)
        base = self.base_layer(x) if type(self.base_layer) is not nn.Linear else linear(x, self.base_layer.weight, compute_dtype=dt)
        low = linear(linear(self.dropout(x), self.lora_A.weight, compute_dtype=dt), self.lora_B.weight, compute_dtype=dt)
        return base + low * self.scaling


def _replace(model: nn.Module, name: str, new: nn.Module) -> None:
    parent, _, leaf = name.rpartition(".")
    setattr(model.get_submodule(parent) if parent else model, leaf, new)


class LoRA(Adapter):
    @classmethod
    def apply(cls, model: nn.Module, target_modules: list[str] | None = None, r: int = 8, alpha: int = 16,
              dropout: float = 0.05, **kwargs: Any) -> None:  # noqa: ANN401, ARG003
        targets = target_modules if target_modules is not None else ["wq", "wv"]
        for name, module in list(model.named_modules()):
            if any(t in name for t in targets) and type(module) is nn.Linear:
                _replace(model, name, LoRALinear(module, r, alpha, dropout))
        for name, p in model.named_parameters():
            if "lora" not in name:
                p.requires_grad = False
