"""QLoRA: frozen 4-bit NF4 base weights plus LoRA adapters.

The reference ships only an API stub (mint/sft/peft/qlora.py:8-29). This implements the method of
Dettmers et al., "QLoRA" (2023): the base weight is split into blocks of 64 values, each block is
scaled by its absmax and every value is stored as the index (4 bits, two per byte) of the nearest
of the 16 NormalFloat-4 levels; the absmax scales are themselves quantized to 8 bits per block of
256 (double quantization) around their mean. Forward dequantizes the base weight to the compute
dtype and adds the LoRA branch; only ``lora_A`` / ``lora_B`` train.
"""

from __future__ import annotations

import math
from typing import Any

import torch
from torch import nn

from mint_b200.nn.base import compute_dtype
from mint_b200.ops.linear import linear
from mint_b200.sft.peft.base import Adapter

# NF4 levels: quantiles of N(0, 1) normalized to [-1, 1] with an exact zero (QLoRA paper, appendix E)
NF4_LEVELS = torch.tensor([
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
    0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0,
])
BLOCK = 64
SCALE_BLOCK = 256


def nf4_quantize(w: torch.Tensor) -> dict[str, Any]:
    flat = w.detach().float().reshape(-1)
    n = flat.numel()
    pad = (-n) % BLOCK
    if pad:
        flat = torch.cat([flat, flat.new_zeros(pad)])
    blocks = flat.view(-1, BLOCK)
    absmax = blocks.abs().amax(dim=1).clamp_min(1e-12)
    normed = blocks / absmax[:, None]
    levels = NF4_LEVELS.to(w.device)
    idx = (normed.unsqueeze(-1) - levels).abs().argmin(dim=-1).to(torch.uint8).reshape(-1)
    packed = (idx[0::2] << 4) | idx[1::2]
    # double quantization of the absmax scales
    nb = absmax.numel()
    spad = (-nb) % SCALE_BLOCK
    s = torch.cat([absmax, absmax.new_full((spad,), float(absmax.mean()))]) if spad else absmax
    offset = s.mean()
    sb = (s - offset).view(-1, SCALE_BLOCK)
    smax = sb.abs().amax(dim=1).clamp_min(1e-12)
    sq = torch.round(sb / smax[:, None] * 127).clamp(-127, 127).to(torch.int8).reshape(-1)
    return {"packed": packed, "scale_q": sq, "scale_max": smax, "scale_offset": offset, "numel": n,
            "nblocks": nb, "shape": tuple(w.shape)}


def nf4_dequantize(q: dict[str, Any], dtype: torch.dtype = torch.float32) -> torch.Tensor:
    packed = q["packed"]
    idx = torch.stack([packed >> 4, packed & 0xF], dim=1).reshape(-1).long()
    levels = NF4_LEVELS.to(packed.device)
    scales = (q["scale_q"].float().view(-1, SCALE_BLOCK) / 127 * q["scale_max"][:, None]).reshape(-1)
    absmax = scales[: q["nblocks"]] + q["scale_offset"]
    vals = levels[idx].view(-1, BLOCK) * absmax[:, None]
    return vals.reshape(-1)[: q["numel"]].view(q["shape"]).to(dtype)


class QLoRALinear(nn.Module):
    def __init__(self, base_layer: nn.Linear, r: int = 8, alpha: int = 16, dropout: float = 0.05) -> None:
        super().__init__()
        q = nf4_quantize(base_layer.weight)
        for k in ("packed", "scale_q", "scale_max"):
            self.register_buffer(k, q[k])
        self.register_buffer("scale_offset", q["scale_offset"].reshape(()))
        self.numel, self.nblocks, self.shape = q["numel"], q["nblocks"], q["shape"]
        self.in_features, self.out_features = base_layer.in_features, base_layer.out_features
        self.bias = None if base_layer.bias is None else nn.Parameter(base_layer.bias.detach().clone(), requires_grad=False)
        self.scaling = alpha / r
        dev, dt = base_layer.weight.device, base_layer.weight.dtype
        self.lora_A = nn.Linear(self.in_features, r, bias=False, device=dev, dtype=dt)
        self.lora_B = nn.Linear(r, self.out_features, bias=False, device=dev, dtype=dt)
        self.dropout = nn.Dropout(dropout)
        nn.init.kaiming_uniform_(self.lora_A.weight, a=math.sqrt(5))
        nn.init.zeros_(self.lora_B.weight)

    def dequantized_weight(self, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        q = {"packed": self.packed, "scale_q": self.scale_q, "scale_max": self.scale_max,
             "scale_offset": self.scale_offset, "numel": self.numel, "nblocks": self.nblocks, "shape": self.shape}
        return nf4_dequantize(q, dtype)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        dt = compute_dtype(x)
        w = self.dequantized_weight(dt)
        out = linear(x, w, compute_dtype=dt)
        if self.bias is not None:
            out = out + self.bias.to(out.dtype)
        low = linear(linear(self.dropout(x), self.lora_A.weight, compute_dtype=dt), self.lora_B.weight, compute_dtype=dt)
        return out + low * self.scaling


class QLoRA(Adapter):
    @classmethod
    def apply(cls, model: nn.Module, target_modules: list[str] | None = None, r: int = 8, alpha: int = 16,
              dropout: float = 0.05, **kwargs: Any) -> None:  # noqa: ANN401, ARG003
        targets = target_modules if target_modules is not None else ["wq", "wv"]
        for name, module in list(model.named_modules()):
            if any(t in name for t in targets) and type(module) is nn.Linear:
                parent, _, leaf = name.rpartition(".")
                setattr(model.get_submodule(parent) if parent else model, leaf, QLoRALinear(module, r, alpha, dropout))
        for name, p in model.named_parameters():
            if "lora" not in name:
                p.requires_grad = False
