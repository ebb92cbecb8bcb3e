"""Positional encodings (mint/nn/pos.py:8-147): RoPE, LinearScaledRoPE, sinusoidal, NoPE, ALiBi.

``RoPE`` keeps the reference's non-persistent ``cos``/``sin`` buffers (``[1, T, 1, D/2]``) and
also exposes them as fp32 ``[T, D/2]`` tables for the fused QK-norm + RoPE kernel.
"""

from __future__ import annotations

import math
from abc import ABC, abstractmethod

import torch
from torch import nn

from mint_b200.ops.rope import _rotate_ref, rope_cos_sin


class PosEmbeddings(nn.Module, ABC):
    #: "rope" (fused rotation), "none" (fused, no rotation) or "module" (call forward)
    fused_kind: str = "module"

    @abstractmethod
    def forward(
        self, q: torch.Tensor, k: torch.Tensor, start_pos: int
    ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor | None]: ...


class SinusoidalPosEmbeddings(PosEmbeddings):
    def __init__(self, seq_len: int, head_dim: int, base: float = 10000.0) -> None:
        super().__init__()
        self.head_dim = head_dim
        pe = torch.zeros(seq_len, head_dim)
        position = torch.arange(0, seq_len, dtype=torch.float32).unsqueeze(1)
        div_term = torch.exp(torch.arange(0, head_dim, 2, dtype=torch.float32) * -(math.log(base) / head_dim))
        pe[:, 0::2] = torch.sin(position * div_term)
        pe[:, 1::2] = torch.cos(position * div_term)
        self.register_buffer("pe", pe[None, :, None, :], persistent=False)
        self.pe: torch.Tensor

    def forward(self, q, k, start_pos: int = 0):  # noqa: ANN001, ANN201
        pe_slice = self.pe[:, start_pos : start_pos + q.shape[1]].to(q.dtype)
        return q + pe_slice, k + pe_slice, None


class RoPE(PosEmbeddings):
    fused_kind = "rope"

    def __init__(
        self,
        seq_len: int,
        head_dim: int,
        rope_base_theta: int | float = 100000,
        dtype: torch.dtype = torch.float32,
        scale_factor: float = 1.0,
    ) -> None:
        super().__init__()
        self.seq_len = seq_len
        self.head_dim = head_dim
        self.base = rope_base_theta
        self.dtype = dtype
        self.scale_factor = scale_factor
        cos, sin = self._precompute_rotary_embeddings()
        self.register_buffer("cos", cos, persistent=False)
        self.register_buffer("sin", sin, persistent=False)
        self.cos: torch.Tensor
        self.sin: torch.Tensor

    def reset_parameters(self) -> None:
        cos, sin = self._precompute_rotary_embeddings()
        self.cos.copy_(cos)
        self.sin.copy_(sin)

    def _precompute_rotary_embeddings(self) -> tuple[torch.Tensor, torch.Tensor]:
        cos, sin = rope_cos_sin(self.seq_len, self.head_dim, float(self.base), self.scale_factor)
        return cos.to(self.dtype)[None, :, None, :], sin.to(self.dtype)[None, :, None, :]

    def tables(self) -> tuple[torch.Tensor, torch.Tensor]:
        """fp32 ``[T, D/2]`` cos/sin tables for the fused kernel."""
        c = self.cos.reshape(self.cos.shape[1], -1)
        s = self.sin.reshape(self.sin.shape[1], -1)
        return c.float().contiguous(), s.float().contiguous()

    @staticmethod
    def _apply_rotary_embs(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        return _rotate_ref(x, cos, sin)

    def forward(self, q, k, start_pos: int = 0):  # noqa: ANN001, ANN201
        end = start_pos + q.shape[1]
        cos = self.cos[:, start_pos:end].to(q.dtype)
        sin = self.sin[:, start_pos:end].to(q.dtype)
        return self._apply_rotary_embs(q, cos, sin), self._apply_rotary_embs(k, cos, sin), None


class LinearScaledRoPE(RoPE):
    """RoPE with positions interpolated by ``1 / scale_factor`` to extend the context window."""

    def __init__(
        self,
        seq_len: int,
        head_dim: int,
        scale_factor: float = 4.0,
        rope_base_theta: int | float = 100000,
        dtype: torch.dtype = torch.float32,
    ) -> None:
        super().__init__(seq_len, head_dim, rope_base_theta, dtype, scale_factor=scale_factor)


class NoPE(PosEmbeddings):
    fused_kind = "none"

    def forward(self, q, k, start_pos: int = 0):  # noqa: ANN001, ANN201, ARG002
        return q, k, None


class ALiBiPositionalBias(PosEmbeddings):
    """Per-head linear distance penalty returned as an additive attention bias."""

    def __init__(self, n_heads: int) -> None:
        super().__init__()
        self.n_heads = n_heads
        slopes = torch.tensor(self._get_slopes(n_heads))
        self.register_buffer("slopes", slopes[None, :, None, None], persistent=False)
        self.slopes: torch.Tensor

    def _get_slopes(self, n_heads: int) -> list[float]:
        def pow2(n: int) -> list[float]:
            start = 2 ** (-(2 ** -(math.log2(n) - 3)))
            return [start * (start**i) for i in range(n)]

        if math.log2(n_heads).is_integer():
            return pow2(n_heads)
        closest = 2 ** math.floor(math.log2(n_heads))
        return pow2(closest) + self._get_slopes(2 * closest)[0::2][: n_heads - closest]

    def forward(self, q, k, start_pos: int = 0):  # noqa: ANN001, ANN201
        t = q.shape[1]
        total = start_pos + t
        q_idx = torch.arange(start_pos, total, device=q.device)[:, None]
        k_idx = torch.arange(total, device=k.device)[None, :]
        bias = self.slopes * (k_idx - q_idx)[None, None, :, :]
        return q, k, bias.to(q.dtype)
