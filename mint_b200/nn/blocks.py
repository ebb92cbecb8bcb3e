"""Sandwich-norm decoder block (mint/nn/blocks.py:11-70).

``h = x + post_attn_norm(attn(pre_attn_norm(x)))``; ``out = h + post_ffn_norm(ffn(pre_ffn_norm(h)))``.
'S' blocks attend within a left window of ``seq_len // 4``; 'L' blocks attend causally over the
whole sequence. The residual stream stays in the parameters' dtype (fp32); the post-attention
residual add and the pre-FFN norm run as one fused kernel, as does the post-FFN residual add.
"""

from __future__ import annotations

import torch
from torch import nn

from mint_b200.kvcache.base import KVCache
from mint_b200.nn.attn import GroupedQueryAttention
from mint_b200.nn.base import compute_dtype
from mint_b200.nn.ffn import GLU
from mint_b200.nn.norm import RMSNorm
from mint_b200.nn.pos import ALiBiPositionalBias, LinearScaledRoPE, NoPE, PosEmbeddings, RoPE, SinusoidalPosEmbeddings
from mint_b200.ops.norm import add_rmsnorm


def make_pos_embeddings(
    kind: str, seq_len: int, head_dim: int, n_heads: int, base: float, dtype: torch.dtype, scale: float
) -> PosEmbeddings:
    if kind == "rope":
        return RoPE(seq_len=seq_len, head_dim=head_dim, rope_base_theta=base, dtype=dtype)
    if kind == "linear_rope":
        return LinearScaledRoPE(seq_len=seq_len, head_dim=head_dim, scale_factor=scale, rope_base_theta=base, dtype=dtype)
    if kind == "nope":
        return NoPE()
    if kind == "alibi":
        return ALiBiPositionalBias(n_heads)
    if kind == "sinusoidal":
        return SinusoidalPosEmbeddings(seq_len=seq_len, head_dim=head_dim)
    raise ValueError(f"unknown positional encoding {kind!r}")


class GQAGluBlock(nn.Module):
    def __init__(
        self,
        n_heads: int,
        n_kv_heads: int,
        head_dim: int,
        embed_dim: int,
        hidden_dim: int,
        seq_len: int,
        rope_base_theta: int | float,
        dtype: torch.dtype,
        attention_type: str = "L",
        pos_embedding: str = "rope",
        rope_scale_factor: float = 4.0,
        window_divisor: int = 4,
    ) -> None:
        super().__init__()
        self.attention_type = attention_type
        self.pre_attn_norm = RMSNorm(embed_dim)
        self.post_attn_norm = RMSNorm(embed_dim)
        self.pre_ffn_norm = RMSNorm(embed_dim)
        self.post_ffn_norm = RMSNorm(embed_dim)
        pos = make_pos_embeddings(pos_embedding, seq_len, head_dim, n_heads, rope_base_theta, dtype, rope_scale_factor)
        window_size = seq_len // window_divisor if attention_type == "S" else -1
        self.gqa = GroupedQueryAttention(
            n_heads=n_heads, n_kv_heads=n_kv_heads, head_dim=head_dim, embed_dim=embed_dim,
            dtype=dtype, pos_embeddings=pos, window_size=window_size,
        )
        self.ffn = GLU(embed_dim=embed_dim, hidden_dim=hidden_dim, dtype=dtype)

    def forward(
        self,
        x: torch.Tensor,
        kv_cache: KVCache | None = None,
        start_pos: int = 0,
        base_attn_mask: torch.Tensor | None = None,
        doc_ids: torch.Tensor | None = None,
        xn: torch.Tensor | None = None,
        next_norm: RMSNorm | None = None,
        chain: bool = False,
    ) -> torch.Tensor | tuple[torch.Tensor, torch.Tensor]:
        if chain:
            return self.forward_chain(x, xn, next_norm, start_pos, base_attn_mask, doc_ids)
        dt = compute_dtype(x)
        h = self.pre_attn_norm(x, out_dtype=dt)
        a = self.gqa(h, kv_cache=kv_cache, start_pos=start_pos, base_attn_mask=base_attn_mask, doc_ids=doc_ids)
        h, hn = add_rmsnorm(x, a, self.post_attn_norm.scale, self.pre_ffn_norm.scale,
                            eps=self.post_attn_norm.eps, y_dtype=dt)
        f = self.ffn(hn)
        out, _ = add_rmsnorm(h, f, self.post_ffn_norm.scale, None, eps=self.post_ffn_norm.eps)
        return out

    def forward_chain(
        self,
        x: torch.Tensor,
        xn: torch.Tensor,
        next_norm: RMSNorm | None,
        start_pos: int = 0,
        base_attn_mask: torch.Tensor | None = None,
        doc_ids: torch.Tensor | None = None,
    ) -> tuple[torch.Tensor, torch.Tensor]:
        """``forward`` with the pre-attention norm of this block's input already applied (``xn``) and
        the norm that follows the block (the next block's pre-attention norm, or the model's final
        norm) folded into the closing residual-add kernel. Returns ``(out, next_norm(out))``: every
        residual tensor then feeds one fused op, so its gradient needs no separate accumulation."""
        dt = compute_dtype(x)
        a = self.gqa(xn, kv_cache=None, start_pos=start_pos, base_attn_mask=base_attn_mask, doc_ids=doc_ids)
        h, hn = add_rmsnorm(x, a, self.post_attn_norm.scale, self.pre_ffn_norm.scale,
                            eps=self.post_attn_norm.eps, y_dtype=dt)
        f = self.ffn(hn)
        return add_rmsnorm(h, f, self.post_ffn_norm.scale, next_norm.scale if next_norm is not None else None,
                           eps=self.post_ffn_norm.eps, y_dtype=dt)
