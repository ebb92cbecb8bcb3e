"""Grouped-query / multi-head attention (mint/nn/attn.py:10-141).

Bias-free q/k/v/o projections, per-head QK-RMSNorm, positional encoding, causal attention
with an optional left window. The q/k/v projections run as one GEMM over ``[Wq; Wk; Wv]``
and QK-norm + RoPE run as one fused kernel. Under tensor parallelism the module holds
``n_heads / tp`` query heads and ``n_kv_heads / tp`` KV heads (column-parallel q/k/v,
row-parallel o).
"""

from __future__ import annotations

import torch
from torch import nn

from mint_b200.kvcache.base import KVCache
from mint_b200.nn.base import compute_dtype
from mint_b200.nn.flashattn import FlashAttention
from mint_b200.nn.norm import RMSNorm
from mint_b200.nn.pos import PosEmbeddings, RoPE
from mint_b200.ops.linear import linear
from mint_b200.ops.rope import qk_norm_rope
from mint_b200.parallel import fused as fused_tp
from mint_b200.parallel import tp as tpc


class GroupedQueryAttention(nn.Module):
    def __init__(
        self,
        n_heads: int,
        n_kv_heads: int,
        head_dim: int,
        embed_dim: int,
        pos_embeddings: PosEmbeddings,
        dtype: torch.dtype,
        window_size: int = -1,
    ) -> None:
        super().__init__()
        self.n_heads = n_heads
        self.n_kv_heads = n_kv_heads
        self.head_dim = head_dim
        self.window_size = window_size
        self.pos_embeddings = pos_embeddings
        self.attention = FlashAttention(use_custom_fa=True)
        self.wq = nn.Linear(embed_dim, n_heads * head_dim, bias=False, dtype=dtype)
        self.wk = nn.Linear(embed_dim, n_kv_heads * head_dim, bias=False, dtype=dtype)
        self.wv = nn.Linear(embed_dim, n_kv_heads * head_dim, bias=False, dtype=dtype)
        self.wo = nn.Linear(n_heads * head_dim, embed_dim, bias=False, dtype=dtype)
        self.q_norm = RMSNorm(head_dim)
        self.k_norm = RMSNorm(head_dim)
        self.tp: tpc.TPInfo | None = None

    def _fusable(self) -> bool:
        return all(type(m) is nn.Linear for m in (self.wq, self.wk, self.wv)) and (
            self.pos_embeddings.fused_kind in ("rope", "none")
        )

    def _norm_rope(self, qkv: torch.Tensor, start_pos: int):  # noqa: ANN202
        """QK-RMSNorm + RoPE on the fused projection ``[B, T, (hq + 2 hkv) * hd]`` -> q, k, v."""
        pe = self.pos_embeddings
        cos, sin = pe.tables() if isinstance(pe, RoPE) else (None, None)
        q, k, v = qk_norm_rope(
            qkv, self.n_heads, self.n_kv_heads, self.head_dim, self.q_norm.scale, self.k_norm.scale, cos, sin,
            start_pos=start_pos, eps=self.q_norm.eps,
        )
        return q, k, v, None

    def _project(self, x: torch.Tensor, dt: torch.dtype, start_pos: int):  # noqa: ANN202
        bsz, seqlen = x.shape[0], x.shape[1]
        hq, hkv, hd = self.n_heads, self.n_kv_heads, self.head_dim
        if self._fusable():
            qkv = linear(x, self.wq.weight, self.wk.weight, self.wv.weight, compute_dtype=dt)
            pe = self.pos_embeddings
            if isinstance(pe, RoPE):
                cos, sin = pe.tables()
            else:
                cos = sin = None
            return self._norm_rope(qkv, start_pos)
        q = self.wq(x).view(bsz, seqlen, hq, hd)
        k = self.wk(x).view(bsz, seqlen, hkv, hd)
        v = self.wv(x).view(bsz, seqlen, hkv, hd)
        q = self.q_norm(q)
        k = self.k_norm(k)
        q, k, bias = self.pos_embeddings(q, k, start_pos=start_pos)
        return q, k, v, bias

    def forward(
        self,
        x: torch.Tensor,
        kv_cache: KVCache | None = None,
        start_pos: int = 0,
        base_attn_mask: torch.Tensor | None = None,
        doc_ids: torch.Tensor | None = None,
    ) -> torch.Tensor:
        dt = compute_dtype(x)
        # TP on CUDA: QKV GEMM with its all-gather (SP) or backward all-reduce (no SP), wo GEMM with its
        # reduce-scatter (SP) or all-reduce (no SP), each as fused kernels
        fuse = (kv_cache is None and self._fusable() and type(self.wo) is nn.Linear and dt == torch.bfloat16
                and fused_tp.enabled(self.tp, x))
        if fuse:
            bsz, seqlen = x.shape[0], x.shape[1] * (self.tp.size if self.tp.sp else 1)
            qkv = fused_tp.column_parallel_linear(x, (self.wq.weight, self.wk.weight, self.wv.weight), self.tp)
            q, k, v, bias = self._norm_rope(qkv, start_pos)
        else:
            x = tpc.enter_column_parallel(x, self.tp)
            bsz, seqlen = x.shape[0], x.shape[1]
            q, k, v, bias = self._project(x, dt, start_pos)
        if bias is not None and bias.shape[1] != q.shape[2] and self.tp is not None and self.tp.size > 1:
            per = q.shape[2]
            bias = bias[:, self.tp.rank * per : (self.tp.rank + 1) * per]
        window = (self.window_size, -1) if self.window_size > 0 else (-1, -1)
        out = self.attention(
            q, k, v, causal=True, window_size=window, kv_cache=kv_cache,
            base_attn_mask=base_attn_mask, doc_ids=doc_ids, bias=bias, start_pos=start_pos,
        )
        out = out.reshape(bsz, seqlen, -1)
        if fuse:
            return fused_tp.row_parallel_linear(out, self.wo.weight, self.tp)
        if type(self.wo) is nn.Linear:
            y = linear(out, self.wo.weight, compute_dtype=dt)
        else:
            y = self.wo(out)
        return tpc.exit_row_parallel(y, self.tp)


class MultiHeadAttention(GroupedQueryAttention):
    """MHA: every query head has its own KV head (``n_kv_heads == n_heads``)."""

    def __init__(
        self,
        n_heads: int,
        head_dim: int,
        embed_dim: int,
        pos_embeddings: PosEmbeddings,
        dtype: torch.dtype,
        window_size: int = -1,
    ) -> None:
        super().__init__(n_heads, n_heads, head_dim, embed_dim, pos_embeddings, dtype, window_size)


class MultiQueryAttention(GroupedQueryAttention):
    """MQA: a single shared KV head (``n_kv_heads == 1``)."""

    def __init__(
        self,
        n_heads: int,
        head_dim: int,
        embed_dim: int,
        pos_embeddings: PosEmbeddings,
        dtype: torch.dtype,
        window_size: int = -1,
    ) -> None:
        super().__init__(n_heads, 1, head_dim, embed_dim, pos_embeddings, dtype, window_size)
