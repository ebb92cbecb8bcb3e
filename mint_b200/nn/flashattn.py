"""Attention dispatcher module (mint/nn/flashattn.py:18-279).

The reference chooses between flash_attn varlen, a Triton kernel (MHA, no window), an FA3 hub
binary (sm_90 only) and SDPA with a materialized mask. Here one path: ``mint_b200.ops.attention``
(the sm_100a FlashAttention kernel for causal / sliding-window / doc-id masking with GQA), with
the KV cache appended first for decoding.
"""

from __future__ import annotations

import torch
from torch import nn

from mint_b200.kvcache.base import KVCache
from mint_b200.ops.attention import attention


class FlashAttention(nn.Module):
    def __init__(self, *, use_custom_fa: bool = True) -> None:
        super().__init__()
        self.use_custom_fa = use_custom_fa

    def forward(
        self,
        q: torch.Tensor,
        k: torch.Tensor,
        v: torch.Tensor,
        *,
        causal: bool = False,
        window_size: tuple[int, int] = (-1, -1),
        kv_cache: KVCache | None = None,
        base_attn_mask: torch.Tensor | None = None,
        doc_ids: torch.Tensor | None = None,
        bias: torch.Tensor | None = None,
        start_pos: int | None = None,
    ) -> torch.Tensor:
        if kv_cache is not None:
            pos = kv_cache.seq_len if start_pos is None else start_pos
            k, v = kv_cache.update(k, v, start_pos=pos)
            k, v = k.to(q.dtype), v.to(q.dtype)
        return attention(
            q, k, v, causal=causal, window_left=window_size[0], doc_ids=doc_ids,
            attn_mask=base_attn_mask, bias=bias,
        )
