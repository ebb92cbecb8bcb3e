"""Preallocated per-layer KV cache ``[B, Tmax, Hkv, D]`` with ``cache_seqlens`` (mint/kvcache/base.py:4-65)."""

from __future__ import annotations

import torch


class KVCache:
    def __init__(
        self,
        max_batch_size: int = 1,
        max_seq_len: int = 2048,
        n_kv_heads: int = 4,
        head_dim: int = 128,
        dtype: torch.dtype = torch.float32,
        device: str | torch.device = "cpu",
    ) -> None:
        self.max_batch_size = max_batch_size
        self.max_seq_len = max_seq_len
        self.n_kv_heads = n_kv_heads
        self.head_dim = head_dim
        self.dtype = dtype
        self.device = device
        shape = (max_batch_size, max_seq_len, n_kv_heads, head_dim)
        self.k_cache = torch.zeros(shape, dtype=dtype, device=device)
        self.v_cache = torch.zeros(shape, dtype=dtype, device=device)
        self.cache_seqlens = torch.zeros(max_batch_size, dtype=torch.int32, device=device)
        self._len = 0  # host mirror of cache_seqlens[0] (avoids a device sync per decode step)

    def update(self, k: torch.Tensor, v: torch.Tensor, start_pos: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
        b, t = k.shape[0], k.shape[1]
        end = start_pos + t
        if end > self.max_seq_len:
            raise ValueError(f"KV cache overflow: {end} > max_seq_len={self.max_seq_len}")
        self.k_cache[:b, start_pos:end] = k.to(self.dtype)
        self.v_cache[:b, start_pos:end] = v.to(self.dtype)
        self.cache_seqlens[:b] = end
        self._len = end
        return self.k_cache[:b, :end], self.v_cache[:b, :end]

    def get(self) -> tuple[torch.Tensor, torch.Tensor]:
        return self.k_cache[:, : self._len], self.v_cache[:, : self._len]

    def get_cache_tensors(self) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        return self.k_cache, self.v_cache, self.cache_seqlens

    @property
    def seq_len(self) -> int:
        return self._len

    def reset(self) -> None:
        self.cache_seqlens.zero_()
        self._len = 0

    def clear(self) -> None:
        self.k_cache.zero_()
        self.v_cache.zero_()
        self.reset()
