"""Token embedding lookup, optionally vocab-parallel.

Reference: ``nn.Embedding`` (mint/models/gemma.py:55-57). For tensor parallelism the table is
sharded by vocabulary rows (Megatron VocabParallelEmbedding): rows outside
``[vocab_start, vocab_start + rows)`` produce zeros and the TP group sums the partial outputs.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F  # noqa: N812

from mint_b200.ops import _ext


class _EmbeddingFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, weight, vocab_start):  # noqa: ANN001, ANN205
        C = _ext.require()
        ids2 = ids.reshape(-1).contiguous()
        out = C.embedding_fwd(ids2, weight, int(vocab_start))
        ctx.save_for_backward(ids2)
        ctx.rows = weight.shape[0]
        ctx.wdtype = weight.dtype
        ctx.vocab_start = int(vocab_start)
        return out.view(*ids.shape, weight.shape[1])

    @staticmethod
    def backward(ctx, dout):  # noqa: ANN001, ANN205
        C = _ext.require()
        (ids2,) = ctx.saved_tensors
        d = dout.shape[-1]
        dw = C.embedding_bwd(dout.reshape(-1, d).contiguous(), ids2, ctx.rows, ctx.vocab_start)
        return None, dw.to(ctx.wdtype), None


def embedding(
    ids: torch.Tensor, weight: torch.Tensor, vocab_start: int = 0, *, vocab_parallel: bool = False
) -> torch.Tensor:
    if _ext.use_cuda_kernels(weight) and weight.dtype == torch.float32:
        return _EmbeddingFn.apply(ids, weight, vocab_start)
    if weight.is_cuda and _ext.kernels_enabled():
        _ext.fallback("embedding", f"{weight.dtype} weight (the kernel takes fp32)")
    if not vocab_parallel:
        return F.embedding(ids, weight)
    local = ids - vocab_start
    valid = (local >= 0) & (local < weight.shape[0])
    out = F.embedding(local.clamp(0, weight.shape[0] - 1), weight)
    return out * valid.unsqueeze(-1).to(out.dtype)
