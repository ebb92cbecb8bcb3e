"""Masked next-token cross-entropy, fused with the LM-head GEMM on CUDA.

Reference semantics (mint/trainer/base.py:65-84): padded vocab columns (``>= vocab_size``) are
excluded, ``loss = sum(ce_t * mask_t) / max(sum(mask), 1)``.

CUDA path: ``lm_head_cross_entropy`` runs the LM-head GEMM (``logits = h @ E^T``, bf16), then ONE
kernel per row keeps the row in shared memory, computes the log-sum-exp and target logit, and
overwrites the logits with the *unscaled* gradient ``(softmax - onehot) * mask / denom``. The
backward multiplies the upstream scalar into the two GEMMs' ``alpha`` (``dh = g * dL @ E``,
``dE = g * dL^T @ h``), so the [tokens, vocab] logits are read once and written once in total and
no fp32 copy of them ever exists. Under tensor parallelism the vocabulary is sharded
(vocab-parallel LM head): per-row max / sum-exp / target logit are combined across the TP group
with three [tokens]-sized all-reduces.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist
import torch.nn.functional as F  # noqa: N812

from mint_b200.ops import _ext
from mint_b200.ops.gemm import matmul
from mint_b200.ops.linear import _cast_weight

# The LM-head weight is cast to the compute dtype on every call (forward and backward). Reusing the
# linears' cached bf16 copy here (MINT_CE_CACHED_WEIGHT=1) crashed 2-GPU runs with SIGSEGV in the
# extension call's argument conversion; 1-GPU runs were unaffected. It stays off until explained.
_CACHED_WEIGHT = os.environ.get("MINT_CE_CACHED_WEIGHT", "0") == "1"


def _head_weight(weight: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    return _cast_weight((weight,), dtype) if _CACHED_WEIGHT else weight.to(dtype).contiguous()


def masked_cross_entropy(
    logits: torch.Tensor,
    targets: torch.Tensor,
    loss_mask: torch.Tensor,
    vocab_size: int | None = None,
) -> torch.Tensor:
    """Reference-exact masked CE over (possibly vocab-padded) logits."""
    if vocab_size is not None and logits.size(-1) > vocab_size:
        cols = torch.arange(logits.size(-1), device=logits.device)
        logits = logits.masked_fill(cols >= vocab_size, float("-inf"))
    loss = F.cross_entropy(logits.reshape(-1, logits.size(-1)).float(), targets.reshape(-1), reduction="none")
    mask = loss_mask.reshape(-1).float()
    return (loss * mask).sum() / mask.sum().clamp(min=1.0)


def _tp_size(group) -> int:  # noqa: ANN001
    return 1 if group is None else dist.get_world_size(group)


class _LMHeadCEFn(torch.autograd.Function):
    """loss = masked CE(h @ E^T) with in-place gradient logits and alpha-scaled backward GEMMs."""

    @staticmethod
    def forward(ctx, h, weight, targets, mask, vocab_size, vocab_start, group, dtype):  # noqa: ANN001, ANN205
        C = _ext.require()
        d = h.shape[-1]
        h2 = h.reshape(-1, d)
        if h2.dtype != dtype or not h2.is_contiguous():
            h2 = h2.to(dtype).contiguous()
        w = _head_weight(weight, dtype)  # cached bf16 copy, refreshed once per optimizer step
        v_rows = w.shape[0]
        if v_rows % 8:
            # pad the (cast) table with zero rows so every logits row is 16-byte aligned; the
            # padded columns are excluded by ``local_valid`` below
            w = torch.cat([w, w.new_zeros(8 - v_rows % 8, w.shape[1])])
        logits = matmul(h2, w, trans_b=True, out_dtype=dtype)  # [M, V_local (padded to 8)]
        t = targets.reshape(-1).to(torch.int64).contiguous()
        m = mask.reshape(-1).to(torch.float32).contiguous()
        denom = m.sum().clamp(min=1.0)
        local_valid = max(0, min(weight.shape[0], vocab_size - vocab_start))
        if _tp_size(group) == 1:
            row_loss = C.ce_fused_fwd_bwd(logits, t, m, denom, local_valid, vocab_start)
        else:
            # pass 1: per-row local max / sum-exp / target logit; combine across the TP group
            mx, se, tl = C.ce_row_stats(logits, t, local_valid, vocab_start)
            gmx = mx.clone()
            dist.all_reduce(gmx, op=dist.ReduceOp.MAX, group=group)
            se = se * torch.exp(mx - gmx)
            dist.all_reduce(se, op=dist.ReduceOp.SUM, group=group)
            dist.all_reduce(tl, op=dist.ReduceOp.SUM, group=group)
            lse = gmx + torch.log(se)
            row_loss = lse - tl
            # pass 2: gradient logits in place
            C.ce_grad_inplace(logits, t, m, lse, denom, local_valid, vocab_start)
        loss = (row_loss * m).sum() / denom
        ctx.save_for_backward(h2, logits)
        ctx.weight = weight
        ctx.v_rows = v_rows
        ctx.h_shape = h.shape
        ctx.h_dtype = h.dtype
        ctx.dtype = dtype
        return loss

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        h2, dlogits = ctx.saved_tensors
        weight = ctx.weight
        g32 = g.reshape(1).float().contiguous()  # upstream scalar stays on the device
        w = _head_weight(weight, ctx.dtype)
        if dlogits.shape[1] != w.shape[0]:
            w = torch.cat([w, w.new_zeros(dlogits.shape[1] - w.shape[0], w.shape[1])])
        dh = matmul(dlogits, w, alpha_tensor=g32, out_dtype=ctx.dtype).view(ctx.h_shape)
        if dh.dtype != ctx.h_dtype:
            dh = dh.to(ctx.h_dtype)
        dw = None
        if ctx.needs_input_grad[1]:
            gdtype = weight.dtype if weight.dtype in (torch.float32, torch.bfloat16) else torch.float32
            dw = matmul(dlogits, h2, trans_a=True, alpha_tensor=g32, out_dtype=gdtype)[: ctx.v_rows]
        return dh, dw, None, None, None, None, None, None


def lm_head_cross_entropy(
    h: torch.Tensor,
    weight: torch.Tensor,
    targets: torch.Tensor,
    loss_mask: torch.Tensor,
    vocab_size: int,
    *,
    vocab_start: int = 0,
    group=None,  # noqa: ANN001
    compute_dtype: torch.dtype | None = None,
) -> torch.Tensor:
    """Masked CE of ``h @ weight^T`` against ``targets``; ``weight`` may be a vocab shard."""
    dtype = compute_dtype or h.dtype
    if _ext.use_cuda_kernels(h):
        return _LMHeadCEFn.apply(h, weight, targets, loss_mask, vocab_size, vocab_start, group, dtype)
    logits = F.linear(h.to(dtype), weight.to(dtype))
    if _tp_size(group) == 1:
        return masked_cross_entropy(logits, targets, loss_mask, vocab_size if logits.size(-1) > vocab_size else None)
    return vocab_parallel_cross_entropy(logits, targets, loss_mask, vocab_size, vocab_start, group)


class _LMHeadLogpFn(torch.autograd.Function):
    """Per-token ``log p(target)`` of ``h @ E^T`` (the DPO sequence log-probs).

    Forward: the LM-head GEMM writes bf16 logits, one row-statistics kernel gives max / sum-exp /
    target logit per row (combined across the TP group for a vocab shard), ``logp = tl - lse``.
    No fp32 or log-softmax copy of the [tokens, vocab] logits is made. Backward: the same in-place
    gradient kernel as the CE loss rewrites the saved logits into ``(softmax - onehot) * (-g_t)``
    with the per-token upstream gradient ``g_t`` as the row weight, then the two GEMMs give
    ``dh`` and ``dE``. The saved logits are consumed, so the graph supports one backward."""

    @staticmethod
    def forward(ctx, h, weight, targets, vocab_size, vocab_start, group, dtype):  # noqa: ANN001, ANN205
        C = _ext.require()
        d = h.shape[-1]
        h2 = h.reshape(-1, d)
        if h2.dtype != dtype or not h2.is_contiguous():
            h2 = h2.to(dtype).contiguous()
        w = _head_weight(weight, dtype)
        v_rows = w.shape[0]
        if v_rows % 8:
            w = torch.cat([w, w.new_zeros(8 - v_rows % 8, w.shape[1])])
        logits = matmul(h2, w, trans_b=True, out_dtype=dtype)
        t = targets.reshape(-1).to(torch.int64).contiguous()
        local_valid = max(0, min(weight.shape[0], vocab_size - vocab_start))
        mx, se, tl = C.ce_row_stats(logits, t, local_valid, vocab_start)
        if _tp_size(group) > 1:
            gmx = mx.clone()
            dist.all_reduce(gmx, op=dist.ReduceOp.MAX, group=group)
            se = se * torch.exp(mx - gmx)
            dist.all_reduce(se, op=dist.ReduceOp.SUM, group=group)
            dist.all_reduce(tl, op=dist.ReduceOp.SUM, group=group)
            mx = gmx
        lse = mx + torch.log(se)
        ctx.save_for_backward(h2, logits, t, lse)
        ctx.weight, ctx.v_rows, ctx.local_valid, ctx.vocab_start = weight, v_rows, local_valid, vocab_start
        ctx.h_shape, ctx.h_dtype, ctx.dtype = h.shape, h.dtype, dtype
        return (tl - lse).view(targets.shape)

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        C = _ext.require()
        h2, logits, t, lse = ctx.saved_tensors
        rows = (-g.reshape(-1)).float().contiguous()
        one = torch.ones(1, dtype=torch.float32, device=logits.device)
        C.ce_grad_inplace(logits, t, rows, lse, one, ctx.local_valid, ctx.vocab_start)
        w = _head_weight(ctx.weight, ctx.dtype)
        if logits.shape[1] != w.shape[0]:
            w = torch.cat([w, w.new_zeros(logits.shape[1] - w.shape[0], w.shape[1])])
        dh = matmul(logits, w, out_dtype=ctx.dtype).view(ctx.h_shape)
        if dh.dtype != ctx.h_dtype:
            dh = dh.to(ctx.h_dtype)
        dw = None
        if ctx.needs_input_grad[1]:
            gdtype = ctx.weight.dtype if ctx.weight.dtype in (torch.float32, torch.bfloat16) else torch.float32
            dw = matmul(logits, h2, trans_a=True, out_dtype=gdtype)[: ctx.v_rows]
        return dh, dw, None, None, None, None, None


class _VocabParallelLogp(torch.autograd.Function):
    """``log p(target)`` per token over a vocab shard, exact across the TP group (PyTorch ops)."""

    @staticmethod
    def forward(ctx, logits, targets, vocab_size, vocab_start, group):  # noqa: ANN001, ANN205
        lf = logits.float()
        v_local = lf.shape[-1]
        cols = vocab_start + torch.arange(v_local, device=lf.device)
        lf = lf.masked_fill(cols >= vocab_size, float("-inf"))
        gmx = lf.max(dim=-1).values
        dist.all_reduce(gmx, op=dist.ReduceOp.MAX, group=group)
        ex = torch.exp(lf - gmx.unsqueeze(-1))
        se = ex.sum(-1)
        dist.all_reduce(se, op=dist.ReduceOp.SUM, group=group)
        local_t = targets - vocab_start
        in_shard = (local_t >= 0) & (local_t < v_local)
        tl = torch.where(in_shard, lf.gather(-1, local_t.clamp(0, v_local - 1).unsqueeze(-1)).squeeze(-1),
                         torch.zeros_like(gmx))
        dist.all_reduce(tl, op=dist.ReduceOp.SUM, group=group)
        ctx.save_for_backward(ex, se, local_t, in_shard)
        ctx.ldtype = logits.dtype
        return tl - (gmx + torch.log(se))

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        ex, se, local_t, in_shard = ctx.saved_tensors
        p = ex / se.unsqueeze(-1)
        onehot = torch.zeros_like(p)
        onehot.scatter_(-1, local_t.clamp(0, p.shape[-1] - 1).unsqueeze(-1), in_shard.unsqueeze(-1).to(p.dtype))
        return ((onehot - p) * g.unsqueeze(-1)).to(ctx.ldtype), None, None, None, None


def lm_head_token_logps(
    h: torch.Tensor,
    weight: torch.Tensor,
    targets: torch.Tensor,
    vocab_size: int,
    *,
    vocab_start: int = 0,
    group=None,  # noqa: ANN001
    compute_dtype: torch.dtype | None = None,
) -> torch.Tensor:
    """fp32 ``log softmax(h @ weight^T)[target]`` per token, shaped like ``targets`` (ids must be
    valid vocabulary indices: mask ignored positions after the call). ``weight`` may be a vocab
    shard; the result is the full-vocabulary log-prob on every TP rank."""
    dtype = compute_dtype or h.dtype
    if _ext.use_cuda_kernels(h):
        return _LMHeadLogpFn.apply(h, weight, targets, vocab_size, vocab_start, group, dtype)
    logits = F.linear(h.to(dtype), weight.to(dtype))
    v = logits.shape[-1]
    if _tp_size(group) == 1:
        lf = logits.float()
        if v > vocab_size:
            lf = lf.masked_fill(torch.arange(v, device=lf.device) >= vocab_size, float("-inf"))
        return torch.log_softmax(lf, dim=-1).gather(-1, targets.unsqueeze(-1)).squeeze(-1)
    out = _VocabParallelLogp.apply(logits.reshape(-1, v), targets.reshape(-1), vocab_size, vocab_start, group)
    return out.view(targets.shape)


class _VocabParallelCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, targets, mask, vocab_size, vocab_start, group):  # noqa: ANN001, ANN205
        lf = logits.float()
        v_local = lf.shape[-1]
        cols = vocab_start + torch.arange(v_local, device=lf.device)
        lf = lf.masked_fill(cols >= vocab_size, float("-inf"))
        mx = lf.max(dim=-1).values
        gmx = mx.clone()
        dist.all_reduce(gmx, op=dist.ReduceOp.MAX, group=group)
        ex = torch.exp(lf - gmx.unsqueeze(-1))
        se = ex.sum(-1)
        dist.all_reduce(se, op=dist.ReduceOp.SUM, group=group)
        local_t = targets - vocab_start
        in_shard = (local_t >= 0) & (local_t < v_local)
        tl = torch.where(in_shard, lf.gather(-1, local_t.clamp(0, v_local - 1).unsqueeze(-1)).squeeze(-1),
                         torch.zeros_like(mx))
        dist.all_reduce(tl, op=dist.ReduceOp.SUM, group=group)
        lse = gmx + torch.log(se)
        m = mask.float()
        denom = m.sum().clamp(min=1.0)
        loss = ((lse - tl) * m).sum() / denom
        ctx.save_for_backward(ex, se, local_t, in_shard, m)
        ctx.denom = denom
        ctx.ldtype = logits.dtype
        return loss

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        ex, se, local_t, in_shard, m = ctx.saved_tensors
        p = ex / se.unsqueeze(-1)
        onehot = torch.zeros_like(p)
        onehot.scatter_(-1, local_t.clamp(0, p.shape[-1] - 1).unsqueeze(-1), in_shard.unsqueeze(-1).to(p.dtype))
        grad = (p - onehot) * (m / ctx.denom).unsqueeze(-1) * g
        return grad.to(ctx.ldtype), None, None, None, None, None


def vocab_parallel_cross_entropy(
    logits: torch.Tensor,
    targets: torch.Tensor,
    loss_mask: torch.Tensor,
    vocab_size: int,
    vocab_start: int,
    group,  # noqa: ANN001
) -> torch.Tensor:
    """CE over a vocab shard ``[.., V/tp]`` (columns ``vocab_start..``), exact across the TP group."""
    v = logits.shape[-1]
    return _VocabParallelCE.apply(
        logits.reshape(-1, v), targets.reshape(-1), loss_mask.reshape(-1), vocab_size, vocab_start, group
    )
