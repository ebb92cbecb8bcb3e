"""Tensor / sequence parallel collectives as autograd functions (Megatron f/g operators).

The reference inserts SP all-gathers before every column-parallel linear and reduce-scatters
after every row-parallel one (mint/utils/parallel.py:264-358, 387-424), but has no f operator
without SP and reduce-scatters the replicated LM head's input gradient with SUM, so its TP
gradients are wrong. Here:

* column-parallel entry: SP -> all-gather along the sequence (bwd: reduce-scatter SUM);
  no SP -> identity (bwd: all-reduce SUM)                                     ["f"]
* row-parallel exit:     SP -> reduce-scatter along the sequence (bwd: all-gather);
  no SP -> all-reduce SUM (bwd: identity)                                      ["g"]
* replicated parameters whose gradient is partial across the TP group (QK-norm scales
  always; block / final norm scales under SP) are summed over TP by the gradient engine.

Activations are ``[B, T, d]``; the sequence dimension is 1. On CUDA with symmetric memory the
column entry + GEMM and the GEMM + row exit run as single fused kernels
(``mint_b200.parallel.fused``); these NCCL functions are the portable path.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch
import torch.distributed as dist


@dataclass
class TPInfo:
    group: Any
    size: int
    rank: int
    sp: bool


def _all_gather_seq(x: torch.Tensor, group: Any, size: int) -> torch.Tensor:
    xt = x.transpose(0, 1).contiguous()
    out = torch.empty((xt.shape[0] * size, *xt.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, xt, group=group)
    return out.transpose(0, 1).contiguous()


def _reduce_scatter_seq(x: torch.Tensor, group: Any, size: int) -> torch.Tensor:
    xt = x.transpose(0, 1).contiguous()
    if xt.shape[0] % size != 0:
        raise ValueError(f"sequence length {xt.shape[0]} not divisible by tp={size}")
    out = torch.empty((xt.shape[0] // size, *xt.shape[1:]), dtype=x.dtype, device=x.device)
    dist.reduce_scatter_tensor(out, xt, op=dist.ReduceOp.SUM, group=group)
    return out.transpose(0, 1).contiguous()


class _CopyToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):  # noqa: ANN001, ANN205
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        g = g.contiguous()
        dist.all_reduce(g, op=dist.ReduceOp.SUM, group=ctx.group)
        return g, None


class _ReduceFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):  # noqa: ANN001, ANN205
        out = x.contiguous().clone()
        dist.all_reduce(out, op=dist.ReduceOp.SUM, group=group)
        return out

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        return g, None


class _GatherSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, size):  # noqa: ANN001, ANN205
        ctx.group, ctx.size = group, size
        return _all_gather_seq(x, group, size)

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        return _reduce_scatter_seq(g, ctx.group, ctx.size), None, None


class _ReduceScatterSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, size):  # noqa: ANN001, ANN205
        ctx.group, ctx.size = group, size
        return _reduce_scatter_seq(x, group, size)

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        return _all_gather_seq(g, ctx.group, ctx.size), None, None


class _ScatterSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, size, rank):  # noqa: ANN001, ANN205
        ctx.group, ctx.size = group, size
        return x.chunk(size, dim=1)[rank].contiguous()

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        return _all_gather_seq(g, ctx.group, ctx.size), None, None, None


def active(tp: TPInfo | None) -> bool:
    return tp is not None and tp.size > 1


def enter_column_parallel(x: torch.Tensor, tp: TPInfo | None) -> torch.Tensor:
    if not active(tp):
        return x
    if tp.sp:
        return _GatherSeq.apply(x, tp.group, tp.size)
    return _CopyToTP.apply(x, tp.group)


def exit_row_parallel(y: torch.Tensor, tp: TPInfo | None) -> torch.Tensor:
    if not active(tp):
        return y
    if tp.sp:
        return _ReduceScatterSeq.apply(y, tp.group, tp.size)
    return _ReduceFromTP.apply(y, tp.group)


def scatter_seq(x: torch.Tensor, tp: TPInfo | None) -> torch.Tensor:
    """Keep this rank's sequence chunk (SP entry after the embedding); bwd all-gathers."""
    if not active(tp) or not tp.sp:
        return x
    return _ScatterSeq.apply(x, tp.group, tp.size, tp.rank)


def reduce_scatter_seq(x: torch.Tensor, tp: TPInfo | None) -> torch.Tensor:
    if not active(tp):
        return x
    return _ReduceScatterSeq.apply(x, tp.group, tp.size)


def reduce_from_tp(x: torch.Tensor, tp: TPInfo | None) -> torch.Tensor:
    if not active(tp):
        return x
    return _ReduceFromTP.apply(x, tp.group)


def gather_seq(x: torch.Tensor, tp: TPInfo | None) -> torch.Tensor:
    if not active(tp) or not tp.sp:
        return x
    return _GatherSeq.apply(x, tp.group, tp.size)


def copy_to_tp(x: torch.Tensor, tp: TPInfo | None) -> torch.Tensor:
    if not active(tp):
        return x
    return _CopyToTP.apply(x, tp.group)
