"""Bias-free linear layer ``y = x @ cat(weights)^T`` with fused multi-weight projections.

The reference computes q/k/v (mint/nn/attn.py:49-53) and fc1/fc2 (mint/nn/ffn.py:13-14) as
separate ``nn.Linear`` calls. Here several weights that read the same input run as ONE GEMM
over their concatenation, and the weight gradient of each comes back as a slice of one fp32
GEMM output. Master weights stay in their own dtype (fp32); the GEMMs run in ``compute_dtype``
(bf16 under mixed precision) with fp32 accumulation; weight grads are produced in fp32 directly.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F  # noqa: N812

from mint_b200.ops import _ext
from mint_b200.ops.gemm import matmul


def _main_grad(w: torch.Tensor) -> torch.Tensor | None:
    """The fp32 gradient-bucket view of an engine-managed weight (CUDA), else None."""
    if not hasattr(w, "_mint_grad_ready"):
        return None
    g = w.grad
    if g is None or g.dtype != torch.float32 or not g.is_cuda or g.shape != getattr(w, "_orig_shape", w.shape):
        return None
    return g


# bf16 compute copies of (concatenated) fp32 master weights: key -> [stamp, copy, weights]
_CAST_CACHE: dict[tuple, list] = {}
_REFRESH_TABLES: dict[tuple, tuple[torch.Tensor, torch.Tensor, torch.Tensor, int]] = {}


def _stamp(weights: tuple[torch.Tensor, ...]) -> tuple | None:
    """Identity of the weights' current values; None disables caching (ZeRO-3 re-gathers)."""
    eng = getattr(weights[0], "_grad_engine", None)
    if eng is not None and eng.level == 3 and eng.dp > 1:
        return None
    epoch = eng.epoch if eng is not None else 0
    return (epoch, tuple(w.data_ptr() for w in weights), tuple(w._version for w in weights))


def _cast_weight(weights: tuple[torch.Tensor, ...], dtype: torch.dtype) -> torch.Tensor:
    """bf16 (compute dtype) copy of the concatenated weights, cached until the weights change."""
    if len(weights) == 1 and weights[0].dtype == dtype and weights[0].is_contiguous():
        return weights[0]
    key = (tuple(id(w) for w in weights), dtype)
    stamp = _stamp(weights)
    if stamp is not None:
        hit = _CAST_CACHE.get(key)
        if hit is not None and hit[0] == stamp:
            return hit[1]
    if len(weights) == 1:
        out = weights[0].detach().to(dtype).contiguous()
    else:
        out = torch.cat([w.detach().to(dtype) for w in weights], dim=0)
    if stamp is not None:
        _CAST_CACHE[key] = [stamp, out, weights]
    return out


def refresh_weight_shadows() -> None:
    """Re-cast every cached bf16 weight copy whose fp32 master changed, in ONE kernel launch.

    Called by the optimizers after each step (the step bumps the engine epoch, so every copy is
    stale): the next forward then finds its copies current instead of casting and concatenating
    each weight group separately. Copies whose weights were re-allocated are dropped."""
    stale = []
    for key, ent in list(_CAST_CACHE.items()):
        stamp, out, weights = ent
        now = _stamp(weights)
        if now is None or now == stamp:
            continue
        if now[1] != stamp[1] or not out.is_cuda or out.dtype != torch.bfloat16:
            del _CAST_CACHE[key]  # storage moved or not a CUDA bf16 copy: rebuilt on next use
            continue
        stale.append((key, ent, now))
    if not stale or not _ext.kernels_enabled():
        return
    segs = []
    for _key, ent, _now in stale:
        out, weights = ent[1], ent[2]
        off = 0
        for w in weights:
            if w.dtype != torch.float32 or not w.is_contiguous():
                segs = None
                break
            segs.append((w.data_ptr(), out.data_ptr() + off * 2, w.numel()))
            off += w.numel()
        if segs is None:
            break
    if segs is None:  # an unusual weight: leave those copies to the lazy per-call cast
        return
    tkey = tuple(segs)
    table = _REFRESH_TABLES.get(tkey)
    dev = stale[0][1][1].device
    if table is None:
        if len(_REFRESH_TABLES) > 8:
            _REFRESH_TABLES.clear()
        rows = _ext.piece_table(segs, (4, 2))
        table = (torch.tensor([a for a, _b, _n in rows], dtype=torch.int64, device=dev),
                 torch.tensor([b for _a, b, _n in rows], dtype=torch.int64, device=dev),
                 torch.tensor([n for _a, _b, n in rows], dtype=torch.int64, device=dev),
                 _ext.PIECE_ELEMS)
        _REFRESH_TABLES[tkey] = table
    _ext.require().cast_multi(table[0], table[1], table[2], table[3])
    for _key, ent, now in stale:
        ent[0] = now


def weight_grads(weights: tuple[torch.Tensor, ...], want: list[bool], dy2: torch.Tensor,
                 x2: torch.Tensor) -> list[torch.Tensor | None]:
    """Gradients of ``y = x @ cat(weights)^T`` w.r.t. each weight from ``dy2 [M, sum N_i]`` and
    ``x2 [M, K]``. Weights managed by the gradient engine get theirs accumulated straight into their
    fp32 bucket views (split-K GEMMs, then the engine's ready hook) and return None; the others are
    returned as tensors."""
    grads: list[torch.Tensor | None] = [None] * len(weights)
    fused = [want[i] and _main_grad(w) is not None for i, w in enumerate(weights)]
    if any(fused):
        off = 0
        for i, w in enumerate(weights):
            rows = w.shape[0]
            if fused[i]:
                mg = _main_grad(w)
                matmul(dy2[:, off : off + rows], x2, trans_a=True, out=mg.view(rows, -1), accumulate=True)
                w._mint_grad_ready()
            off += rows
    if any(want[i] and not fused[i] for i in range(len(weights))):
        gdtype = weights[0].dtype if weights[0].dtype in (torch.float32, torch.bfloat16) else torch.float32
        dw = matmul(dy2, x2, trans_a=True, out_dtype=gdtype)
        off = 0
        for i, w in enumerate(weights):
            rows = w.shape[0]
            if want[i] and not fused[i]:
                grads[i] = dw[off : off + rows]
            off += rows
    return grads


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, dtype, *weights):  # noqa: ANN001, ANN205
        k = x.shape[-1]
        x2 = x.reshape(-1, k)
        if x2.dtype != dtype or not x2.is_contiguous():
            x2 = x2.to(dtype).contiguous()
        w = _cast_weight(weights, dtype)
        y = matmul(x2, w, trans_b=True, out_dtype=dtype)
        # weights are kept as objects (not saved tensors) so ZeRO-3 can re-materialize them
        ctx.weights = weights
        ctx.x_shape = x.shape
        ctx.x_dtype = x.dtype
        ctx.dtype = dtype
        ctx.save_for_backward(x2)
        return y.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):  # noqa: ANN001, ANN205
        (x2,) = ctx.saved_tensors
        weights = ctx.weights
        n = dy.shape[-1]
        dy2 = dy.reshape(-1, n)
        if dy2.dtype != ctx.dtype or not dy2.is_contiguous():
            dy2 = dy2.to(ctx.dtype).contiguous()
        dx = None
        if ctx.needs_input_grad[0]:
            w = _cast_weight(weights, ctx.dtype)
            dx = matmul(dy2, w, out_dtype=ctx.dtype).view(ctx.x_shape)
            if dx.dtype != ctx.x_dtype:
                dx = dx.to(ctx.x_dtype)
        want = [ctx.needs_input_grad[2 + i] for i in range(len(weights))]
        grads = weight_grads(weights, want, dy2, x2)
        return (dx, None, *grads)


def linear(x: torch.Tensor, *weights: torch.Tensor, compute_dtype: torch.dtype | None = None) -> torch.Tensor:
    """``x @ cat(weights, 0)^T`` in ``compute_dtype`` (default: x's dtype)."""
    dtype = compute_dtype or x.dtype
    if _ext.use_cuda_kernels(x):
        return _LinearFn.apply(x, dtype, *weights)
    w = weights[0] if len(weights) == 1 else torch.cat(list(weights), dim=0)
    return F.linear(x.to(dtype), w.to(dtype))
