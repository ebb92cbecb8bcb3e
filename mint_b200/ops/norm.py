"""RMSNorm ops: ``y = x * rsqrt(mean(x^2) + eps) * (1 + scale) [+ shift]`` computed in fp32.

Semantics follow the reference RMSNorm (mint/nn/norm.py:17-25). ``add_rmsnorm`` fuses the
sandwich-norm residual update of a block (mint/nn/blocks.py:60-70):
``h = res + rmsnorm(a; post)`` (the normed branch rounded to ``a.dtype`` first, as the reference
does) and optionally ``y = rmsnorm(h; pre)`` for the next sub-layer, in one pass.
"""

from __future__ import annotations

import torch

from mint_b200.ops import _ext


def _rms_ref(x: torch.Tensor, scale: torch.Tensor, eps: float, shift: torch.Tensor | None) -> torch.Tensor:
    xf = x.float()
    out = xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps) * (1.0 + scale.float())
    if shift is not None:
        out = out + shift.float()
    return out


def _dtype_code(dtype: torch.dtype) -> int:
    return {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[dtype]


class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, scale, eps, out_dtype):  # noqa: ANN001, ANN205
        C = _ext.require()
        x2 = x.reshape(-1, x.shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        y, rstd = C.rmsnorm_fwd(x2, scale, float(eps), _dtype_code(out_dtype))
        ctx.save_for_backward(x2, rstd, scale)
        ctx.in_shape = x.shape
        ctx.in_dtype = x.dtype
        return y.view(*x.shape[:-1], x.shape[-1])

    @staticmethod
    def backward(ctx, dy):  # noqa: ANN001, ANN205
        C = _ext.require()
        x2, rstd, scale = ctx.saved_tensors
        dy2 = dy.reshape(-1, dy.shape[-1]).contiguous()
        dx, dscale = C.rmsnorm_bwd(dy2, x2, rstd, scale, _dtype_code(ctx.in_dtype))
        return dx.view(ctx.in_shape), dscale.to(scale.dtype), None, None


def rmsnorm(
    x: torch.Tensor,
    scale: torch.Tensor,
    eps: float = 1e-6,
    shift: torch.Tensor | None = None,
    out_dtype: torch.dtype | None = None,
) -> torch.Tensor:
    out_dtype = out_dtype or x.dtype
    if shift is None and _ext.use_cuda_kernels(x):
        return _RMSNormFn.apply(x, scale, eps, out_dtype)
    if x.is_cuda and _ext.kernels_enabled():
        _ext.fallback("rmsnorm", "shift (AdaRMSNorm) term")
    return _rms_ref(x, scale, eps, shift).to(out_dtype)


class _AddRMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, res, a, post, pre, eps, y_dtype):  # noqa: ANN001, ANN205
        C = _ext.require()
        d = a.shape[-1]
        r2 = res.reshape(-1, d).contiguous()
        a2 = a.reshape(-1, d).contiguous()
        h, y, rstd_a, rstd_h = C.add_rmsnorm_fwd(
            r2, a2, post, pre, float(eps), _dtype_code(y_dtype) if pre is not None else -1
        )
        ctx.save_for_backward(a2, h, rstd_a, rstd_h, post, pre)
        ctx.has_pre = pre is not None
        ctx.shape = res.shape
        ctx.a_dtype = a.dtype
        h = h.view(res.shape)
        if pre is None:
            return h, None
        return h, y.view(*res.shape[:-1], d)

    @staticmethod
    def backward(ctx, dh, dy):  # noqa: ANN001, ANN205
        C = _ext.require()
        a2, h, rstd_a, rstd_h, post, pre = ctx.saved_tensors
        d = a2.shape[-1]
        dh2 = None if dh is None else dh.reshape(-1, d).contiguous()
        dy2 = None if (dy is None or not ctx.has_pre) else dy.reshape(-1, d).contiguous()
        dres, da, dpost, dpre = C.add_rmsnorm_bwd(dh2, dy2, a2, h, rstd_a, rstd_h, post, pre)
        return (
            dres.view(ctx.shape),
            da.view(ctx.shape),
            dpost.to(post.dtype),
            None if pre is None else dpre.to(pre.dtype),
            None,
            None,
        )


def add_rmsnorm(
    res: torch.Tensor,
    a: torch.Tensor,
    post_scale: torch.Tensor,
    pre_scale: torch.Tensor | None = None,
    eps: float = 1e-6,
    y_dtype: torch.dtype | None = None,
) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Return ``(h, y)`` with ``h = res + rmsnorm(a; post)`` and ``y = rmsnorm(h; pre)`` (or None)."""
    y_dtype = y_dtype or a.dtype
    if _ext.use_cuda_kernels(res) and res.dtype == torch.float32:
        return _AddRMSNormFn.apply(res, a, post_scale, pre_scale, eps, y_dtype)
    if res.is_cuda and _ext.kernels_enabled():
        _ext.fallback("add_rmsnorm", f"{res.dtype} residual (the kernel takes fp32)")
    n = _rms_ref(a, post_scale, eps, None).to(a.dtype)
    h = res + n
    y = None if pre_scale is None else _rms_ref(h, pre_scale, eps, None).to(y_dtype)
    return h, y
