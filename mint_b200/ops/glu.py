"""GeGLU activation ``gelu_tanh(a) * b`` (mint/nn/ffn.py:13-15) and the whole GeGLU MLP.

``geglu(ab)`` takes the fused fc1||fc2 GEMM output ``[..., 2F]`` (fc1 columns first) and
returns ``[..., F]``; the CUDA kernel computes in fp32 and rounds once to the input dtype.

``geglu_mlp(x, w1, w2, w3)`` is ``fc3(geglu(fc1(x) || fc2(x)))`` with the activation inside the
GEMMs on CUDA: the fc1||fc2 GEMM's epilogue writes ``ab`` (kept for the backward) and ``h``, and
the fc3 input-gradient GEMM's epilogue turns ``dh`` into ``dab`` without ``dh`` reaching memory
(``gemm_geglu_fwd`` / ``gemm_geglu_bwd`` in ``csrc/gemm_sm100.cu``). No separate GeGLU pass runs.
"""

from __future__ import annotations

import os

import torch
import torch.nn.functional as F  # noqa: N812

from mint_b200.ops import _ext
from mint_b200.ops.gemm import matmul
from mint_b200.ops.linear import _cast_weight, weight_grads


class _GeGLUFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ab):  # noqa: ANN001, ANN205
        C = _ext.require()
        ab2 = ab.contiguous()
        h = C.geglu_fwd(ab2)
        ctx.save_for_backward(ab2)
        return h

    @staticmethod
    def backward(ctx, dh):  # noqa: ANN001, ANN205
        C = _ext.require()
        (ab2,) = ctx.saved_tensors
        return C.geglu_bwd(dh.contiguous(), ab2)


def geglu(ab: torch.Tensor) -> torch.Tensor:
    if _ext.use_cuda_kernels(ab):
        return _GeGLUFn.apply(ab)
    a, b = ab.chunk(2, dim=-1)
    return F.gelu(a, approximate="tanh") * b


# The backward's fused form (GeGLU backward inside the fc3 input-gradient GEMM) moves the same bytes
# as the separate kernel, but inside the GEMM's epilogue, whose two loads and a transcendental per
# element then bound the GEMM: on the d12 shapes it measured 0.67 ms per layer against 0.58 ms for
# the GEMM plus the separate kernel, so it is opt-in (MINT_GEGLU_BWD_FUSED=1).
_FUSED_BWD = os.environ.get("MINT_GEGLU_BWD_FUSED", "0") == "1"


class _GeGLUMLPFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, dtype, w1, w2, w3):  # noqa: ANN001, ANN205
        C = _ext.require()
        k = x.shape[-1]
        x2 = x.reshape(-1, k)
        if x2.dtype != dtype or not x2.is_contiguous():
            x2 = x2.to(dtype).contiguous()
        w12 = _cast_weight((w1, w2), dtype)
        m, f = x2.shape[0], w1.shape[0]
        ab = torch.empty(m, 2 * f, dtype=dtype, device=x.device)
        h = torch.empty(m, f, dtype=dtype, device=x.device)
        C.gemm_geglu_fwd(x2, w12, ab, h)
        y = matmul(h, _cast_weight((w3,), dtype), trans_b=True, out_dtype=dtype)
        ctx.weights = (w1, w2, w3)  # objects, not saved tensors: ZeRO-3 may re-materialize them
        ctx.x_shape, ctx.x_dtype, ctx.dtype = x.shape, x.dtype, dtype
        ctx.save_for_backward(x2, ab, h)
        return y.view(*x.shape[:-1], w3.shape[0])

    @staticmethod
    def backward(ctx, dy):  # noqa: ANN001, ANN205
        C = _ext.require()
        x2, ab, h = ctx.saved_tensors
        w1, w2, w3 = ctx.weights
        dtype = ctx.dtype
        dy2 = dy.reshape(-1, dy.shape[-1])
        if dy2.dtype != dtype or not dy2.is_contiguous():
            dy2 = dy2.to(dtype).contiguous()
        (dw3,) = weight_grads((w3,), [ctx.needs_input_grad[4]], dy2, h)
        if _FUSED_BWD:
            dab = torch.empty_like(ab)
            C.gemm_geglu_bwd(dy2, _cast_weight((w3,), dtype), ab, dab)
        else:  # fc3 input-gradient GEMM, then the GeGLU backward kernel
            dab = C.geglu_bwd(matmul(dy2, _cast_weight((w3,), dtype), out_dtype=dtype), ab)
        dx = None
        if ctx.needs_input_grad[0]:
            dx = matmul(dab, _cast_weight((w1, w2), dtype), out_dtype=dtype).view(ctx.x_shape)
            if dx.dtype != ctx.x_dtype:
                dx = dx.to(ctx.x_dtype)
        dw1, dw2 = weight_grads((w1, w2), [ctx.needs_input_grad[2], ctx.needs_input_grad[3]], dab, x2)
        return dx, None, dw1, dw2, dw3


def geglu_mlp_fusable(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, w3: torch.Tensor,
                      dtype: torch.dtype) -> bool:
    """The fused path takes bf16 compute, hidden width a multiple of 128, 16-byte rows."""
    return (
        x.is_cuda and _ext.kernels_enabled() and dtype == torch.bfloat16 and hasattr(_ext.require(), "gemm_geglu_fwd")
        and w1.shape == w2.shape and w1.shape[0] % 128 == 0 and w1.shape[1] % 8 == 0
        and w3.shape == (w1.shape[1], w1.shape[0]) and x.shape[-1] == w1.shape[1] and x.numel() > 0
    )


def geglu_mlp(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, w3: torch.Tensor,
              compute_dtype: torch.dtype | None = None) -> torch.Tensor:
    """``fc3(gelu_tanh(fc1(x)) * fc2(x))`` with weights ``w1, w2 [F, d]``, ``w3 [d, F]``."""
    dtype = compute_dtype or x.dtype
    if geglu_mlp_fusable(x, w1, w2, w3, dtype):
        return _GeGLUMLPFn.apply(x, dtype, w1, w2, w3)
    if x.is_cuda and _ext.kernels_enabled():
        _ext.fallback("geglu_mlp", "shape or dtype without the fused kernel (unfused GEMMs + GeGLU kernel)")
    from mint_b200.ops.linear import linear  # noqa: PLC0415

    return linear(geglu(linear(x, w1, w2, compute_dtype=dtype)), w3, compute_dtype=dtype)
