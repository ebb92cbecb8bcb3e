"""GeGLU activation ``gelu_tanh(a) * b`` (mint/nn/ffn.py:13-15).

``geglu(ab)`` takes the fused fc1||fc2 GEMM output ``[..., 2F]`` (fc1 columns first) and
returns ``[..., F]``; the CUDA kernel computes in fp32 and rounds once to the input dtype.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F  # noqa: N812

from mint_b200.ops import _ext


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
