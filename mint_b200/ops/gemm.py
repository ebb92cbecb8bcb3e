"""Dense GEMM entry point: ``C = alpha * op(A) @ op(B) + beta * D``.

Row-major convention: ``op(A)`` is ``[M, K]`` (``A`` stored ``[M, K]``, or ``[K, M]`` with
``trans_a``), ``op(B)`` is ``[K, N]`` (``B`` stored ``[K, N]``, or ``[N, K]`` with ``trans_b``).
On CUDA this runs the tcgen05/TMEM kernel in ``mint_b200/csrc/gemm_sm100.cu``: operands are
staged by TMA in 128B-swizzled shared memory (K-major or MN-major as stored, no transposes),
fp32 accumulation in tensor memory, bf16 or fp32 output with optional ``beta * D`` epilogue.
The reference runs every GEMM through ``nn.Linear`` / ``torch.matmul`` (cuBLAS).
"""

from __future__ import annotations

import torch

from mint_b200.ops import _ext


def _ref(a, b, trans_a, trans_b, alpha, beta, d, out_dtype):  # noqa: ANN001, ANN202
    a_ = a.mT if trans_a else a
    b_ = b.mT if trans_b else b
    c = alpha * (a_.float() @ b_.float())
    if d is not None and beta != 0.0:
        c = c + beta * d.float()
    return c.to(out_dtype)


def _tma_ok(t: torch.Tensor) -> bool:
    """A 2-D / 3-D bf16 operand the TMA path can read: unit inner stride, 16-byte aligned strides and base."""
    return (
        t.dtype == torch.bfloat16
        and t.stride(-1) == 1
        and all((t.stride(i) * 2) % 16 == 0 for i in range(t.dim() - 1))
        and t.data_ptr() % 16 == 0
    )


def _rows_ok(t: torch.Tensor) -> bool:
    return t.stride(-1) == 1 and all((t.stride(i) * t.element_size()) % 16 == 0 for i in range(t.dim() - 1))


def matmul(
    a: torch.Tensor,
    b: torch.Tensor,
    *,
    trans_a: bool = False,
    trans_b: bool = False,
    alpha: float = 1.0,
    beta: float = 0.0,
    d: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    out_dtype: torch.dtype | None = None,
    alpha_tensor: torch.Tensor | None = None,
    accumulate: bool = False,
) -> torch.Tensor:
    """2-D GEMM, or a batch of equally shaped GEMMs with 3-D ``[batch, rows, cols]`` operands.

    ``d`` may alias ``out`` (in-place accumulate). ``alpha_tensor`` (1-element fp32 on the device)
    multiplies ``alpha`` without a host synchronization. ``accumulate=True`` adds the product into
    the fp32 ``out`` (split-K with TMA reduce-adds on CUDA)."""
    if accumulate:
        if out is None or out.dtype != torch.float32:
            raise ValueError("accumulate=True needs an fp32 out tensor")
        if d is not None:
            raise ValueError("accumulate=True adds into out; pass no d")
    assert a.dim() == b.dim() and a.dim() in (2, 3)
    lead = tuple(a.shape[:-2])
    m = a.shape[-1] if trans_a else a.shape[-2]
    k = a.shape[-2] if trans_a else a.shape[-1]
    n = b.shape[-2] if trans_b else b.shape[-1]
    kb = b.shape[-1] if trans_b else b.shape[-2]
    if k != kb:
        raise ValueError(f"GEMM shape mismatch: op(A) is [{m},{k}], op(B) is [{kb},{n}]")
    if lead and b.shape[0] != a.shape[0]:
        raise ValueError("batched GEMM operands have different batch sizes")
    out_dtype = out.dtype if out is not None else (out_dtype or a.dtype)
    if _ext.use_cuda_kernels(a):
        C = _ext.require()
        if a.stride(-1) != 1:
            a = a.contiguous()
        if b.stride(-1) != 1:
            b = b.contiguous()
        if out is None:
            out = torch.empty((*lead, m, n), dtype=out_dtype, device=a.device)
        out_ok = _rows_ok(out)
        d_ok = d is None or _rows_ok(d)
        if _tma_ok(a) and _tma_ok(b) and out_ok and d_ok:
            C.gemm(a, b, out, d, not trans_a, trans_b, float(alpha), float(beta), alpha_tensor, accumulate)
            return out
        # operands whose rows are not 16-byte multiples cannot be described to TMA
        _ext.fallback("matmul", "operand not TMA-describable (dtype, strides or alignment)")
        res = _ref(a, b, trans_a, trans_b, alpha, beta, d, torch.float32)
        if alpha_tensor is not None:
            res = res * alpha_tensor.float()
        if accumulate:
            out.add_(res)
        else:
            out.copy_(res)
        return out
    res = _ref(a, b, trans_a, trans_b, alpha, beta, d, out_dtype)
    if alpha_tensor is not None:
        res = (res.float() * alpha_tensor.float()).to(out_dtype)
    if accumulate:
        out.add_(res.float())
        return out
    if out is not None:
        out.copy_(res)
        return out
    return res
