"""Scaled-dot-product attention with causal / sliding-window / document masking and GQA.

Mask semantics follow the reference SDPA fallback (mint/nn/flashattn.py:218-279): a query at
row ``i`` (aligned bottom-right when ``Tq < Tk``, i.e. with a KV cache) sees key ``j`` iff
``j <= i`` (causal), ``i - j <= window_left`` (when ``window_left >= 0``), ``doc[i] == doc[j]``
(when ``doc_ids`` is given) and ``attn_mask[.., i, j]`` (when given). GQA shares each KV head
among ``Hq / Hkv`` query heads. CUDA tensors run the tcgen05 FlashAttention kernels in
``mint_b200/csrc/attention_sm100.cu`` (causal + window + doc-id masking, GQA head packing);
arbitrary boolean masks and ALiBi biases use the reference path.
"""

from __future__ import annotations

import math
import weakref

import torch
import torch.nn.functional as F  # noqa: N812

from mint_b200.ops import _ext


def build_mask(
    q_len: int,
    k_len: int,
    device: torch.device,
    *,
    causal: bool,
    window_left: int,
    doc_ids: torch.Tensor | None,
    attn_mask: torch.Tensor | None,
) -> torch.Tensor | None:
    mask = None
    if doc_ids is not None:
        mask = doc_ids[:, None, :, None] == doc_ids[:, None, None, :]
    if attn_mask is not None:
        mask = attn_mask if mask is None else (mask & attn_mask)
    if causal:
        row = (k_len - q_len) + torch.arange(q_len, device=device)[:, None]
        col = torch.arange(k_len, device=device)[None, :]
        cm = col <= row
        if 0 <= window_left < k_len:
            cm = cm & ((row - col) <= window_left)
        mask = cm if mask is None else (mask & cm)
    return mask


def attention_reference(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    causal: bool = True,
    window_left: int = -1,
    doc_ids: torch.Tensor | None = None,
    attn_mask: torch.Tensor | None = None,
    bias: torch.Tensor | None = None,
    scale: float | None = None,
) -> torch.Tensor:
    """Math-mode attention in the input dtype via SDPA; q/k/v are ``[B, T, H, D]``."""
    qt, kt, vt = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    if qt.shape[1] != kt.shape[1]:
        rep = qt.shape[1] // kt.shape[1]
        kt = kt.repeat_interleave(rep, dim=1)
        vt = vt.repeat_interleave(rep, dim=1)
    mask = build_mask(qt.shape[2], kt.shape[2], q.device, causal=causal, window_left=window_left,
                      doc_ids=doc_ids, attn_mask=attn_mask)
    if bias is not None:
        fmask = bias.to(qt.dtype)
        if mask is not None:
            fmask = fmask.masked_fill(~mask, float("-inf"))
        mask = fmask
    out = F.scaled_dot_product_attention(qt, kt, vt, attn_mask=mask, scale=scale)
    return out.transpose(1, 2)


_DOC_CACHE: dict = {}


def _doc_inputs(doc_ids: torch.Tensor | None) -> tuple[torch.Tensor | None, torch.Tensor | None]:
    """int32 document ids and their per-token ``[start, end)`` runs, computed once per ids tensor
    (every layer, forward and backward, shares them). The kernels skip key / query tiles outside
    each tile's documents when a row's ids are sorted."""
    if doc_ids is None:
        return None, None
    key = (id(doc_ids), doc_ids._version, doc_ids.data_ptr(), tuple(doc_ids.shape))
    hit = _DOC_CACHE.get("entry")
    if hit is not None and hit[0] == key and hit[1]() is doc_ids:
        return hit[2], hit[3]
    d = doc_ids.to(torch.int32).contiguous()
    bounds = _ext.require().doc_bounds(d.view(d.shape[0], -1))
    _DOC_CACHE["entry"] = (key, weakref.ref(doc_ids), d, bounds)
    return d, bounds


class _FlashAttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal, window_left, doc_ids, scale, bounds):  # noqa: ANN001, ANN205
        C = _ext.require()
        o, lse = C.flash_attn_fwd(q, k, v, doc_ids, bool(causal), int(window_left), float(scale), bounds)
        ctx.save_for_backward(q, k, v, o, lse, doc_ids, bounds)
        ctx.meta = (bool(causal), int(window_left), float(scale))
        return o

    @staticmethod
    def backward(ctx, do):  # noqa: ANN001, ANN205
        C = _ext.require()
        q, k, v, o, lse, doc_ids, bounds = ctx.saved_tensors
        causal, window_left, scale = ctx.meta
        dq, dk, dv = C.flash_attn_bwd(do.contiguous(), q, k, v, o, lse, doc_ids, causal, window_left, scale,
                                      bounds)
        return dq, dk, dv, None, None, None, None, None


def _kernel_supported(q: torch.Tensor, k: torch.Tensor) -> bool:
    return (
        q.dtype in (torch.bfloat16,)
        and q.shape[-1] == 128
        and k.shape[-1] == 128
        and q.shape[2] % k.shape[2] == 0
        and q.shape[1] == k.shape[1]
        and hasattr(_ext.require(), "flash_attn_fwd")
    )


def _decode_supported(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> bool:
    """Decoding against a KV cache (fewer query than key rows, at most 16 query rows per KV head):
    the split-KV decode kernel, which reads the cache prefix in place (rows contiguous)."""
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        return False
    if q.shape[-1] != 128 or k.shape[-1] != 128 or q.shape[1] >= k.shape[1] or q.shape[2] % k.shape[2]:
        return False
    if (q.shape[2] // k.shape[2]) * q.shape[1] > 16 or k.stride() != v.stride():
        return False
    return k.stride(3) == 1 and k.stride(2) == 128 and k.stride(1) == k.shape[2] * 128 and hasattr(
        _ext.require(), "decode_attention")


def attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    causal: bool = True,
    window_left: int = -1,
    doc_ids: torch.Tensor | None = None,
    attn_mask: torch.Tensor | None = None,
    bias: torch.Tensor | None = None,
    scale: float | None = None,
) -> torch.Tensor:
    """Attention over ``[B, T, H, D]`` tensors; returns ``[B, Tq, Hq, D]``."""
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    if (
        _ext.use_cuda_kernels(q)
        and attn_mask is None
        and bias is None
        and _kernel_supported(q, k)
    ):
        d, bounds = _doc_inputs(doc_ids)
        return _FlashAttnFn.apply(q.contiguous(), k.contiguous(), v.contiguous(), causal, window_left, d, scale,
                                  bounds)
    if (
        _ext.use_cuda_kernels(q)
        and attn_mask is None
        and bias is None
        and doc_ids is None
        and _decode_supported(q, k, v)
        and not (torch.is_grad_enabled() and (q.requires_grad or k.requires_grad or v.requires_grad))
    ):
        return _ext.require().decode_attention(q.contiguous(), k, v, bool(causal), int(window_left), float(scale))
    if q.is_cuda and _ext.kernels_enabled():
        if attn_mask is not None or bias is not None:
            _ext.fallback("attention", "explicit mask or bias")
        elif q.shape[1] != k.shape[1]:
            _ext.fallback("attention", "query and key lengths differ (decode)")
        else:
            _ext.fallback("attention", "dtype / head_dim / head grouping without a kernel")
    return attention_reference(
        q, k, v, causal=causal, window_left=window_left, doc_ids=doc_ids, attn_mask=attn_mask,
        bias=bias, scale=scale,
    )
