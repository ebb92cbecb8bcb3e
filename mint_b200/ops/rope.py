"""Fused QK-RMSNorm + rotary embedding that also splits the fused QKV projection.

Reference math: per-head RMSNorm over head_dim (mint/nn/attn.py:55-56) followed by the
half-split rotation ``[x1*cos - x2*sin, x1*sin + x2*cos]`` (mint/nn/pos.py:79-90) with
positions ``start_pos + t`` (``/ scale_factor`` for LinearScaledRoPE, pos.py:93-104).
The reference runs these as ~10 eager kernels; here one pass reads the QKV GEMM output
``[B, T, (Hq + 2*Hkv) * D]`` and writes normalized, rotated ``q``/``k`` and ``v`` as
``[B, T, H, D]`` tensors.
"""

from __future__ import annotations

import torch

from mint_b200.ops import _ext
from mint_b200.ops.norm import _rms_ref


def rope_cos_sin(seq_len: int, head_dim: int, base: float, scale_factor: float = 1.0) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 ``cos, sin`` tables of shape ``[seq_len, head_dim // 2]`` (mint/nn/pos.py:66-75)."""
    channel = torch.arange(0, head_dim, 2, dtype=torch.float32)
    inv_freq = 1.0 / (base ** (channel / head_dim))
    t = torch.arange(seq_len, dtype=torch.float32) / scale_factor
    freqs = torch.outer(t, inv_freq)
    return freqs.cos(), freqs.sin()


def _rotate_ref(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    d = x.shape[-1] // 2
    x1, x2 = x[..., :d], x[..., d:]
    return torch.cat([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1)


class _QKNormRopeFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, n_q, n_kv, head_dim, q_scale, k_scale, cos, sin, start_pos, eps, use_rope):  # noqa: ANN001, ANN205
        C = _ext.require()
        B, T, _ = qkv.shape
        qkv2 = qkv.contiguous()
        q, k, v, rq, rk = C.qk_norm_rope_fwd(
            qkv2, n_q, n_kv, head_dim, q_scale, k_scale, cos, sin, int(start_pos), float(eps), bool(use_rope)
        )
        ctx.save_for_backward(qkv2, rq, rk, q_scale, k_scale, cos, sin)
        ctx.meta = (n_q, n_kv, head_dim, int(start_pos), bool(use_rope))
        return q.view(B, T, n_q, head_dim), k.view(B, T, n_kv, head_dim), v.view(B, T, n_kv, head_dim)

    @staticmethod
    def backward(ctx, dq, dk, dv):  # noqa: ANN001, ANN205
        C = _ext.require()
        qkv2, rq, rk, q_scale, k_scale, cos, sin = ctx.saved_tensors
        n_q, n_kv, head_dim, start_pos, use_rope = ctx.meta
        dq = torch.zeros_like(qkv2[..., : n_q * head_dim]) if dq is None else dq
        dk = torch.zeros_like(qkv2[..., : n_kv * head_dim]) if dk is None else dk
        dv = torch.zeros_like(qkv2[..., : n_kv * head_dim]) if dv is None else dv
        dqkv, dqs, dks = C.qk_norm_rope_bwd(
            dq.contiguous(), dk.contiguous(), dv.contiguous(), qkv2, rq, rk, q_scale, k_scale, cos, sin,
            n_q, n_kv, head_dim, start_pos, use_rope,
        )
        return dqkv, None, None, None, dqs.to(q_scale.dtype), dks.to(k_scale.dtype), None, None, None, None, None


def qk_norm_rope(
    qkv: torch.Tensor,
    n_q: int,
    n_kv: int,
    head_dim: int,
    q_scale: torch.Tensor,
    k_scale: torch.Tensor,
    cos: torch.Tensor | None,
    sin: torch.Tensor | None,
    start_pos: int = 0,
    eps: float = 1e-6,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Split ``qkv`` ([B, T, (n_q+2 n_kv) D]) into normed+rotated q, k and v, each [B, T, H, D].

    ``cos``/``sin`` are fp32 ``[>= start_pos + T, D/2]`` tables, or None for no rotation.
    """
    B, T, _ = qkv.shape
    use_rope = cos is not None
    if _ext.use_cuda_kernels(qkv):
        if cos is None:
            cos = sin = torch.zeros(1, head_dim // 2, dtype=torch.float32, device=qkv.device)
        return _QKNormRopeFn.apply(qkv, n_q, n_kv, head_dim, q_scale, k_scale, cos, sin, start_pos, eps, use_rope)
    q = qkv[..., : n_q * head_dim].reshape(B, T, n_q, head_dim)
    k = qkv[..., n_q * head_dim : (n_q + n_kv) * head_dim].reshape(B, T, n_kv, head_dim)
    v = qkv[..., (n_q + n_kv) * head_dim :].reshape(B, T, n_kv, head_dim)
    q = _rms_ref(q, q_scale, eps, None).to(qkv.dtype)
    k = _rms_ref(k, k_scale, eps, None).to(qkv.dtype)
    if use_rope:
        c = cos[start_pos : start_pos + T].to(qkv.dtype)[None, :, None, :]
        s = sin[start_pos : start_pos + T].to(qkv.dtype)[None, :, None, :]
        q = _rotate_ref(q, c, s)
        k = _rotate_ref(k, c, s)
    return q, k, v
