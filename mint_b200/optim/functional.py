"""Optimizer math shared by ``MuonAdamW`` and ``DistMuonAdamW``.

AdamW (mint/optim/muon_adamw.py:69-92): decoupled weight decay, lerp moments, bias-corrected
step. NorMuon (muon_adamw.py:187-252): Nesterov momentum, Frobenius normalization,
Polar-Express orthogonalization (5 quintic iterations with the published coefficients of
Amsel et al., "The Polar Express", 2025), NorMuon row/column second-moment rescaling back to the
pre-normalization norm, cautious weight decay, LR x sqrt(max(1, rows/cols)).

On CUDA: AdamW is one fused kernel per bucket shard; the Polar-Express chain runs on the
tcgen05 GEMM with the ``b*A + c*A@A`` and ``a*X + B@X`` combinations folded into the GEMM
epilogue (``alpha``/``beta`` with a ``D`` operand), bf16 operands and fp32 accumulation.
"""

from __future__ import annotations

import torch

from mint_b200.ops import _ext
from mint_b200.ops.gemm import matmul

POLAR_EXPRESS_COEFFS = [
    (8.156554524902461, -22.48329292557795, 15.878769915207462),
    (4.042929935166739, -2.808917465908714, 0.5000178451051316),
    (3.8916678022926607, -2.772484153217685, 0.5060648178503393),
    (3.285753657755655, -2.3681294933425376, 0.46449024233003106),
    (2.3465413258596377, -1.7097828382687081, 0.42323551169305323),
]


@torch.no_grad()
def adamw_update(
    p: torch.Tensor,
    g: torch.Tensor,
    exp_avg: torch.Tensor,
    exp_avg_sq: torch.Tensor,
    step: int,
    lr: float,
    beta1: float,
    beta2: float,
    eps: float,
    wd: float,
    grad_scale: torch.Tensor | None = None,
) -> None:
    """``grad_scale``: optional 1-element device tensor multiplied into ``g`` (gradient clipping)."""
    if p.is_cuda and _ext.kernels_enabled():
        _ext.require().adamw_step(p, g, exp_avg, exp_avg_sq, float(lr), float(beta1), float(beta2),
                                  float(eps), float(wd), int(step), grad_scale)
        return
    if grad_scale is not None:
        g = g * grad_scale
    p.mul_(1 - lr * wd)
    exp_avg.lerp_(g, 1 - beta1)
    exp_avg_sq.lerp_(g.square(), 1 - beta2)
    bias1 = 1 - beta1**step
    bias2 = 1 - beta2**step
    denom = (exp_avg_sq / bias2).sqrt() + eps
    p.add_(exp_avg / denom, alpha=-(lr / bias1))


@torch.no_grad()
def polar_express(g: torch.Tensor, ns_steps: int) -> torch.Tensor:
    """Orthogonalize a 2-D matrix: ``X <- X / (1.01 ||X||_F + 1e-6)`` then ``ns_steps`` quintic steps."""
    tall = g.shape[0] > g.shape[1]
    if g.is_cuda and _ext.kernels_enabled():
        x = g.float()
        x = (x / (x.norm() * 1.01 + 1e-6)).to(torch.bfloat16)
        for a, b, c in POLAR_EXPRESS_COEFFS[:ns_steps]:
            if tall:
                A = matmul(x, x, trans_a=True)  # X^T X
                B = matmul(A, A, alpha=c, beta=b, d=A)
                x = matmul(x, B, alpha=1.0, beta=a, d=x)  # a X + X B
            else:
                A = matmul(x, x, trans_b=True)  # X X^T
                B = matmul(A, A, alpha=c, beta=b, d=A)
                x = matmul(B, x, alpha=1.0, beta=a, d=x)  # a X + B X
        return x.float()
    x = g.float()
    x = x / (x.norm() * 1.01 + 1e-6)
    for a, b, c in POLAR_EXPRESS_COEFFS[:ns_steps]:
        if tall:
            A = x.mT @ x
            B = b * A + c * (A @ A)
            x = a * x + x @ B
        else:
            A = x @ x.mT
            B = b * A + c * (A @ A)
            x = a * x + B @ x
    return x


@torch.no_grad()
def polar_express_chain_bf16(x: torch.Tensor, ns_steps: int) -> torch.Tensor:
    """The Polar-Express iterations on an already normalized bf16 stack ``[n, rows, cols]`` (or one
    matrix): three tcgen05 GEMM launches per iteration for the whole stack, the ``b*A + c*A@A`` and
    ``a*X + B@X`` combinations folded into the GEMM epilogues."""
    tall = x.shape[-2] > x.shape[-1]
    for a, b, c in POLAR_EXPRESS_COEFFS[:ns_steps]:
        if tall:
            A = matmul(x, x, trans_a=True)  # X^T X per matrix
            B = matmul(A, A, alpha=c, beta=b, d=A)
            x = matmul(x, B, alpha=1.0, beta=a, d=x)  # a X + X B
        else:
            A = matmul(x, x, trans_b=True)  # X X^T per matrix
            B = matmul(A, A, alpha=c, beta=b, d=A)
            x = matmul(B, x, alpha=1.0, beta=a, d=x)  # a X + B X
    return x


@torch.no_grad()
def polar_express_batched(g: torch.Tensor, ns_steps: int) -> torch.Tensor:
    """``polar_express`` on a stack ``[n, rows, cols]`` of equally shaped matrices at once.

    Each of the ``3 * ns_steps`` products is one batched tcgen05 GEMM launch for the whole stack
    (the per-matrix form needs ``3 * ns_steps`` launches per matrix)."""
    n, rows, cols = g.shape
    tall = rows > cols
    x = g.float()
    norms = x.flatten(1).norm(dim=1).view(n, 1, 1)
    x = x / (norms * 1.01 + 1e-6)
    if g.is_cuda and _ext.kernels_enabled():
        return polar_express_chain_bf16(x.to(torch.bfloat16), ns_steps).float()
    for a, b, c in POLAR_EXPRESS_COEFFS[:ns_steps]:
        if tall:
            A = x.mT @ x
            B = b * A + c * (A @ A)
            x = a * x + x @ B
        else:
            A = x @ x.mT
            B = b * A + c * (A @ A)
            x = a * x + B @ x
    return x


def _tp_gather(t: torch.Tensor, dim: int, group) -> torch.Tensor:  # noqa: ANN001
    import torch.distributed as dist  # noqa: PLC0415

    size = dist.get_world_size(group)
    parts = [torch.empty_like(t) for _ in range(size)]
    dist.all_gather(parts, t.contiguous(), group=group)
    return torch.cat(parts, dim=dim)


@torch.no_grad()
def normuon_update(
    p: torch.Tensor,
    grad: torch.Tensor,
    momentum_buffer: torch.Tensor,
    second_momentum_buffer: torch.Tensor,
    *,
    lr: float,
    momentum: float,
    beta2: float,
    wd: float,
    ns_steps: int,
    tp_group=None,  # noqa: ANN001
    tp_dim: int = 0,
) -> None:
    """One NorMuon step on a 2-D matrix ``p`` (views of ZeRO shards are fine).

    With ``tp_group``, ``p``/``grad``/``momentum_buffer`` are this rank's tensor-parallel shard of a
    matrix split along ``tp_dim``: the Nesterov gradient is all-gathered so orthogonalization and the
    NorMuon statistics see the whole matrix (``second_momentum_buffer`` has the full matrix's shape
    and is replicated), and each rank applies its slice of the update.
    """
    momentum_buffer.lerp_(grad, 1 - momentum)
    g = grad.lerp(momentum_buffer, momentum)
    shard_rows, shard_cols = p.shape
    if tp_group is not None:
        g = _tp_gather(g, tp_dim, tp_group)
    rows, cols = g.shape
    red_dim = -1 if rows >= cols else -2
    lr = lr * max(1.0, rows / cols) ** 0.5
    g = polar_express(g, ns_steps)
    v_mean = g.square().mean(dim=red_dim, keepdim=True)
    red = g.size(red_dim)
    v_norm = (v_mean.sum() * red).sqrt()
    second_momentum_buffer.lerp_(v_mean, 1 - beta2)
    step_scale = second_momentum_buffer.clamp_min(1e-10).rsqrt()
    v_norm_new = ((v_mean * red) * step_scale.square()).sum().sqrt()
    g = g * (step_scale * (v_norm / v_norm_new.clamp_min(1e-10)))
    if tp_group is not None:
        import torch.distributed as dist  # noqa: PLC0415

        r = dist.get_rank(tp_group)
        g = g.narrow(tp_dim, r * (shard_rows if tp_dim == 0 else shard_cols), shard_rows if tp_dim == 0 else shard_cols)
    pf = p.float()
    mask = (g * pf) >= 0
    p.sub_((lr * g + lr * wd * pf * mask).to(p.dtype))


@torch.no_grad()
def normuon_update_batched(
    params: list[torch.Tensor],
    grads: torch.Tensor,
    momentum_buffer: torch.Tensor,
    second_momentum_buffer: torch.Tensor,
    *,
    lr: float,
    momentum: float,
    beta2: float,
    wd: float,
    ns_steps: int,
    tp_group=None,  # noqa: ANN001
    tp_dim: int = 0,
) -> None:
    """``normuon_update`` for ``n`` equally shaped matrices in one pass.

    ``params`` are the ``n`` parameter matrices (views are fine), ``grads`` / ``momentum_buffer``
    their stacked ``[n, rows, cols]`` fp32 gradients and momenta, ``second_momentum_buffer`` the
    stacked ``[n, rows, 1]`` (tall or square) or ``[n, 1, cols]`` (wide) NorMuon statistics of the
    full matrices. Under tensor parallelism (``tp_group``) the matrices are this rank's shards along
    ``tp_dim`` and are gathered for orthogonalization as in ``normuon_update``. The result equals
    ``n`` calls of ``normuon_update`` up to floating-point summation order."""
    momentum_buffer.lerp_(grads, 1 - momentum)
    g = grads.lerp(momentum_buffer, momentum)
    n, shard_rows, shard_cols = g.shape
    if tp_group is not None:
        g = _tp_gather(g, 1 + tp_dim, tp_group)
    _, rows, cols = g.shape
    red_dim = -1 if rows >= cols else -2
    lr = lr * max(1.0, rows / cols) ** 0.5
    g = polar_express_batched(g, ns_steps)
    v_mean = g.square().mean(dim=red_dim, keepdim=True)
    red = g.size(red_dim)
    v_norm = (v_mean.sum(dim=(1, 2), keepdim=True) * red).sqrt()
    second_momentum_buffer.lerp_(v_mean, 1 - beta2)
    step_scale = second_momentum_buffer.clamp_min(1e-10).rsqrt()
    v_norm_new = ((v_mean * red) * step_scale.square()).sum(dim=(1, 2), keepdim=True).sqrt()
    g = g * (step_scale * (v_norm / v_norm_new.clamp_min(1e-10)))
    if tp_group is not None:
        import torch.distributed as dist  # noqa: PLC0415

        r = dist.get_rank(tp_group)
        size = shard_rows if tp_dim == 0 else shard_cols
        g = g.narrow(1 + tp_dim, r * size, size)
    pf = torch.stack([p.float() for p in params]) if len(params) > 1 else params[0].float().unsqueeze(0)
    mask = (g * pf) >= 0
    new = pf - (lr * g + lr * wd * pf * mask)
    torch._foreach_copy_(params, list(new.to(params[0].dtype).unbind(0)))


class NorMuonStack:
    """Device-side NorMuon for ``n`` equally shaped whole matrices whose gradients and parameters
    live anywhere in device memory (gradient-engine bucket views), with no stacking copies.

    One step is: ``normuon_prep`` (momentum, Nesterov, the clip coefficient read on the device,
    per-matrix squared norm; the Nesterov gradient overwrites the gradient), ``normuon_cast``
    (Frobenius normalization into a bf16 stack), the Polar-Express GEMM chain, ``normuon_stats`` /
    ``normuon_scale`` (row or column second moments, the NorMuon rescale back to the pre-norm
    Frobenius norm) and ``normuon_apply`` (update with cautious weight decay). Same math as
    ``normuon_update_batched``; the pointer tables are rebuilt only when a view moves."""

    def __init__(self, params: list[torch.Tensor], grads: list[torch.Tensor], mb: torch.Tensor, smb: torch.Tensor,
                 tp_group=None, tp_dim: int = 0) -> None:  # noqa: ANN001
        """``params`` / ``grads``: this rank's matrices (tensor-parallel shards along ``tp_dim`` when
        ``tp_group`` is given); ``smb``: ``[n, J]`` second moments of the FULL matrices."""
        import torch.distributed as dist  # noqa: PLC0415

        self.n = len(params)
        self.shard_rows, self.shard_cols = params[0].shape
        self.tp_group, self.tp_dim = tp_group, tp_dim
        self.tp = dist.get_world_size(tp_group) if tp_group is not None else 1
        self.tp_rank = dist.get_rank(tp_group) if tp_group is not None else 0
        self.rows = self.shard_rows * (self.tp if tp_dim == 0 else 1)
        self.cols = self.shard_cols * (self.tp if tp_dim == 1 else 1)
        dev = params[0].device
        self.key = None
        self.mb = mb
        self.smb = smb
        self.sumsq = torch.zeros(self.n, dtype=torch.float32, device=dev)
        self.x = torch.empty(self.n, self.rows, self.cols, dtype=torch.bfloat16, device=dev)
        if self.tp > 1:  # this rank's normalized shards, all-gathered into x
            self.x_local = torch.empty(self.n, self.shard_rows, self.shard_cols, dtype=torch.bfloat16, device=dev)
            self.x_gather = torch.empty(self.tp * self.n * self.shard_rows * self.shard_cols, dtype=torch.bfloat16,
                                        device=dev)
        j = self.rows if self.rows >= self.cols else self.cols
        self.scale = torch.empty(self.n, j, dtype=torch.float32, device=dev)
        self.bind(params, grads)

    @staticmethod
    def supported(params: list[torch.Tensor], grads: list[torch.Tensor]) -> bool:
        """Device path: CUDA fp32 contiguous 16-byte-aligned matrices whose (shard) columns are a
        multiple of 8 (16-byte bf16 rows for the Polar-Express GEMMs and the update kernel)."""
        if not params or not params[0].is_cuda or not _ext.kernels_enabled():
            return False
        rows, cols = params[0].shape
        if cols % 8 or (rows * cols) % 8:
            return False
        for t in list(params) + list(grads):
            if t.dtype != torch.float32 or not t.is_contiguous() or t.data_ptr() % 16 or tuple(t.shape) != (rows, cols):
                return False
        return True

    def bind(self, params: list[torch.Tensor], grads: list[torch.Tensor]) -> None:
        key = (tuple(p.data_ptr() for p in params), tuple(g.data_ptr() for g in grads))
        if key == self.key:
            return
        dev = params[0].device
        self.pptrs = torch.tensor([p.data_ptr() for p in params], dtype=torch.int64, device=dev)
        self.gptrs = torch.tensor([g.data_ptr() for g in grads], dtype=torch.int64, device=dev)
        self._keep = (list(params), list(grads))  # the kernels hold raw pointers: keep the memory alive
        self.key = key

    @torch.no_grad()
    def step(self, *, lr: float, momentum: float, beta2: float, wd: float, ns_steps: int,
             grad_scale: torch.Tensor | None = None, peer_ptrs: torch.Tensor | None = None, rank: int = 0,
             world: int = 1) -> None:
        """``peer_ptrs`` ([n * world] addresses of every data-parallel rank's copy of each matrix):
        the update kernel also stores the new values there (ZeRO-2 all-gather fused)."""
        C = _ext.require()
        rows, cols = self.rows, self.cols
        rs, cs = self.shard_rows, self.shard_cols
        C.normuon_prep(self.gptrs, self.mb, self.sumsq, rs * cs, float(momentum), grad_scale)
        if self.tp == 1:
            C.normuon_cast(self.gptrs, self.sumsq, self.x)
        else:
            self._gather_full()
        x = polar_express_chain_bf16(self.x, ns_steps)
        tall = rows >= cols
        partial = C.normuon_stats(x, tall)
        red = cols if tall else rows
        C.normuon_scale(partial, self.smb, self.scale, red, float(beta2))
        lr = lr * max(1.0, rows / cols) ** 0.5
        r0 = self.tp_rank * rs if self.tp_dim == 0 and self.tp > 1 else 0
        c0 = self.tp_rank * cs if self.tp_dim == 1 and self.tp > 1 else 0
        C.normuon_apply(x, self.scale, self.pptrs, r0, c0, rs, cs, tall, float(lr), float(wd), peer_ptrs, rank, world)

    def _gather_full(self) -> None:
        """Tensor parallelism: the Frobenius norms are summed over the TP group, every rank
        normalizes its shards to bf16 and the shards are all-gathered into the full matrices (every
        rank then orthogonalizes the whole stack, so each can update its own slice)."""
        import torch.distributed as dist  # noqa: PLC0415

        C = _ext.require()
        dist.all_reduce(self.sumsq, group=self.tp_group)
        C.normuon_cast(self.gptrs, self.sumsq, self.x_local)
        dist.all_gather_into_tensor(self.x_gather, self.x_local.view(-1), group=self.tp_group)
        parts = self.x_gather.view(self.tp, self.n, self.shard_rows, self.shard_cols)
        if self.tp_dim == 0:
            self.x.view(self.n, self.tp, self.shard_rows, self.shard_cols).copy_(parts.transpose(0, 1))
        else:
            self.x.view(self.n, self.shard_rows, self.tp, self.shard_cols).copy_(parts.permute(1, 2, 0, 3))
