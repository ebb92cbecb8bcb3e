"""Tensor-parallel linears with their collectives fused into the GEMM over NVLink peer memory.

The reference all-gathers the sequence-parallel activation before every column-parallel linear and
reduce-scatters after every row-parallel one with separate NCCL calls (mint/utils/parallel.py:264-319,
387-424). Here, on CUDA with symmetric memory, each of these is one sm_100a kernel
(``mint_b200/csrc/gemm_sm100.cu``, CTA-pair tcgen05 GEMM):

* column-parallel forward -- all-gather -> GEMM: this rank's sequence shard is placed in a symmetric
  gathered buffer, copy warps of the GEMM pull the peers' shards over NVLink while the tensor cores
  start on the local rows; the gathered input is kept for the weight gradient;
  backward -- GEMM -> reduce-scatter for the input gradient, local GEMM for the weight gradient;
* row-parallel forward -- GEMM -> reduce-scatter: partial output tiles of the peers' rows are pushed
  into their receive buffers from the epilogue, this rank's rows are reduced in its epilogue;
  backward -- all-gather of the output gradient -> GEMM for the input gradient, local GEMM for the
  weight gradient on the gathered output gradient.

Without sequence parallelism (replicated activations) the row-parallel exit is an all-reduce:
the GEMM -> reduce-scatter kernel writes each rank's reduced block of rows into its part of a
symmetric buffer, one push kernel stores the block into every peer's buffer and a stream barrier
over NVLink flags publishes it (the reference: ``_AllReduce`` at mint/utils/parallel.py:322-333).
The column-parallel entry is then the identity and its backward the same fused all-reduce.

Sequence-parallel activations are ``[B, T / tp, d]`` (a shard of every sequence); the gathered
layout is ``[B, T, d]`` (rows of rank p's shard of sequence b at rows ``b*T + p*T/tp ...``).
Gradients are those of the NCCL path in ``mint_b200.parallel.tp``; only the transport differs.

Buffers: the gathered input of a column-parallel forward is kept for its weight gradient in a
symmetric buffer taken from a per-group pool and handed back when that backward has run (at once
when no backward will follow: no-grad forwards, frozen weights). Every rank runs the same sequence
of forwards and backwards, so the pool evolves identically on all ranks and a new buffer -- a
collective ``torch.distributed._symmetric_memory`` allocation -- is made at the same call on every
rank. Several forwards may be outstanding at once (a frozen reference model, gradient
accumulation, recomputation); a forward whose backward never runs keeps its buffer until the next
step boundary (``reset_pools``, called when the gradients are zeroed). Flags carry a call sequence
number and are never reset; a call touches a peer's buffers of that call only after the peer
announced it entered the call, which also keeps the two-slot ring of transient buffers safe to
reuse.
"""

from __future__ import annotations

import os
from typing import Any

import torch
import torch.distributed as dist

from mint_b200.ops import _ext
from mint_b200.ops.gemm import matmul
from mint_b200.ops.linear import _cast_weight, weight_grads


class _Symm:
    """One symmetric buffer: the local tensor and every rank's address of it."""

    def __init__(self, nbytes: int, group: Any, device: torch.device) -> None:
        import torch.distributed._symmetric_memory as symm_mem  # noqa: PLC0415

        self.nbytes = nbytes
        self.buf = symm_mem.empty(nbytes, dtype=torch.uint8, device=device)
        self.buf.zero_()
        self.handle = symm_mem.rendezvous(self.buf, group)
        me = self.handle.buffer_ptrs[self.handle.rank]
        off = self.buf.data_ptr() - me
        self.ptrs = [int(p) + off for p in self.handle.buffer_ptrs]

    def view(self, shape: tuple[int, ...], dtype: torch.dtype, offset: int = 0) -> torch.Tensor:
        n = 1
        for d in shape:
            n *= d
        esz = torch.empty((), dtype=dtype).element_size()
        assert offset + n * esz <= self.nbytes
        return self.buf[offset : offset + n * esz].view(dtype).view(shape)


class TPComm:
    """Symmetric buffers, flags and call sequence numbers of one tensor-parallel group."""

    MAX_FLAG_BLOCKS = 1 << 16  # (rows / 128) x column tiles x 4 per source rank

    def __init__(self, group: Any, device: torch.device) -> None:
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = device
        self.seq = 0
        # control block: arrive[world] int32, then reduce-scatter flags [world][MAX_FLAG_BLOCKS] int32
        ctrl_bytes = 256 + self.world * self.MAX_FLAG_BLOCKS * 4
        self.ctrl = _Symm(ctrl_bytes, group, device)
        self.arrive = self.ctrl.view((self.world,), torch.int32)
        self.arrive_ptrs = list(self.ctrl.ptrs)
        self.rs_flags = self.ctrl.view((self.world * self.MAX_FLAG_BLOCKS,), torch.int32, offset=256)
        self.rowflag = torch.zeros(1 << 16, dtype=torch.int32, device=device)
        self.claim = torch.zeros(1, dtype=torch.int64, device=device)
        self._pool: list[_Symm] = []  # gathered-input buffers, in allocation order
        self._busy: set[int] = set()  # pool slots held by a forward whose backward has not run
        self._last_use: list[int] = []  # sequence number of the fused call that last let peers read a slot
        self._ring: list[_Symm | None] = [None, None]
        self._ring_idx = 0
        # all-reduce (no SP): output ring and the barrier's flags (bytes 128.. of the control block)
        self._ar: list[_Symm | None] = [None, None]
        self._ar_idx = 0
        self.bar_flags = self.ctrl.view((self.world,), torch.int32, offset=128)
        self.bar_ptrs = [p + 128 for p in self.ctrl.ptrs]

    # -------------------------------------------------------------- buffers
    def acquire(self, nbytes: int) -> tuple[int, _Symm]:
        """A free pooled buffer of at least ``nbytes`` (first fit), or a new one (collective).

        A peer can still be one fused call behind this rank (each kernel waits for every peer to
        enter the same call, so no rank is further ahead), and the caller writes its own shard
        into the buffer before its next kernel starts. A slot whose last peer-read call is the
        current one or the one before it is therefore skipped even when released."""
        for i, b in enumerate(self._pool):
            if i not in self._busy and b.nbytes >= nbytes and self._last_use[i] <= self.seq - 1:
                self._busy.add(i)
                return i, b
        b = _Symm(nbytes, self.group, self.device)  # every rank reaches this call alike
        self._pool.append(b)
        self._last_use.append(-(1 << 62))
        i = len(self._pool) - 1
        self._busy.add(i)
        return i, b

    def mark_read_by_peers(self, slot: int) -> None:
        """The fused call just issued (sequence ``self.seq``) lets peers read ``slot``."""
        self._last_use[slot] = self.seq

    def release(self, slot: int) -> None:
        self._busy.discard(slot)

    def reset_pool(self) -> None:
        """Step boundary: no backward is pending, so every pooled buffer is free again."""
        self._busy.clear()

    def in_use(self) -> int:
        return len(self._busy)

    def _ring_buffer(self, nbytes: int) -> _Symm:
        i = self._ring_idx
        self._ring_idx ^= 1
        b = self._ring[i]
        if b is None or b.nbytes < nbytes:
            b = _Symm(nbytes, self.group, self.device)
            self._ring[i] = b
        return b

    def next_seq(self) -> int:
        self.seq += 1
        return self.seq

    # -------------------------------------------------------------- fused GEMMs
    def gemm_ag(self, gathered: _Symm, rows: int, K: int, w: torch.Tensor, b_kmajor: bool, seg: int) -> torch.Tensor:
        """``C = gathered[rows, K] @ op(w)`` with the peers' row chunks pulled in by the kernel."""
        C = _ext.require()
        A = gathered.view((rows, K), torch.bfloat16)
        n = w.shape[0] if b_kmajor else w.shape[1]
        out = torch.empty(rows, n, dtype=torch.bfloat16, device=A.device)
        C.gemm_ag(A, w, out, b_kmajor, gathered.ptrs, self.arrive, self.arrive_ptrs, self.rowflag, self.claim,
                  self.rank, self.world, seg, self.next_seq())
        return out

    def gemm_rs(self, A: torch.Tensor, w: torch.Tensor, b_kmajor: bool, seg: int,
                out: torch.Tensor | None = None) -> torch.Tensor:
        """This rank's rows of ``sum over ranks (A @ op(w))`` (reduce-scatter fused into the GEMM)."""
        C = _ext.require()
        rows = A.shape[0]
        mc = rows // self.world
        n = w.shape[0] if b_kmajor else w.shape[1]
        tiles_n = (n + 255) // 256
        fslot = (mc // 128) * tiles_n * 4
        if fslot > self.MAX_FLAG_BLOCKS:
            raise ValueError(f"fused reduce-scatter of {rows} x {n} exceeds the flag block")
        recv = self._ring_buffer(self.world * mc * n * 2)
        recv_t = recv.view((self.world, mc, n), torch.bfloat16)
        slot_bytes = mc * n * 2
        push = [recv.ptrs[p] + self.rank * slot_bytes for p in range(self.world)]
        flag_ptrs = [self.ctrl.ptrs[p] + 256 + self.rank * self.MAX_FLAG_BLOCKS * 4 for p in range(self.world)]
        flags = self.rs_flags.view(self.world, self.MAX_FLAG_BLOCKS)
        if out is None:
            out = torch.empty(mc, n, dtype=torch.bfloat16, device=A.device)
        C.gemm_rs(A, w, out, b_kmajor, push, recv_t, flag_ptrs, flags, self.arrive, self.arrive_ptrs,
                  self.rank, self.world, seg, self.next_seq())
        return out

    def gemm_ar(self, A: torch.Tensor, w: torch.Tensor, b_kmajor: bool) -> torch.Tensor:
        """``sum over ranks (A @ op(w))`` on every rank (tensor parallelism without SP).

        The fused GEMM -> reduce-scatter kernel writes this rank's reduced rows (a contiguous
        ``rows / world`` block) straight into its part of a symmetric buffer; one push kernel stores
        that block into every peer's buffer at the same offset, and a stream barrier over NVLink flags
        publishes the pushes. The result is copied out of the (two-deep) ring of buffers."""
        C = _ext.require()
        rows = A.shape[0]
        n = w.shape[0] if b_kmajor else w.shape[1]
        seg = rows // self.world
        i = self._ar_idx
        self._ar_idx ^= 1
        full = self._ar[i]
        if full is None or full.nbytes < rows * n * 2:
            full = _Symm(rows * n * 2, self.group, self.device)
            self._ar[i] = full
        fullv = full.view((rows, n), torch.bfloat16)
        mine = fullv[self.rank * seg : (self.rank + 1) * seg]
        self.gemm_rs(A, w, b_kmajor, seg, out=mine)
        C.zero_all_gather(mine.view(torch.float32).view(-1), full.ptrs, self.rank, self.world)
        C.zero_barrier(self.bar_ptrs, self.bar_flags, self.rank, self.world, self.next_seq())
        return fullv.clone()


_COMMS: dict[Any, TPComm] = {}


def get_comm(group: Any, device: torch.device) -> TPComm:
    key = (id(group), device.index)
    comm = _COMMS.get(key)
    if comm is None:
        comm = TPComm(group, device)
        _COMMS[key] = comm
    return comm


# ------------------------------------------------------------------------------------------ autograd
def _place_shard(gathered: _Symm, x: torch.Tensor, rank: int, world: int) -> None:
    """Copy this rank's sequence shard ``x [B, seg, K]`` (bf16) into its rows of the gathered
    layout ``[B, world, seg, K]``: one strided 2-D copy (B rows of seg*K elements)."""
    B, seg, K = x.shape
    x = x if (x.dtype == torch.bfloat16 and x.is_contiguous()) else x.to(torch.bfloat16).contiguous()
    row = seg * K * 2
    _ext.require().copy_rows_2d(gathered.buf, rank * row, world * row, x, row, row, B)


def _bf16_2d(t: torch.Tensor) -> torch.Tensor:
    t2 = t.reshape(-1, t.shape[-1])
    if t2.dtype != torch.bfloat16 or not t2.is_contiguous():
        t2 = t2.to(torch.bfloat16).contiguous()
    return t2


class _ColumnParallelFn(torch.autograd.Function):
    """``y [B, T, N/tp] = all_gather_T(x [B, T/tp, K]) @ cat(weights)^T``."""

    @staticmethod
    def forward(ctx, x, comm, keep, *weights):  # noqa: ANN001, ANN205
        B, seg, K = x.shape
        world, rank = comm.world, comm.rank
        T = seg * world
        rows = B * T
        slot, gathered = comm.acquire(rows * K * 2)
        _place_shard(gathered, x, rank, world)  # this rank's shard in place; the kernel pulls the others
        w = _cast_weight(weights, torch.bfloat16)
        y = comm.gemm_ag(gathered, rows, K, w, True, seg)
        comm.mark_read_by_peers(slot)
        if not keep:
            comm.release(slot)  # no backward will read the gathered input
        ctx.comm, ctx.weights, ctx.shape, ctx.x_dtype, ctx.slot = comm, weights, (B, seg, K), x.dtype, slot
        ctx.save_for_backward(gathered.view((rows, K), torch.bfloat16))
        return y.view(B, T, -1)

    @staticmethod
    def backward(ctx, dy):  # noqa: ANN001, ANN205
        (G,) = ctx.saved_tensors
        comm, weights = ctx.comm, ctx.weights
        B, seg, K = ctx.shape
        dy2 = _bf16_2d(dy)
        dx = None
        if ctx.needs_input_grad[0]:
            w = _cast_weight(weights, torch.bfloat16)  # [N, K]: op(B) = w read MN-major
            dx = comm.gemm_rs(dy2, w, False, seg).view(B, seg, K).to(ctx.x_dtype)
        want = [ctx.needs_input_grad[3 + i] for i in range(len(weights))]
        grads = weight_grads(weights, want, dy2, G)
        comm.release(ctx.slot)  # stream order keeps the weight-gradient GEMM ahead of any reuse
        return (dx, None, None, *grads)


class _RowParallelFn(torch.autograd.Function):
    """``y [B, T/tp, N] = reduce_scatter_T(x [B, T, K/tp] @ w^T)``."""

    @staticmethod
    def forward(ctx, x, comm, w):  # noqa: ANN001, ANN205
        B, T, K = x.shape
        seg = T // comm.world
        x2 = _bf16_2d(x)
        wc = _cast_weight((w,), torch.bfloat16)
        y = comm.gemm_rs(x2, wc, True, seg)
        ctx.comm, ctx.w, ctx.shape, ctx.x_dtype = comm, w, (B, T, K), x.dtype
        ctx.save_for_backward(x2)
        return y.view(B, seg, -1)

    @staticmethod
    def backward(ctx, dy):  # noqa: ANN001, ANN205
        (x2,) = ctx.saved_tensors
        comm, w = ctx.comm, ctx.w
        B, T, K = ctx.shape
        world, rank = comm.world, comm.rank
        seg = T // world
        n = dy.shape[-1]
        rows = B * T
        gathered = comm._ring_buffer(rows * n * 2)
        _place_shard(gathered, dy, rank, world)
        dx = None
        wc = _cast_weight((w,), torch.bfloat16)  # [N, K/tp] = op(B) read MN-major
        dy_full = comm.gemm_ag(gathered, rows, n, wc, False, seg) if ctx.needs_input_grad[0] else None
        if dy_full is not None:
            dx = dy_full.view(B, T, K).to(ctx.x_dtype)
        grads = weight_grads((w,), [ctx.needs_input_grad[2]], gathered.view((rows, n), torch.bfloat16), x2)
        return (dx, None, *grads)


class _ColumnParallelARFn(torch.autograd.Function):
    """No SP: ``y = x @ cat(weights)^T`` on the replicated input (a local GEMM); the backward's
    ``dx = all_reduce(dy @ W)`` runs as the fused GEMM -> reduce-scatter + push all-gather."""

    @staticmethod
    def forward(ctx, x, comm, *weights):  # noqa: ANN001, ANN205
        x2 = _bf16_2d(x)
        w = _cast_weight(weights, torch.bfloat16)
        y = matmul(x2, w, trans_b=True, out_dtype=torch.bfloat16)
        ctx.comm, ctx.weights, ctx.x_shape, ctx.x_dtype = comm, weights, x.shape, x.dtype
        ctx.save_for_backward(x2)
        return y.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):  # noqa: ANN001, ANN205
        (x2,) = ctx.saved_tensors
        dy2 = _bf16_2d(dy)
        dx = None
        if ctx.needs_input_grad[0]:
            w = _cast_weight(ctx.weights, torch.bfloat16)
            dx = ctx.comm.gemm_ar(dy2, w, False).view(ctx.x_shape).to(ctx.x_dtype)
        want = [ctx.needs_input_grad[2 + i] for i in range(len(ctx.weights))]
        return (dx, None, *weight_grads(ctx.weights, want, dy2, x2))


class _RowParallelARFn(torch.autograd.Function):
    """No SP: ``y = all_reduce(x @ w^T)`` as one fused GEMM -> reduce-scatter plus a push
    all-gather; the backward needs no collective (``dx = dy @ w`` on the replicated ``dy``)."""

    @staticmethod
    def forward(ctx, x, comm, w):  # noqa: ANN001, ANN205
        x2 = _bf16_2d(x)
        wc = _cast_weight((w,), torch.bfloat16)
        y = comm.gemm_ar(x2, wc, True)
        ctx.w, ctx.x_shape, ctx.x_dtype = w, x.shape, x.dtype
        ctx.save_for_backward(x2)
        return y.view(*x.shape[:-1], -1)

    @staticmethod
    def backward(ctx, dy):  # noqa: ANN001, ANN205
        (x2,) = ctx.saved_tensors
        dy2 = _bf16_2d(dy)
        dx = None
        if ctx.needs_input_grad[0]:
            wc = _cast_weight((ctx.w,), torch.bfloat16)
            dx = matmul(dy2, wc, out_dtype=torch.bfloat16).view(ctx.x_shape).to(ctx.x_dtype)
        return (dx, None, *weight_grads((ctx.w,), [ctx.needs_input_grad[2]], dy2, x2))


def enabled(tp: Any, x: torch.Tensor) -> bool:
    """Fused collectives apply to CUDA TP groups of 2..8 ranks whose row chunks are whole 256-row
    tiles: with SP the per-rank sequence shard, without SP the rows / tp block of the all-reduce."""
    if os.environ.get("MINT_FUSED_TP", "1") == "0" or tp is None or tp.size < 2 or tp.size > 8 or not x.is_cuda:
        return False
    if not _ext.kernels_enabled() or not hasattr(_ext.require(), "gemm_ag") or x.dim() != 3:
        return False
    if tp.sp:
        return x.shape[1] % 256 == 0
    return (x.shape[0] * x.shape[1]) % (256 * tp.size) == 0


def column_parallel_linear(x: torch.Tensor, weights: tuple[torch.Tensor, ...], tp: Any) -> torch.Tensor:
    """SP: sequence-parallel input ``[B, T/tp, K]`` -> ``[B, T, sum N_i / tp]`` (all-gather fused
    into the GEMM). No SP: replicated ``[B, T, K]`` -> ``[B, T, sum N_i / tp]`` (backward all-reduce
    fused)."""
    comm = get_comm(tp.group, x.device)
    if not tp.sp:
        return _ColumnParallelARFn.apply(x, comm, *weights)
    keep = torch.is_grad_enabled() and (x.requires_grad or any(w.requires_grad for w in weights))
    return _ColumnParallelFn.apply(x, comm, keep, *weights)


def row_parallel_linear(x: torch.Tensor, w: torch.Tensor, tp: Any) -> torch.Tensor:
    """``[B, T, K/tp]`` -> SP: sequence-parallel ``[B, T/tp, N]`` (reduce-scatter fused); no SP:
    replicated ``[B, T, N]`` (all-reduce fused)."""
    comm = get_comm(tp.group, x.device)
    if not tp.sp:
        return _RowParallelARFn.apply(x, comm, w)
    return _RowParallelFn.apply(x, comm, w)


def begin_forward(tp: Any, device: torch.device) -> None:  # noqa: ARG001
    """Kept for callers of the earlier API: buffers are now pooled per forward/backward pair."""


def reset_pools() -> None:
    """Step boundary (gradients zeroed): free every pooled gathered-input buffer. A forward whose
    backward never ran (an extra forward with gradients enabled) holds its buffer until here."""
    for comm in _COMMS.values():
        comm.reset_pool()
