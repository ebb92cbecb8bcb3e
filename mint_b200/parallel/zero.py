"""Bucketed data-parallel gradient engine: DDP and ZeRO-1/2/3 (reference: mint/utils/parallel.py:92-522).

The reference keeps one ``_ZeROParam`` per tensor and issues one synchronous NCCL call per
parameter from its grad hook. Here parameters are packed into flat fp32 **buckets** (one per
(module group, kind) — e.g. the matrices of block 7 — capped in size) so that:

* every rank's gradient communication is a handful of large async collectives issued as soon as
  a bucket's last gradient lands, overlapping the rest of backward;
* grads are views into the bucket buffer (no per-step allocation; one fused optimizer launch
  sweeps a whole shard);
* ``ddp_level`` 0/1 all-reduce the bucket, 2/3 reduce-scatter it; 1/2 all-gather updated
  parameter shards after the step; 3 keeps only the shard resident and all-gathers each block's
  buckets right before the block runs (forward and backward, with one-block-ahead prefetch).

Bucket kinds: ``flat`` (element-granular shards, AdamW-style elementwise updates) and ``owner``
(2-D block matrices assigned whole to one rank each, padded per rank) so NorMuon can
orthogonalize complete matrices on their owner rank.
"""

from __future__ import annotations

import math
from collections import defaultdict
from dataclasses import dataclass, field
from typing import Any

import torch
import torch.distributed as dist
from torch import nn

from mint_b200.parallel.context import ParallelContext

_ALIGN = 64  # elements: keeps every shard / param offset 256-byte aligned for fp32


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


def param_kind(name: str, p: torch.Tensor) -> str:
    """Optimizer grouping of the reference's configure_optimizer (mint/models/gemma.py:195-206)."""
    if "tok_embeddings" in name:
        return "embedding"
    if "output" in name:
        return "lm_head"
    if p.ndim == 2:
        return "matrix"
    return "scalar"


def _module_group(name: str) -> str:
    parts = name.split(".")
    if len(parts) >= 2 and parts[0] == "blocks" and parts[1].isdigit():
        return f"blocks.{parts[1]}"
    return "top"


@dataclass
class Slot:
    param: nn.Parameter
    name: str
    start: int  # offset in the bucket's padded flat space
    numel: int
    shape: torch.Size
    owner: int  # owning dp rank for owner buckets, -1 for flat buckets


@dataclass
class Bucket:
    index: int
    group: str
    kind: str  # "flat" | "owner"
    pkind: str  # optimizer param kind (matrix / scalar / embedding / lm_head)
    dtype: torch.dtype
    slots: list[Slot]
    size: int
    shard: int
    data: torch.Tensor | None = None  # full params [size] (levels 0-2; transient at level 3)
    shard_data: torch.Tensor | None = None  # this rank's param shard [shard]
    grad: torch.Tensor | None = None  # full grads [size] (persistent 0-2, transient 3)
    grad_shard: torch.Tensor | None = None  # reduced grad shard [shard] (levels 2/3)
    ready: int = 0
    handle: Any = None
    gather_handle: Any = None
    gathered: bool = True
    pending_scale: bool = False
    extra: dict = field(default_factory=dict)


class _BackwardGather(torch.autograd.Function):
    """Identity whose backward re-gathers a ZeRO-3 module group before that group's backward."""

    @staticmethod
    def forward(ctx, x, engine, group):  # noqa: ANN001, ANN205
        ctx.engine, ctx.group = engine, group
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        ctx.engine._pre_backward(ctx.group)
        return g, None, None


def _ext_mod():  # noqa: ANN202
    from mint_b200.ops import _ext  # noqa: PLC0415

    return _ext.require()


class GradEngine:
    def __init__(self, model: nn.Module, parallel: ParallelContext, bucket_cap_mb: float = 256.0) -> None:
        self.model = model
        self.parallel = parallel
        self.level = parallel.ddp_level
        self.dp = parallel.dp_size
        self.rank = parallel.dp_rank
        self.group = parallel.dp_group
        self.tp_group = parallel.tp_group
        self.distributed = self.dp > 1 and dist.is_available() and dist.is_initialized()
        self.sync_grads = True
        self.epoch = 0  # bumped whenever parameter values change (optimizer step, load)
        # gradient clipping: with defer_clip the coefficient stays on the device (grad_scale) and the
        # optimizer's update kernels multiply it in, instead of a separate pass scaling every gradient
        self.defer_clip = False
        self.grad_scale: torch.Tensor | None = None
        self._norm_tables: dict[tuple, tuple[torch.Tensor, torch.Tensor, int]] = {}
        self._in_backward: set[str] = set()
        self._pushed_buckets: set[int] = set()  # buckets / params whose update kernel already pushed them
        self._pushed_params: set[int] = set()
        self.fused_update_pushes = 0  # update kernels that stored their results into the peers' copies
        # ZeRO-2 on CUDA: gradient reduce-scatter and parameter all-gather as NVLink peer-memory kernels
        # (csrc/zero_comm.cu) over symmetric bucket buffers instead of NCCL; MINT_FUSED_ZERO=0 disables
        self.fused = self._fused_possible(model)
        # ZeRO-3 on CUDA: parameter shards in symmetric memory, gathered by a kernel that pulls every
        # peer's shard over NVLink (on a side stream, one group ahead) instead of NCCL all-gathers
        self.fused3 = self._fused3_possible(model)
        self._z3_dirty = True  # shards changed since the last barrier: the next gather starts with one
        self._zc = None
        self.buckets: list[Bucket] = []
        self.by_param: dict[int, tuple[Bucket, Slot]] = {}
        self.groups: dict[str, list[Bucket]] = defaultdict(list)
        self.group_order: list[str] = []
        self._build(bucket_cap_mb)
        self._install_hooks()

    # ------------------------------------------------------------------ layout
    def _build(self, cap_mb: float) -> None:
        seen: set[int] = set()
        entries: dict[tuple[str, str, str, torch.dtype], list[tuple[str, nn.Parameter]]] = defaultdict(list)
        order: list[tuple[str, str, str, torch.dtype]] = []
        for name, p in self.model.named_parameters():
            if id(p) in seen or not p.requires_grad:
                continue
            seen.add(id(p))
            pk = param_kind(name, p)
            kind = "owner" if (pk == "matrix" and self.dp > 1) else "flat"
            key = (_module_group(name), kind, pk, p.dtype)
            if key not in entries:
                order.append(key)
            entries[key].append((name, p))
        cap = max(1, int(cap_mb * 1024 * 1024 / 4))
        for key in order:
            grp, kind, pk, dtype = key
            chunk: list[tuple[str, nn.Parameter]] = []
            acc = 0
            for name, p in entries[key]:
                if chunk and acc + p.numel() > cap:
                    self._add_bucket(grp, kind, pk, dtype, chunk)
                    chunk, acc = [], 0
                chunk.append((name, p))
                acc += p.numel()
            if chunk:
                self._add_bucket(grp, kind, pk, dtype, chunk)
        for b in self.buckets:
            if b.group not in self.groups:
                self.group_order.append(b.group)
            self.groups[b.group].append(b)

    def _add_bucket(self, grp: str, kind: str, pk: str, dtype: torch.dtype, items: list[tuple[str, nn.Parameter]]) -> None:
        dp = self.dp
        slots: list[Slot] = []
        if kind == "owner":
            # greedy largest-first assignment of whole matrices to ranks
            loads = [0] * dp
            assign: list[list[tuple[str, nn.Parameter]]] = [[] for _ in range(dp)]
            for name, p in sorted(items, key=lambda it: -it[1].numel()):
                r = min(range(dp), key=lambda i: loads[i])
                assign[r].append((name, p))
                loads[r] += _round_up(p.numel(), _ALIGN)
            shard = _round_up(max(max(loads), 1), _ALIGN)
            for r in range(dp):
                off = r * shard
                for name, p in assign[r]:
                    slots.append(Slot(p, name, off, p.numel(), p.shape, r))
                    off += _round_up(p.numel(), _ALIGN)
            size = shard * dp
        else:
            off = 0
            for name, p in items:
                slots.append(Slot(p, name, off, p.numel(), p.shape, -1))
                off += _round_up(p.numel(), _ALIGN)
            size = _round_up(max(off, 1), _ALIGN * dp)
            shard = size // dp
        b = Bucket(len(self.buckets), grp, kind, pk, dtype, slots, size, shard)
        dev = items[0][1].device
        if self.fused and dtype == torch.float32 and shard % 4 == 0:
            b.extra["symm_data"] = self._symm(size * 4, dev)
            b.extra["symm_grad"] = self._symm(size * 4, dev)
            data = b.extra["symm_data"].view((size,), torch.float32)
        else:
            data = torch.zeros(size, dtype=dtype, device=dev)
        for s in slots:
            data[s.start : s.start + s.numel].copy_(s.param.detach().reshape(-1))
            self.by_param[id(s.param)] = (b, s)
            s.param._orig_shape = s.shape  # logical shape while ZeRO-3 keeps only a shard
        lo = self.rank * shard
        if self.level == 3 and self.dp > 1:
            if self.fused3 and dtype == torch.float32 and shard % 4 == 0:
                b.extra["symm_shard"] = self._symm(shard * 4, dev)
                b.shard_data = b.extra["symm_shard"].view((shard,), torch.float32)
                b.shard_data.copy_(data[lo : lo + shard])
            else:
                b.shard_data = data[lo : lo + shard].clone()
            b.data = None
            b.gathered = False
            for s in slots:
                s.param.data = torch.empty(0, dtype=dtype, device=dev)
        else:
            b.data = data
            b.shard_data = data[lo : lo + shard]
            for s in slots:
                s.param.data = data[s.start : s.start + s.numel].view(s.shape)
            b.grad = (b.extra["symm_grad"].view((size,), torch.float32) if "symm_grad" in b.extra
                      else torch.zeros(size, dtype=dtype, device=dev))
        if self.level >= 2 and self.dp > 1:
            b.grad_shard = torch.zeros(shard, dtype=dtype, device=dev)
        self.buckets.append(b)
        for s in slots:
            s.param._grad_engine = self  # lets the optimizer find the engine

    # ------------------------------------------------------------------ fused ZeRO-2 transport
    def _fused_possible(self, model: nn.Module) -> bool:
        import os  # noqa: PLC0415

        if os.environ.get("MINT_FUSED_ZERO", "1") == "0" or self.level != 2 or not self.distributed:
            return False
        if self.dp > 8 or not torch.cuda.is_available():
            return False
        dev = next((p.device for p in model.parameters()), torch.device("cpu"))
        if dev.type != "cuda":
            return False
        from mint_b200.ops import _ext  # noqa: PLC0415

        return _ext.kernels_enabled() and hasattr(_ext.require(), "zero_reduce_scatter")

    def _fused3_possible(self, model: nn.Module) -> bool:
        import os  # noqa: PLC0415

        if os.environ.get("MINT_FUSED_ZERO", "1") == "0" or self.level != 3 or not self.distributed:
            return False
        if self.dp > 8 or not torch.cuda.is_available():
            return False
        dev = next((p.device for p in model.parameters()), torch.device("cpu"))
        if dev.type != "cuda":
            return False
        from mint_b200.ops import _ext  # noqa: PLC0415

        return _ext.kernels_enabled() and hasattr(_ext.require(), "zero_gather_pull")

    def _zero3_barrier(self) -> None:
        """Stream-ordered barrier of the dp group (ZeRO-3 over peer memory): every rank's shard
        changes queued before it are complete before any peer's later gather reads them."""
        zc = self._zc
        _ext_mod().zero_barrier(zc["ctrl"].ptrs, zc["flags"], self.rank, self.dp, self._next_seq())
        self._z3_dirty = False

    def _symm(self, nbytes: int, dev: torch.device):  # noqa: ANN202
        from mint_b200.parallel.fused import _Symm  # noqa: PLC0415

        if self._zc is None:
            # control: flags [dp] int32 (one slot per peer), one sequence counter for both collectives
            ctrl = _Symm(256, self.group, dev)
            self._zc = {"ctrl": ctrl, "flags": ctrl.view((self.dp,), torch.int32), "seq": 0,
                        "stream": torch.cuda.Stream(device=dev)}
        return _Symm(nbytes, self.group, dev)

    def _next_seq(self) -> int:
        self._zc["seq"] += 1
        return self._zc["seq"]

    def _fused_reduce_scatter(self, b: Bucket) -> torch.Tensor:
        """This rank's shard of sum over ranks of the bucket's gradient, / dp, on the comm stream,
        written straight into ``grad_shard`` (zero before: at ZeRO-2 the reduce-scatter runs once per
        optimizer step, on the last micro-batch)."""
        zc = self._zc
        out = b.grad_shard
        stream = zc["stream"]
        stream.wait_stream(torch.cuda.current_stream())  # every gradient of the bucket has landed
        with torch.cuda.stream(stream):
            _ext_mod().zero_reduce_scatter(b.extra["symm_grad"].ptrs, out, 1.0 / self.dp, None,
                                               zc["ctrl"].ptrs, zc["flags"], self.rank, self.dp, self._next_seq())
        out.record_stream(stream)
        return out

    def _fused_all_gather(self, b: Bucket) -> None:
        _ext_mod().zero_all_gather(b.shard_data, b.extra["symm_data"].ptrs, self.rank, self.dp)

    def push_fusable(self, b: Bucket) -> bool:
        """True when an update kernel may store bucket ``b``'s new values straight into the peers'
        copies (ZeRO-2 over symmetric peer memory), so ``after_step`` needs no push for it."""
        return self.level == 2 and self.distributed and "symm_data" in b.extra

    def peer_pointers(self, b: Bucket, view: torch.Tensor) -> list[int]:
        """Every rank's address of ``view`` (a piece of bucket ``b``'s parameters on this rank)."""
        off = view.data_ptr() - b.data.data_ptr()
        return [int(base) + off for base in b.extra["symm_data"].ptrs]

    def mark_pushed(self, b: Bucket | None = None, params: list[torch.Tensor] = ()) -> None:
        """An update kernel already pushed bucket ``b`` (this rank's whole shard) or ``params``."""
        if b is not None:
            self._pushed_buckets.add(b.index)
        self._pushed_params.update(id(p) for p in params)
        self.fused_update_pushes += 1

    def _needs_push(self, b: Bucket) -> bool:
        if b.index in self._pushed_buckets:
            return False
        if b.kind == "owner":
            owned = [s for s in b.slots if s.owner == self.rank]
            return not owned or not all(id(s.param) in self._pushed_params for s in owned)
        return True

    # ------------------------------------------------------------------ grads
    def _install_grad_views(self, b: Bucket) -> None:
        if b.grad is None:
            return
        for s in b.slots:
            s.param.grad = b.grad[s.start : s.start + s.numel].view(s.shape)

    def zero_grad(self) -> None:
        from mint_b200.parallel import fused  # noqa: PLC0415

        fused.reset_pools()  # a step boundary: no tensor-parallel backward is pending
        self.grad_scale = None
        for b in self.buckets:
            if b.grad is not None:
                b.grad.zero_()
                self._install_grad_views(b)
            if b.grad_shard is not None:
                b.grad_shard.zero_()
            b.ready = 0
            b.handle = None
            b.pending_scale = False

    def _install_hooks(self) -> None:
        for b in self.buckets:
            hook = self._make_hook(b)
            for s in b.slots:
                s.param.register_post_accumulate_grad_hook(hook)
                # kernels that accumulate a weight gradient directly into the bucket call this
                s.param._mint_grad_ready = (lambda h=hook, prm=s.param: h(prm))
        self.zero_grad()
        if self.level == 3 and self.dp > 1:
            self._install_zero3_hooks()

    def _make_hook(self, b: Bucket):  # noqa: ANN202
        def hook(_p: torch.Tensor) -> None:
            b.ready += 1
            if b.ready == len(b.slots):
                self._launch(b)
        return hook

    def _launch(self, b: Bucket) -> None:
        b.ready = 0
        if b.grad is None:
            return
        if not self.distributed:
            if self.level == 3 and self.dp > 1:
                pass
            return
        if self.level in (0, 1):
            if not self.sync_grads:
                return
            b.handle = dist.all_reduce(b.grad, op=dist.ReduceOp.SUM, group=self.group, async_op=True)
        else:
            if not self.sync_grads and self.level == 2:
                return
            if "symm_grad" in b.extra:
                b.handle = ("fused", self._fused_reduce_scatter(b))
                b.pending_scale = False
                return
            out = torch.empty_like(b.grad_shard)
            h = dist.reduce_scatter_tensor(out, b.grad, op=dist.ReduceOp.SUM, group=self.group, async_op=True)
            b.handle = (h, out)
        b.pending_scale = True
        if self.level == 3:
            self._finish_bucket(b)  # level 3 must release the full grad buffer promptly

    def _finish_bucket(self, b: Bucket) -> None:
        if b.handle is None:
            return
        if isinstance(b.handle, tuple) and b.handle[0] == "fused":
            zc = self._zc
            torch.cuda.current_stream().wait_stream(zc["stream"])  # the kernel wrote grad_shard, scaled
        elif isinstance(b.handle, tuple):
            h, out = b.handle
            h.wait()
            b.grad_shard.add_(out)
        else:
            b.handle.wait()
        b.handle = None
        if self.level == 3:
            self._release_grads(b)

    def finish_grad_sync(self) -> None:
        """Wait for all bucket collectives (launching any bucket a hook never completed) and scale by 1/dp."""
        if not self.distributed:
            return
        for b in self.buckets:
            if b.handle is None and b.grad is not None and (self.sync_grads or self.level == 3):
                if b.ready or self.level != 3:
                    self._launch(b)
            self._finish_bucket(b)
        inv = 1.0 / self.dp
        for b in self.buckets:
            if self.level in (0, 1):
                if b.grad is not None:
                    b.grad.mul_(inv)
            elif b.grad_shard is not None and "symm_grad" not in b.extra:
                b.grad_shard.mul_(inv)
            b.pending_scale = False

    def sync_tp_partial_grads(self) -> None:
        """Sum grads of TP-replicated params whose contributions are partial (QK-norm, SP norms).

        Runs after the dp collectives on this rank's *reduced* gradient pieces (full grads at
        ddp_level 0/1, reduce-scattered shards at 2/3); every rank of a TP group has the same bucket
        layout for replicated parameters, so the pieces line up across the group.
        """
        tp_group = self.tp_group
        if tp_group is None or dist.get_world_size(tp_group) == 1:
            return
        pieces = []
        for b in self.buckets:
            for s in b.slots:
                if getattr(s.param, "_tp_partial_grad", False):
                    pieces.extend(gv for _pv, gv, _o, _n in self.segments(s.param))
        if not pieces:
            return
        flat = torch.cat([g.reshape(-1) for g in pieces])
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=tp_group)
        off = 0
        for g in pieces:
            g.copy_(flat[off : off + g.numel()].view_as(g))
            off += g.numel()

    # ------------------------------------------------------------------ optimizer views
    def segments(self, p: torch.Tensor) -> list[tuple[torch.Tensor, torch.Tensor, int, int]]:
        """This rank's ``(param_view, grad_view, elem_offset_in_param, numel)`` pieces of ``p``."""
        b, s = self.by_param[id(p)]
        if self.level == 0 or self.dp == 1:
            return [(b.data[s.start : s.start + s.numel], b.grad[s.start : s.start + s.numel], 0, s.numel)]
        lo, hi = self.rank * b.shard, (self.rank + 1) * b.shard
        a, e = max(lo, s.start), min(hi, s.start + s.numel)
        if a >= e:
            return []
        pv = b.shard_data[a - lo : e - lo]
        if self.level == 1:
            gv = b.grad[a:e]
        else:
            gv = b.grad_shard[a - lo : e - lo]
        return [(pv, gv, a - s.start, e - a)]

    def owns_whole(self, p: torch.Tensor) -> bool:
        b, s = self.by_param[id(p)]
        if self.level == 0 or self.dp == 1:
            return True
        return s.owner == self.rank

    def slot(self, p: torch.Tensor) -> tuple[Bucket, Slot]:
        return self.by_param[id(p)]

    def after_step(self) -> None:
        """Propagate updated shards: all-gather params (levels 1/2); level 3 drops stale full copies."""
        self.epoch += 1
        if not self.distributed or self.level == 0:
            return
        if self.level == 3:
            for grp in self.group_order:
                self.free_group(grp)
            for b in self.buckets:  # a gather prefetched but never bound holds the old values
                if b.gather_handle is not None and not isinstance(b.gather_handle, tuple):
                    b.gather_handle.wait()
                b.gather_handle = None
                b.extra.pop("full", None)
            self._in_backward.clear()
            if self.fused3:
                # the updated shards are published before any peer's next gather reads them; the
                # update itself started only after every peer's gathers of this step had completed
                # (they precede each rank's last gradient reduce-scatter, which the update waits for)
                self._zero3_barrier()
            return
        handles = []
        pushed = False
        for b in self.buckets:
            if "symm_data" in b.extra:
                if self._needs_push(b):
                    self._fused_all_gather(b)
                pushed = True
                continue
            src = b.shard_data.clone()
            handles.append(dist.all_gather_into_tensor(b.data, src, group=self.group, async_op=True))
        for h in handles:
            h.wait()
        if pushed:
            # one barrier for every bucket's push: peers' shards have landed here, and no peer still
            # reads this rank's gradient buckets, so the next zero_grad and forward may proceed
            zc = self._zc
            _ext_mod().zero_barrier(zc["ctrl"].ptrs, zc["flags"], self.rank, self.dp, self._next_seq())
        self._pushed_buckets.clear()
        self._pushed_params.clear()

    # ------------------------------------------------------------------ grad norm
    def _reduced_grad(self, b: Bucket) -> torch.Tensor | None:
        """This rank's reduced gradient piece of bucket ``b`` (full, slice or reduce-scattered shard)."""
        if self.level == 0 or self.dp == 1 or not self.distributed:
            return b.grad
        if self.level == 1:
            lo = self.rank * b.shard
            return b.grad[lo : lo + b.shard]
        return b.grad_shard

    def grad_norm_sq(self) -> torch.Tensor:
        """Squared global grad norm over dp x tp, each element counted once (fused per-bucket norms)."""
        tp = self.parallel.tp_size
        pieces = []
        for b in self.buckets:
            g = self._reduced_grad(b)
            if g is None:
                continue
            sharded = [getattr(sl.param, "_tp_sharded", False) for sl in b.slots]
            if tp > 1 and not all(sharded):
                if any(sharded):  # mixed bucket: fall back to per-parameter pieces
                    for sl in b.slots:
                        if getattr(sl.param, "_tp_sharded", False) or self.parallel.tp_rank == 0:
                            pieces.extend(gv for _pv, gv, _o, _n in self.segments(sl.param))
                    continue
                if self.parallel.tp_rank != 0:
                    continue
            pieces.append(g)
        dev = self.buckets[0].shard_data.device if self.buckets else torch.device("cpu")
        if pieces and self._kernel_norm_ok(pieces):
            total = self._sumsq_kernel(pieces)
        elif pieces:
            norms = torch._foreach_norm([t.float() if t.dtype != torch.float32 else t for t in pieces])
            total = torch.stack(norms).square().sum()
        else:
            total = torch.zeros((), dtype=torch.float32, device=dev)
        if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
            if self.level == 0 or self.dp == 1:
                # dp replicas hold identical full gradients: reduce over the TP group only
                if tp > 1:
                    dist.all_reduce(total, op=dist.ReduceOp.SUM, group=self.tp_group)
            else:
                dist.all_reduce(total, op=dist.ReduceOp.SUM)
        return total

    @staticmethod
    def _kernel_norm_ok(pieces: list[torch.Tensor]) -> bool:
        from mint_b200.ops import _ext  # noqa: PLC0415

        return (pieces[0].is_cuda and _ext.kernels_enabled()
                and all(t.dtype == torch.float32 and t.is_contiguous() for t in pieces))

    def _sumsq_kernel(self, pieces: list[torch.Tensor]) -> torch.Tensor:
        """Sum of squares of every piece in one launch (pointer table cached per layout)."""
        key = tuple((t.data_ptr(), t.numel()) for t in pieces)
        hit = self._norm_tables.get(key)
        dev = pieces[0].device
        if hit is None:
            from mint_b200.ops import _ext  # noqa: PLC0415

            rows = _ext.piece_table(list(key), (4,))
            ptrs = torch.tensor([r[0] for r in rows], dtype=torch.int64, device=dev)
            sizes = torch.tensor([r[1] for r in rows], dtype=torch.int64, device=dev)
            hit = (ptrs, sizes, _ext.PIECE_ELEMS)
            self._norm_tables[key] = hit
        out = torch.zeros(1, dtype=torch.float32, device=dev)
        _ext_mod().sumsq_multi(hit[0], hit[1], out, hit[2])
        return out.view(())

    def clip_on_device(self) -> bool:
        """True when the clip coefficient can stay on the device for the update kernels."""
        from mint_b200.ops import _ext  # noqa: PLC0415

        dev = self.buckets[0].shard_data.device if self.buckets else torch.device("cpu")
        return dev.type == "cuda" and _ext.kernels_enabled() and _ext.available()

    def clip_grad_norm(self, max_norm: float) -> torch.Tensor:
        total = self.grad_norm_sq()
        if self.defer_clip and total.is_cuda:
            coef = torch.empty(1, dtype=torch.float32, device=total.device)
            norm = torch.empty(1, dtype=torch.float32, device=total.device)
            _ext_mod().clip_coef(total.reshape(1).contiguous(), float(max_norm), coef, norm)
            self.grad_scale = coef
            return norm.view(())
        norm = total.sqrt()
        coef = (max_norm / (norm + 1e-6)).clamp(max=1.0)
        grads = [g for g in (self._reduced_grad(b) for b in self.buckets) if g is not None]
        if grads:
            torch._foreach_mul_(grads, coef)
        return norm

    # ------------------------------------------------------------------ ZeRO-3 gather / free
    def _gather_bucket(self, b: Bucket, async_op: bool = False) -> None:
        if b.gathered or b.gather_handle is not None:
            return
        full = torch.empty(b.size, dtype=b.dtype, device=b.shard_data.device)
        if "symm_shard" in b.extra:
            # pull every peer's shard over NVLink on the side stream; _bind_full joins it
            if self._z3_dirty:
                self._zero3_barrier()
            stream = self._zc["stream"]
            stream.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(stream):
                _ext_mod().zero_gather_pull(b.extra["symm_shard"].ptrs, full, self.rank, self.dp)
            full.record_stream(stream)
            ev = torch.cuda.Event()
            ev.record(stream)
            b.extra["full"] = full
            b.gather_handle = ("pull", ev)
            if not async_op:
                self._bind_full(b)
            return
        h = dist.all_gather_into_tensor(full, b.shard_data, group=self.group, async_op=async_op)
        b.extra["full"] = full
        if async_op:
            b.gather_handle = h
        else:
            self._bind_full(b)

    def _bind_full(self, b: Bucket) -> None:
        if isinstance(b.gather_handle, tuple):
            torch.cuda.current_stream().wait_event(b.gather_handle[1])
            b.gather_handle = None
        elif b.gather_handle is not None:
            b.gather_handle.wait()
            b.gather_handle = None
        full = b.extra.pop("full", None)
        if full is None:
            return
        b.data = full
        for s in b.slots:
            s.param.data = full[s.start : s.start + s.numel].view(s.shape)
        b.gathered = True

    def _free_bucket(self, b: Bucket) -> None:
        if not b.gathered:
            return
        for s in b.slots:
            s.param.data = torch.empty(0, dtype=b.dtype, device=b.shard_data.device)
        b.data = None
        b.gathered = False

    def gather_group(self, grp: str, async_op: bool = False) -> None:
        for b in self.groups.get(grp, []):
            self._gather_bucket(b, async_op=async_op)

    def wait_group(self, grp: str) -> None:
        for b in self.groups.get(grp, []):
            if not b.gathered:
                if b.gather_handle is None and "full" not in b.extra:
                    self._gather_bucket(b)
                self._bind_full(b)

    def free_group(self, grp: str) -> None:
        for b in self.groups.get(grp, []):
            self._free_bucket(b)

    def _alloc_grads(self, grp: str) -> None:
        for b in self.groups.get(grp, []):
            if b.grad is None:
                b.grad = torch.zeros(b.size, dtype=b.dtype, device=b.shard_data.device)
                self._install_grad_views(b)

    def _release_grads(self, b: Bucket) -> None:
        for s in b.slots:
            s.param.grad = None
        b.grad = None
        if b.group != "top" and all(x.grad is None for x in self.groups[b.group]):
            self._in_backward.discard(b.group)
            for x in self.groups[b.group]:
                self._free_bucket(x)

    def _pre_backward(self, grp: str) -> None:
        self._in_backward.add(grp)
        self.wait_group(grp)
        self._alloc_grads(grp)
        i = self.group_order.index(grp)
        if i - 1 >= 0 and self.group_order[i - 1] != "top":
            self.gather_group(self.group_order[i - 1], async_op=True)

    def _install_zero3_hooks(self) -> None:
        model = self.model
        blocks = getattr(model, "blocks", None)
        order = [g for g in self.group_order if g != "top"]

        def model_pre(_m, _args):  # noqa: ANN001, ANN202
            self.wait_group("top")
            if torch.is_grad_enabled():
                self._alloc_grads("top")
            if order:
                self.gather_group(order[0], async_op=True)

        if hasattr(model, "_before_forward"):
            # models with entry points other than forward() (Gemma.loss) call this themselves
            model._before_forward = lambda: model_pre(model, ())
        else:
            model.register_forward_pre_hook(model_pre)
        if blocks is None:
            return
        for i, blk in enumerate(blocks):
            grp = f"blocks.{i}"
            if grp not in self.groups:
                continue
            nxt = f"blocks.{i + 1}" if f"blocks.{i + 1}" in self.groups else None

            def pre(_m, _args, grp=grp, nxt=nxt):  # noqa: ANN001, ANN202
                self.wait_group(grp)
                if nxt is not None:
                    self.gather_group(nxt, async_op=True)

            def post(_m, _args, out, grp=grp):  # noqa: ANN001, ANN202
                if grp not in self._in_backward:  # a recompute inside backward keeps the params
                    self.free_group(grp)
                if not torch.is_grad_enabled():
                    return out
                if isinstance(out, torch.Tensor):
                    return _BackwardGather.apply(out, self, grp) if out.requires_grad else out
                if isinstance(out, tuple):  # every output re-gathers before the block's backward
                    return tuple(_BackwardGather.apply(o, self, grp) if isinstance(o, torch.Tensor) and o.requires_grad
                                 else o for o in out)
                return out

            blk.register_forward_pre_hook(pre)
            blk.register_forward_hook(post)

    # ------------------------------------------------------------------ state
    def full_param(self, p: torch.Tensor) -> torch.Tensor:
        """The full (dp-consolidated) value of ``p`` (collective at ZeRO-3)."""
        b, s = self.by_param[id(p)]
        if b.gathered and b.data is not None:
            return b.data[s.start : s.start + s.numel].view(s.shape)
        full = torch.empty(b.size, dtype=b.dtype, device=b.shard_data.device)
        dist.all_gather_into_tensor(full, b.shard_data, group=self.group)
        return full[s.start : s.start + s.numel].view(s.shape)

    def load_full_param(self, p: torch.Tensor, value: torch.Tensor) -> None:
        self.epoch += 1
        self._z3_dirty = True
        b, s = self.by_param[id(p)]
        flat = value.reshape(-1).to(b.dtype)
        lo = self.rank * b.shard
        a, e = max(lo, s.start), min(lo + b.shard, s.start + s.numel)
        if a < e:
            b.shard_data[a - lo : e - lo].copy_(flat[a - s.start : e - s.start])
        if b.data is not None:
            b.data[s.start : s.start + s.numel].copy_(flat)


def get_engine(model: nn.Module) -> GradEngine | None:
    return getattr(model, "_grad_engine", None)


def apply_ddp(model: nn.Module, parallel: ParallelContext, bucket_cap_mb: float = 256.0) -> nn.Module:
    engine = GradEngine(model, parallel, bucket_cap_mb=bucket_cap_mb)
    model._grad_engine = engine
    return model


def bucket_summary(engine: GradEngine) -> str:
    lines = []
    for b in engine.buckets:
        lines.append(f"bucket {b.index}: {b.group}/{b.kind}/{b.pkind} params={len(b.slots)} size={b.size} "
                     f"shard={b.shard} ({b.size * 4 / 2**20:.1f} MiB)")
    return "\n".join(lines)


__all__ = ["GradEngine", "apply_ddp", "bucket_summary", "get_engine", "param_kind", "math"]
