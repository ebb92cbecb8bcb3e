"""DistMuonAdamW: AdamW / NorMuon over the gradient engine's shards (mint/optim/dist/muon_adamw.py).

With a :class:`~mint_b200.parallel.zero.GradEngine` attached to the parameters:

* AdamW groups update this rank's shard of every bucket with one fused kernel per bucket
  (element-granular shards, same as the reference's flat slices);
* NorMuon groups update whole matrices on their owner rank (owner buckets), so Polar-Express
  runs on complete matrices. The reference flattens shards to 1-D and thereby degenerates
  Muon to a plain normalization (mint/optim/dist/muon_adamw.py:250-254, 129-130);
* after the step the engine all-gathers updated shards (ZeRO-1/2) or keeps them (ZeRO-3).

``state_dict()`` is per parameter with full tensors (``step, exp_avg, exp_avg_sq`` or
``momentum_buffer, second_momentum_buffer``) independent of the dp layout; on a ZeRO run it is
a collective (every rank must call it) and ``load_state_dict`` re-shards for the current layout.
"""

from __future__ import annotations

from collections.abc import Callable
from typing import Any

import torch
import torch.distributed as dist
from torch.optim import Optimizer

from mint_b200.optim.functional import POLAR_EXPRESS_COEFFS, NorMuonStack, adamw_update, normuon_update_batched
from mint_b200.optim.muon_adamw import AdamConfig, MuonAdamWConfig, MuonConfig


class DistMuonAdamWConfig(MuonAdamWConfig):
    pass


class DistMuonAdamW(Optimizer):
    def __init__(self, param_groups: list[dict], group: dist.ProcessGroup | None = None) -> None:
        super().__init__(param_groups, defaults={})
        self.process_group = group
        self._engine = None
        for g in self.param_groups:
            for p in g["params"]:
                eng = getattr(p, "_grad_engine", None)
                if eng is not None:
                    self._engine = eng
                    break
        # per-unit state, keyed by (param id, piece offset)
        self._shard_state: dict[int, dict[str, Any]] = {}
        # stacked NorMuon state per (group, shape, dtype, tp split) of the matrices this rank updates
        self._muon_stacks: dict[tuple, dict[str, Any]] = {}
        if self._engine is not None:
            # the update kernels read the clip coefficient on the device: no separate scaling pass
            self._engine.defer_clip = self._engine.clip_on_device()

    def _grad_scale(self):  # noqa: ANN202
        eng = self._engine
        return None if eng is None else eng.grad_scale

    @property
    def engine(self):  # noqa: ANN201
        return self._engine

    def zero_grad(self, set_to_none: bool = True) -> None:  # noqa: ARG002
        if self._engine is not None:
            self._engine.zero_grad()
            # params outside the engine (frozen or foreign) follow torch semantics
            for g in self.param_groups:
                for p in g["params"]:
                    if id(p) not in self._engine.by_param:
                        p.grad = None
            return
        super().zero_grad(set_to_none=True)

    # ------------------------------------------------------------------ units
    def _bucket_shard(self, b) -> tuple[torch.Tensor, torch.Tensor, int]:  # noqa: ANN001
        """(param shard, grad shard, shard offset in bucket coordinates) of bucket ``b`` on this rank."""
        eng = self._engine
        if eng.level == 0 or eng.dp == 1:
            return b.data, b.grad, 0
        lo = eng.rank * b.shard
        gv = b.grad[lo : lo + b.shard] if eng.level == 1 else b.grad_shard
        return b.shard_data, gv, lo

    def _ensure_bucket_state(self, b) -> dict:  # noqa: ANN001
        """Bucket-level AdamW moments; every parameter's state holds views into them."""
        st = self._shard_state.get(b.index)
        if st is not None:
            return st
        pv, _gv, lo = self._bucket_shard(b)
        st = {"step": 0, "exp_avg": torch.zeros_like(pv), "exp_avg_sq": torch.zeros_like(pv), "views": []}
        n = pv.numel()
        for sl in b.slots:
            a, e = max(lo, sl.start), min(lo + n, sl.start + sl.numel)
            if a >= e:
                continue
            sub = {"step": 0, "exp_avg": st["exp_avg"][a - lo : e - lo], "exp_avg_sq": st["exp_avg_sq"][a - lo : e - lo],
                   "offset": a - sl.start, "numel": e - a}
            self.state[sl.param][f"shard@{a - sl.start}"] = sub
            st["views"].append(sub)
        self._shard_state[b.index] = st
        return st

    def _step_adamw(self, group: dict) -> None:
        beta1, beta2 = group["betas"]
        eng = self._engine
        ids = {id(p) for p in group["params"]}
        covered: set[int] = set()
        if eng is not None:
            # one fused update per bucket shard whose parameters all belong to this group
            for b in eng.buckets:
                if not all(id(sl.param) in ids for sl in b.slots):
                    continue
                covered.update(id(sl.param) for sl in b.slots)
                pv, gv, _lo = self._bucket_shard(b)
                if gv is None or pv.numel() == 0:
                    continue
                st = self._ensure_bucket_state(b)
                st["step"] += 1
                if eng.push_fusable(b):
                    # ZeRO-2: one kernel updates the shard and stores it into every peer's bucket
                    from mint_b200.ops import _ext  # noqa: PLC0415

                    _ext.require().zero_adamw_push(pv, gv, st["exp_avg"], st["exp_avg_sq"], float(group["lr"]),
                                                   float(beta1), float(beta2), float(group["eps"]),
                                                   float(group["weight_decay"]), int(st["step"]), self._grad_scale(),
                                                   b.extra["symm_data"].ptrs, eng.rank, eng.dp)
                    eng.mark_pushed(b)
                else:
                    adamw_update(pv, gv, st["exp_avg"], st["exp_avg_sq"], st["step"], group["lr"], beta1, beta2,
                                 group["eps"], group["weight_decay"], grad_scale=self._grad_scale())
                for sub in st["views"]:
                    sub["step"] = st["step"]
        for p in group["params"]:
            if id(p) in covered:
                continue
            if eng is None or id(p) not in eng.by_param:
                if p.grad is None:
                    continue
                units = [(p.data, p.grad, self.state[p])]
            else:
                units = []
                for pv, gv, off, n in eng.segments(p):
                    key = f"shard@{off}"
                    st = self.state[p]
                    if key not in st:
                        st[key] = {"step": 0, "exp_avg": torch.zeros_like(pv), "exp_avg_sq": torch.zeros_like(pv),
                                   "offset": off, "numel": n}
                    units.append((pv, gv, st[key]))
            in_engine = eng is not None and id(p) in eng.by_param
            for pv, gv, st in units:
                if "step" not in st:
                    st["step"] = 0
                    st["exp_avg"] = torch.zeros_like(pv)
                    st["exp_avg_sq"] = torch.zeros_like(pv)
                st["step"] += 1
                adamw_update(pv, gv, st["exp_avg"], st["exp_avg_sq"], st["step"], group["lr"], beta1, beta2,
                             group["eps"], group["weight_decay"],
                             grad_scale=self._grad_scale() if in_engine else None)

    def _muon_units(self, group: dict) -> list[tuple[torch.Tensor, torch.Tensor, torch.Tensor]]:
        """(param, this rank's whole matrix view, its gradient view) for every matrix this rank updates."""
        eng = self._engine
        units = []
        for p in group["params"]:
            if len(getattr(p, "_orig_shape", p.shape)) != 2:
                raise ValueError("NorMuon groups must hold 2-D matrices")
            if eng is not None and id(p) in eng.by_param:
                if not eng.owns_whole(p):
                    continue
                (pv, gv, off, n), = eng.segments(p)
                _b, slot = eng.slot(p)
                # (ZeRO-3 has released p's full storage by now: compare against the slot)
                assert off == 0 and n == slot.numel, "owner buckets hold whole matrices"
                units.append((p, pv.view(slot.shape), gv.view(slot.shape)))
            else:
                if p.grad is None:
                    continue
                units.append((p, p.data, p.grad))
        return units

    def _muon_stack_state(self, key: tuple, members: list[torch.Tensor], shape: torch.Size, device) -> dict:  # noqa: ANN001
        """Stacked NorMuon state of one shape group; every parameter's state holds views into it."""
        st = self._muon_stacks.get(key)
        if st is not None and st["params"] == [id(p) for p in members]:
            return st
        rows, cols = self._full_shape(members[0], shape)
        sshape = (rows, 1) if rows >= cols else (1, cols)
        n = len(members)
        mb = torch.zeros((n, *shape), dtype=torch.float32, device=device)
        smb = torch.zeros((n, *sshape), dtype=torch.float32, device=device)
        for i, p in enumerate(members):
            old = self.state.get(p, {})
            if "momentum_buffer" in old:  # e.g. loaded from a checkpoint: move into the stack
                mb[i].copy_(old["momentum_buffer"].reshape(shape))
                smb[i].copy_(old["second_momentum_buffer"].reshape(sshape))
            self.state[p]["momentum_buffer"] = mb[i]
            self.state[p]["second_momentum_buffer"] = smb[i]
        st = {"params": [id(p) for p in members], "mb": mb, "smb": smb}
        self._muon_stacks[key] = st
        return st

    def _step_muon(self, group: dict) -> None:
        """NorMuon on every matrix this rank owns, batched by (shape, tensor-parallel split): one
        Nesterov / Polar-Express / rescale / update sequence per shape group instead of per matrix."""
        by_key: dict[tuple, list[tuple[torch.Tensor, torch.Tensor, torch.Tensor]]] = {}
        for p, pm, gm in self._muon_units(group):
            tp_group, tp_dim = self._tp_of(p)
            key = (id(group), tuple(pm.shape), pm.dtype, tp_group is not None, tp_dim)
            by_key.setdefault(key, []).append((p, pm, gm))
        for key, units in by_key.items():
            members = [u[0] for u in units]
            shape = units[0][1].shape
            st = self._muon_stack_state(key, members, shape, units[0][1].device)
            tp_group, tp_dim = self._tp_of(members[0])
            pviews, gviews = [u[1] for u in units], [u[2] for u in units]
            if NorMuonStack.supported(pviews, gviews):
                dev = st.get("device_stack")
                if dev is None:
                    n = len(units)
                    dev = NorMuonStack(pviews, gviews, st["mb"], st["smb"].view(n, -1), tp_group=tp_group, tp_dim=tp_dim)
                    st["device_stack"] = dev
                dev.bind(pviews, gviews)
                push = self._push_table(st, members, pviews)
                dev.step(lr=group["lr"], momentum=group["momentum"],
                         beta2=group["beta2"] if group.get("beta2") is not None else 0.0,
                         wd=group["weight_decay"], ns_steps=group.get("ns_steps", 5), grad_scale=self._grad_scale(),
                         peer_ptrs=push, rank=self._engine.rank if push is not None else 0,
                         world=self._engine.dp if push is not None else 1)
                if push is not None:
                    self._engine.mark_pushed(params=members)
                continue
            grads = torch.stack([u[2].float() for u in units])
            gs = self._grad_scale()
            if gs is not None:
                grads.mul_(gs)
            normuon_update_batched(
                [u[1] for u in units], grads, st["mb"], st["smb"],
                lr=group["lr"], momentum=group["momentum"],
                beta2=group["beta2"] if group.get("beta2") is not None else 0.0,
                wd=group["weight_decay"], ns_steps=group.get("ns_steps", 5), tp_group=tp_group, tp_dim=tp_dim,
            )

    def _push_table(self, st: dict, members: list[torch.Tensor], pviews: list[torch.Tensor]) -> torch.Tensor | None:
        """[n * dp] peer addresses of the owned matrices when their buckets live in symmetric peer
        memory (ZeRO-2): ``normuon_apply`` then stores the new values into every peer's copy."""
        eng = self._engine
        if eng is None:
            return None
        buckets = [eng.slot(p)[0] for p in members]
        if not all(eng.push_fusable(b) for b in buckets):
            return None
        key = tuple(v.data_ptr() for v in pviews)
        cached = st.get("push_table")
        if cached is not None and cached[0] == key:
            return cached[1]
        rows = [eng.peer_pointers(b, v) for b, v in zip(buckets, pviews, strict=True)]
        table = torch.tensor([a for row in rows for a in row], dtype=torch.int64, device=pviews[0].device)
        st["push_table"] = (key, table)
        return table

    def _tp_of(self, p: torch.Tensor):  # noqa: ANN202
        """(TP group, split dim) for a tensor-parallel sharded parameter, else (None, 0)."""
        eng = self._engine
        if eng is None or not getattr(p, "_tp_sharded", False) or eng.parallel.tp_size <= 1:
            return None, 0
        return eng.tp_group, getattr(p, "_tp_dim", 0)

    def _full_shape(self, p: torch.Tensor, local: torch.Size) -> tuple[int, int]:
        group, dim = self._tp_of(p)
        if group is None:
            return tuple(local)
        size = self._engine.parallel.tp_size
        return (local[0] * size, local[1]) if dim == 0 else (local[0], local[1] * size)

    def _tp_consolidate(self, p: torch.Tensor, t: torch.Tensor, name: str) -> torch.Tensor:
        """Full-matrix view of a per-parameter state tensor under TP (collective over the TP group)."""
        group, dim = self._tp_of(p)
        if group is None or name == "second_momentum_buffer":
            return t
        size = self._engine.parallel.tp_size
        parts = [torch.empty_like(t) for _ in range(size)]
        dist.all_gather(parts, t.contiguous(), group=group)
        return torch.cat(parts, dim=dim)

    @torch.no_grad()
    def step(self, closure: Callable[[], float] | None = None) -> float | None:  # type: ignore[override]
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        eng = self._engine
        if eng is not None and not getattr(eng, "_synced", False):
            eng.finish_grad_sync()
            eng.sync_tp_partial_grads()
        for group in self.param_groups:
            kind = group.get("kind", "adamw")
            if kind == "adamw":
                self._step_adamw(group)
            elif kind == "muon":
                self._step_muon(group)
            else:
                raise ValueError(f"Unknown optimizer kind: {kind}")
        if eng is not None:
            eng.after_step()
            eng._synced = False
        from mint_b200.ops.linear import refresh_weight_shadows  # noqa: PLC0415

        refresh_weight_shadows()  # bf16 compute copies of the updated weights, one launch
        return loss

    # ------------------------------------------------------------------ (de)serialization
    def _full_state_tensor(self, p: torch.Tensor, st: dict, name: str) -> torch.Tensor:
        """Assemble the full-shaped state ``name`` of ``p`` from this rank's pieces (collective when sharded)."""
        eng = self._engine
        if eng is None or id(p) not in eng.by_param or eng.level == 0 or eng.dp == 1:
            for key, sub in st.items():
                if key.startswith("shard@"):
                    return sub[name].view(p.shape if p.numel() else eng.slot(p)[1].shape)
            return st[name]
        b, slot = eng.slot(p)
        buf = torch.zeros(b.size, dtype=torch.float32, device=b.shard_data.device)
        lo = eng.rank * b.shard
        for key, sub in st.items():
            if key.startswith("shard@"):
                off = sub["offset"]
                a = slot.start + off
                buf[a : a + sub["numel"]].copy_(sub[name])
        if name in st and isinstance(st[name], torch.Tensor) and st[name].shape == slot.shape:
            buf[slot.start : slot.start + slot.numel].copy_(st[name].reshape(-1))
        dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=eng.group)
        del lo
        return buf[slot.start : slot.start + slot.numel].view(slot.shape)

    def state_dict(self) -> dict[str, Any]:  # type: ignore[override]
        groups = []
        state: dict[int, dict[str, Any]] = {}
        idx = 0
        eng = self._engine
        for g in self.param_groups:
            ids = []
            for p in g["params"]:
                st = self.state.get(p, {})
                full: dict[str, Any] = {}
                kind = g.get("kind", "adamw")
                if kind == "adamw":
                    steps = [sub["step"] for k, sub in st.items() if k.startswith("shard@")]
                    if not steps and "step" in st:
                        steps = [st["step"]]
                    step = max(steps) if steps else 0
                    if eng is not None and eng.dp > 1 and eng.level > 0:
                        t = torch.tensor([step], dtype=torch.float64, device=eng.buckets[0].shard_data.device)
                        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=eng.group)
                        step = int(t.item())
                    if step > 0:
                        full["step"] = step
                        for nm in ("exp_avg", "exp_avg_sq"):
                            t = self._full_state_tensor(p, st, nm)
                            full[nm] = self._tp_consolidate(p, t, nm).detach().cpu().clone()
                else:
                    have = "momentum_buffer" in st
                    shape = p.shape if eng is None or id(p) not in eng.by_param else eng.slot(p)[1].shape
                    mb = st["momentum_buffer"] if have else torch.zeros(shape, dtype=torch.float32,
                                                                          device=self._device_of(p))
                    rows, cols = self._full_shape(p, shape)
                    sshape = (rows, 1) if rows >= cols else (1, cols)
                    smb = st["second_momentum_buffer"] if have else torch.zeros(sshape, dtype=torch.float32,
                                                                                 device=mb.device)
                    if eng is not None and id(p) in eng.by_param and eng.dp > 1 and eng.level > 0:
                        mb, smb = mb.clone(), smb.clone()
                        if not eng.owns_whole(p):
                            mb.zero_()
                            smb.zero_()
                        flag = torch.tensor([1.0 if have else 0.0], device=mb.device)
                        dist.all_reduce(mb, group=eng.group)
                        dist.all_reduce(smb, group=eng.group)
                        dist.all_reduce(flag, group=eng.group)
                        have = flag.item() > 0
                    if have:
                        full["momentum_buffer"] = self._tp_consolidate(p, mb, "momentum_buffer").detach().cpu().clone()
                        full["second_momentum_buffer"] = smb.detach().cpu().clone()
                if full:
                    state[idx] = full
                ids.append(idx)
                idx += 1
            gcopy = {k: v for k, v in g.items() if k != "params"}
            gcopy["params"] = ids
            groups.append(gcopy)
        return {"state": state, "param_groups": groups}

    def _tp_local(self, p: torch.Tensor, st: dict) -> dict:
        group, dim = self._tp_of(p)
        if group is None:
            return st
        size, rank = self._engine.parallel.tp_size, self._engine.parallel.tp_rank
        out = dict(st)
        for nm in ("exp_avg", "exp_avg_sq", "momentum_buffer"):
            if nm in st:
                out[nm] = st[nm].chunk(size, dim=dim)[rank]
        return out

    def _device_of(self, p: torch.Tensor) -> torch.device:
        eng = self._engine
        if eng is not None and id(p) in eng.by_param:
            return eng.slot(p)[0].shard_data.device
        return p.device

    def load_state_dict(self, state_dict: dict[str, Any]) -> None:  # type: ignore[override]
        saved_groups = state_dict["param_groups"]
        if len(saved_groups) != len(self.param_groups):
            raise ValueError("optimizer state has a different number of param groups")
        eng = self._engine
        self.state.clear()
        self._shard_state.clear()
        self._muon_stacks.clear()
        for g, sg in zip(self.param_groups, saved_groups, strict=True):
            for k, v in sg.items():
                if k != "params":
                    g[k] = v
            for p, pid in zip(g["params"], sg["params"], strict=True):
                st_saved = state_dict["state"].get(pid, state_dict["state"].get(str(pid)))
                if not st_saved:
                    continue
                st_saved = self._tp_local(p, st_saved)
                if g.get("kind", "adamw") == "adamw":
                    if eng is None or id(p) not in eng.by_param:
                        dev = p.device
                        self.state[p] = {"step": int(st_saved["step"]),
                                         "exp_avg": st_saved["exp_avg"].to(dev, torch.float32).view_as(p).clone(),
                                         "exp_avg_sq": st_saved["exp_avg_sq"].to(dev, torch.float32).view_as(p).clone()}
                        continue
                    bkt, _slot = eng.slot(p)
                    bst = self._ensure_bucket_state(bkt)
                    bst["step"] = int(st_saved["step"])
                    for key, sub in self.state[p].items():
                        if not key.startswith("shard@"):
                            continue
                        off, n = sub["offset"], sub["numel"]
                        sub["exp_avg"].copy_(st_saved["exp_avg"].reshape(-1)[off : off + n])
                        sub["exp_avg_sq"].copy_(st_saved["exp_avg_sq"].reshape(-1)[off : off + n])
                        sub["step"] = int(st_saved["step"])
                else:
                    if eng is not None and id(p) in eng.by_param and not eng.owns_whole(p):
                        continue
                    dev = self._device_of(p)
                    self.state[p] = {
                        "momentum_buffer": st_saved["momentum_buffer"].to(dev, torch.float32).clone(),
                        "second_momentum_buffer": st_saved["second_momentum_buffer"].to(dev, torch.float32).clone(),
                    }


__all__ = ["POLAR_EXPRESS_COEFFS", "AdamConfig", "DistMuonAdamW", "DistMuonAdamWConfig", "MuonConfig"]
