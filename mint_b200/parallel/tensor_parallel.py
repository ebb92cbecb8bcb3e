"""Apply a glob-matched tensor-parallel plan to a model (mint/utils/parallel.py:361-426).

Plan format is the reference's: ``{"blocks.*.gqa.wq": "col", "blocks.*.gqa.wo": "row", ...}``
where ``col`` splits a weight's rows (output features) and ``row`` splits its columns.
Differences from the reference, all for correct gradients:

* attention / FFN modules get a :class:`TPInfo`; they insert the f/g operators themselves,
  so TP without SP also all-reduces input gradients;
* the (tied) embedding and LM head become vocab-parallel (row shards of the table), so the
  LM head's input gradient really is partial and its reduce-scatter is correct;
* replicated parameters whose gradients are partial across TP ranks are tagged
  ``_tp_partial_grad`` and summed over the TP group by the gradient engine.
"""

from __future__ import annotations

import fnmatch

from torch import nn

from mint_b200.nn.attn import GroupedQueryAttention
from mint_b200.nn.ffn import GLU
from mint_b200.nn.norm import RMSNorm
from mint_b200.parallel.context import ParallelContext
from mint_b200.parallel.tp import TPInfo


def _match_plan(name: str, plan: dict[str, str]) -> str | None:
    for pattern, kind in plan.items():
        if fnmatch.fnmatch(name, pattern):
            return kind
    return None


def _shard_linear(module: nn.Linear, dim: int, size: int, rank: int) -> None:
    w = module.weight
    if w.shape[dim] % size != 0:
        raise ValueError(f"cannot split weight {tuple(w.shape)} dim {dim} over tp={size}")
    module.weight = nn.Parameter(w.detach().chunk(size, dim=dim)[rank].contiguous(), requires_grad=w.requires_grad)
    if module.bias is not None and dim == 0:
        b = module.bias
        module.bias = nn.Parameter(b.detach().chunk(size, dim=0)[rank].contiguous(), requires_grad=b.requires_grad)
    module.out_features, module.in_features = module.weight.shape


def apply_tp(model: nn.Module, parallel: ParallelContext, tp_plan: dict[str, str] | None = None) -> nn.Module:
    if parallel.tp_size <= 1:
        return model
    plan = tp_plan or getattr(getattr(model, "config", None), "tp_plan", None)
    if not plan:
        return model
    size, rank = parallel.tp_size, parallel.tp_rank
    tp = TPInfo(group=parallel.tp_group, size=size, rank=rank, sp=parallel.sp)

    kinds: dict[str, str] = {}
    for name, module in list(model.named_modules()):
        kind = _match_plan(name, plan)
        if kind is None or not isinstance(module, nn.Linear):
            continue
        if kind not in ("col", "row"):
            raise ValueError(f"unknown TP kind {kind!r} for {name}")
        _shard_linear(module, 0 if kind == "col" else 1, size, rank)
        module.weight._tp_sharded = True
        module.weight._tp_dim = 0 if kind == "col" else 1
        kinds[name] = kind

    for name, module in model.named_modules():
        prefix = f"{name}." if name else ""
        if isinstance(module, GroupedQueryAttention):
            want = {"wq": "col", "wk": "col", "wv": "col", "wo": "row"}
            got = {k: kinds.get(prefix + k) for k in want}
            if got != want:
                raise NotImplementedError(f"{name}: TP plan must shard q/k/v by column and o by row, got {got}")
            if module.n_heads % size or module.n_kv_heads % size:
                raise ValueError(f"{name}: n_heads={module.n_heads}, n_kv_heads={module.n_kv_heads} not divisible by tp={size}")
            module.n_heads //= size
            module.n_kv_heads //= size
            module.tp = tp
            for p in (module.q_norm.scale, module.k_norm.scale):
                p._tp_partial_grad = True  # each rank normalizes different heads
        elif isinstance(module, GLU):
            want = {"fc1": "col", "fc2": "col", "fc3": "row"}
            got = {k: kinds.get(prefix + k) for k in want}
            if got != want:
                raise NotImplementedError(f"{name}: TP plan must shard fc1/fc2 by column and fc3 by row, got {got}")
            module.tp = tp

    if parallel.sp:
        for name, module in model.named_modules():
            if isinstance(module, RMSNorm) and not name.endswith(("q_norm", "k_norm")):
                module.scale._tp_partial_grad = True  # norms run on sequence shards

    emb = getattr(model, "tok_embeddings", None)
    out = getattr(model, "output", None)
    if isinstance(emb, nn.Embedding):
        rows = emb.weight.shape[0]
        if rows % size != 0:
            raise ValueError(
                f"vocab rows {rows} not divisible by tp={size}; set pad_vocab_multiple to a multiple of {size}"
            )
        tied = out is not None and out.weight is emb.weight
        shard = nn.Parameter(emb.weight.detach().chunk(size, dim=0)[rank].contiguous())
        shard._tp_sharded = True
        shard._tp_dim = 0
        emb.weight = shard
        emb.num_embeddings = shard.shape[0]
        if isinstance(out, nn.Linear):
            if tied:
                out.weight = shard
            else:
                out.weight = nn.Parameter(out.weight.detach().chunk(size, dim=0)[rank].contiguous())
                out.weight._tp_sharded = True
                out.weight._tp_dim = 0
            out.out_features = out.weight.shape[0]
        model.vocab_start = rank * shard.shape[0]
    model.tp = tp
    return model
