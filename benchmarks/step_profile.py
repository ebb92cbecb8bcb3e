#!/usr/bin/env python
"""Per-kernel device-time breakdown of the bench.py training step (torch.profiler / CUPTI).

    python benchmarks/step_profile.py [--steps 2] [--warmup 3] [--matrix-optimizer muon] [--out DIR]
    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \
        benchmarks/step_profile.py --gpus 2 --out DIR

Runs the same model, layout and inputs as ``bench.py`` and records ``--steps`` full steps under
``torch.profiler`` (kernel activity only). Every rank writes ``<out>/step_profile_rank<R>.txt``:
kernels grouped by name with their total device time, and the same grouped into categories
(tcgen05 GEMM, fused TP GEMM, attention, norms, cross-entropy, NCCL, PyTorch elementwise, ...).
The numbers are kernel durations summed per step, so kernels that overlap on different streams
(the ZeRO comm stream, NCCL) add up to more than the step time: compare shares between runs,
and take step times from ``bench.py``.
"""

from __future__ import annotations

import argparse
import sys
from collections import defaultdict
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

CATEGORIES = [
    ("fused TP GEMM (AG/RS)", ("gemm_ag", "gemm_rs")),
    ("tcgen05 GEMM", ("gemm::",)),
    ("attention", ("fa::", "fab::", "fa_fwd", "fa_bwd", "doc_bounds")),
    ("norms / qk-norm+rope", ("rmsnorm", "qk_norm")),
    ("geglu", ("geglu",)),
    ("cross-entropy", ("ce_",)),
    ("embedding", ("embedding",)),
    ("optimizer kernels", ("adamw", "normuon", "grad_norm", "sumsq")),
    ("ZeRO peer collectives", ("zero_",)),
    ("NCCL", ("nccl",)),
    ("PyTorch elementwise / reduce", ("at::", "void at::", "elementwise", "reduce_kernel", "multi_tensor")),
    ("memcpy / memset", ("Memcpy", "Memset", "memcpy", "memset")),
]


def category(name: str) -> str:
    for cat, keys in CATEGORIES:
        if any(k in name for k in keys):
            return cat
    return "other"


def main() -> None:
    import torch
    from torch.profiler import ProfilerActivity, profile

    import bench

    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--model", choices=list(bench.MODELS), default="d12")
    ap.add_argument("--micro-batch", type=int, default=0)
    ap.add_argument("--matrix-optimizer", choices=["muon", "adamw"], default="muon")
    ap.add_argument("--out", default="profiles_out")
    args = ap.parse_args()

    world, rank, _local, dist = bench.dist_setup()
    cfg = dict(bench.MODELS[args.model])
    if args.micro_batch:
        cfg["micro_batch"] = args.micro_batch
    lay = bench.layout_for(args.gpus, args.model)
    device, step, _ = bench.build_ours(args, cfg, lay)
    mb, T, V = cfg["micro_batch"], cfg["seq_length"], cfg["vocab_size"]
    gen = torch.Generator().manual_seed(4321 + rank // lay["tp"])
    row = torch.randint(0, V, (mb, T + 1), generator=gen)
    x, y = row[:, :-1].contiguous().cuda(), row[:, 1:].contiguous().cuda()
    mask = torch.ones(mb, T, device="cuda", dtype=torch.float32)
    doc = (torch.arange(T, device="cuda") // (T // bench.DOCS_PER_ROW)).to(torch.int32).expand(mb, -1).contiguous()
    for _ in range(args.warmup):
        step(x, y, mask, doc)
    torch.cuda.synchronize()
    bench.barrier()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(args.steps):
            step(x, y, mask, doc)
        torch.cuda.synchronize()
    per_name: dict[str, list[float]] = defaultdict(lambda: [0.0, 0])
    for ev in prof.events():
        if ev.device_type != torch.autograd.DeviceType.CUDA:
            continue
        rec = per_name[ev.name]
        rec[0] += ev.device_time_total / 1e3 / args.steps  # ms per step
        rec[1] += 1
    total = sum(v[0] for v in per_name.values())
    cats: dict[str, float] = defaultdict(float)
    for name, (ms, _n) in per_name.items():
        cats[category(name)] += ms
    lines = [f"# step_profile: {args.gpus} GPU(s), rank {rank}, layout {lay}, {args.steps} steps, "
             f"optimizer {args.matrix_optimizer}",
             f"summed kernel time per step: {total:.3f} ms", "", "## categories (ms per step, share)"]
    for cat, ms in sorted(cats.items(), key=lambda kv: -kv[1]):
        lines.append(f"{ms:9.3f}  {100 * ms / max(total, 1e-9):5.1f} %  {cat}")
    lines += ["", "## kernels (ms per step, launches per step, share)"]
    for name, (ms, n) in sorted(per_name.items(), key=lambda kv: -kv[1][0])[:60]:
        lines.append(f"{ms:9.3f}  {n / args.steps:7.1f}  {100 * ms / max(total, 1e-9):5.1f} %  {name[:150]}")
    out = Path(args.out)
    out.mkdir(parents=True, exist_ok=True)
    (out / f"step_profile_{args.gpus}gpu_rank{rank}.txt").write_text("\n".join(lines) + "\n")
    if rank == 0:
        print("\n".join(lines[:40]))
    if dist.is_available() and dist.is_initialized():
        bench.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
