#!/usr/bin/env python
"""DPO training-step throughput (the benchmark plan's DPO configuration).

    python benchmarks/dpo_step.py [--impl ours|reference] [--pairs 16] [--seq 1024] [--ddp-level 3]
    torchrun --nproc-per-node N benchmarks/dpo_step.py --gpus N ...

One step = policy forward + backward on ``pairs`` chosen/rejected sequence pairs per rank, a
no-grad forward of the frozen reference model on the same pairs, the sigmoid DPO loss, and the
optimizer step (d12 policy, synthetic uniform-random ids, random-init weights, labels masked on
the first quarter of every sequence as a prompt). Ours computes the sequence log-probs with the
fused LM head + row-statistics kernels (``Gemma.token_logps``): no fp32 [2B, T, V] log-softmax. The
reference arm runs the reference's own model, ``setup_parallel`` and ``compute_logps`` from
``baseline/_ref``. Device-timed (CUDA events), max over ranks; rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402  (dist_setup / max_over_ranks / barrier / MODELS)


def _batch(torch, pairs: int, seq: int, vocab: int, dev, seed: int):  # noqa: ANN001, ANN202
    g = torch.Generator(device="cpu").manual_seed(seed)
    ids = torch.randint(0, vocab, (2 * pairs, seq), generator=g)
    labels = ids.clone()
    labels[:, : seq // 4] = -100
    return ids.to(dev), labels.to(dev)


def build_ours(args, cfg: dict):  # noqa: ANN001, ANN201
    import torch

    from mint_b200.loss.dpo import DPOLoss, sequence_logps
    from mint_b200.models.gemma import Gemma, GemmaConfig, configure_optimizer
    from mint_b200.optim.muon_adamw import MuonAdamWConfig
    from mint_b200.scripts.common import build_model
    from mint_b200.trainer.base import BasetrainConfig
    from mint_b200.trainer.scheduler import SchedulerConfig
    from mint_b200.utils.device import Device, DeviceConfig

    device = Device(DeviceConfig(mixed_precision=True, tp_size=1, ddp_level=args.ddp_level, sp=False))
    mcfg = GemmaConfig(**cfg)
    tcfg = BasetrainConfig(use_meta_device=True, compile_model=False, gradient_checkpointing=False)
    policy = build_model(mcfg, tcfg, device, seed=1234)
    with torch.device("meta"):
        reference = Gemma(mcfg, gradient_checkpointing=False)
    reference = device.move_to_device(reference, from_meta=True)
    reference.requires_grad_(False)
    opt = configure_optimizer(policy, mcfg, SchedulerConfig(), MuonAdamWConfig(), dp_group=device.parallel.dp_group)
    crit = DPOLoss(beta=0.1)

    def step(ids, labels):  # noqa: ANN001, ANN202
        with device.autocast():
            pc, pr = sequence_logps(policy, ids, labels).chunk(2)
            with torch.no_grad():
                rc, rr = sequence_logps(reference, ids, labels).chunk(2)
            loss, _ = crit(pc, pr, rc, rr)
        device.backward(loss)
        device.optimizer_step(opt, grad_clip=1.0, params=None)
        opt.zero_grad()
        return loss

    return step


def build_reference(args, cfg: dict):  # noqa: ANN001, ANN201
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "mint").exists():
        raise RuntimeError("reference not installed under baseline/_ref")
    sys.path.insert(0, str(ref))
    import torch
    from mint.loss.dpo import DPOLoss, compute_logps
    from mint.models.gemma import Gemma, GemmaConfig, configure_optimizer
    from mint.optim.muon_adamw import MuonAdamWConfig
    from mint.trainer.scheduler import SchedulerConfig
    from mint.utils.device import Device, DeviceConfig

    device = Device(DeviceConfig(mixed_precision=True, tp_size=1, ddp_level=args.ddp_level, sp=False))
    mcfg = GemmaConfig(**cfg)
    torch.manual_seed(1234)
    with torch.device("meta"):
        policy = Gemma(mcfg, gradient_checkpointing=False)
        reference = Gemma(mcfg, gradient_checkpointing=False)
    policy = device.move_to_device(policy, from_meta=True)
    policy = device.setup_parallel(policy, tp_plan=mcfg.tp_plan)
    reference = device.move_to_device(reference, from_meta=True)
    reference.requires_grad_(False)
    opt = configure_optimizer(policy, mcfg, SchedulerConfig(), MuonAdamWConfig(), dp_group=device.parallel.dp_group)
    crit = DPOLoss(beta=0.1)

    def step(ids, labels):  # noqa: ANN001, ANN202
        with device.autocast():
            lc, lr = policy(ids).chunk(2)
            cl, rl = labels.chunk(2)
            pc, pr = compute_logps(lc, cl), compute_logps(lr, rl)
            with torch.no_grad():
                rlc, rlr = reference(ids).chunk(2)
                rc, rr = compute_logps(rlc, cl), compute_logps(rlr, rl)
            out = crit(pc, pr, rc, rr)
            loss = out[0] if isinstance(out, tuple) else out
        device.backward(loss)
        device.optimizer_step(opt, grad_clip=1.0, params=policy.parameters())
        opt.zero_grad(set_to_none=True)
        return loss

    return step


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--pairs", type=int, default=16, help="chosen/rejected pairs per rank")
    ap.add_argument("--seq", type=int, default=1024)
    ap.add_argument("--ddp-level", type=int, default=3)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args()
    world, rank, local, _dist = bench.dist_setup()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    import torch

    cfg = {k: v for k, v in bench.MODELS["d12"].items() if k != "micro_batch"}
    cfg["seq_length"] = args.seq
    line = {"metric": "dpo_tokens_per_sec", "unit": "tokens/s", "impl": args.impl, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "dtype": "bf16",
            "data": "synthetic (uniform-random ids, random-init weights)",
            "config": {"model": "d12 policy + frozen d12 reference", "pairs_per_rank": args.pairs, "seq_len": args.seq,
                       "parallelism": f"zero{args.ddp_level}_dp{world}" if world > 1 else "single"}}
    try:
        step = (build_reference if args.impl == "reference" else build_ours)(args, cfg)
    except Exception as exc:  # noqa: BLE001
        if rank == 0:
            print(json.dumps({**line, "unavailable": f"{type(exc).__name__}: {exc}"[:400]}), flush=True)
        raise
    dev = torch.device("cuda", local)
    batches = [_batch(torch, args.pairs, args.seq, cfg["vocab_size"], dev, 100 * rank + i) for i in range(2)]
    try:
        for i in range(args.warmup):
            step(*batches[i % 2])
        torch.cuda.synchronize()
    except Exception as exc:  # noqa: BLE001
        if args.impl != "reference":
            raise
        # the reference's stock path fails on this box (its Triton attention kernel rejects bf16
        # operands for this shape): report it instead of a number
        if rank == 0:
            print(json.dumps({**line, "unavailable": f"reference step failed: {type(exc).__name__}: {exc}"[:400]}),
                  flush=True)
        if _dist.is_available() and _dist.is_initialized():
            _dist.destroy_process_group()
        return
    bench.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(args.steps):
        loss = step(*batches[i % 2])
    e.record()
    torch.cuda.synchronize()
    ms = bench.max_over_ranks(s.elapsed_time(e) / args.steps)
    tokens = 2 * args.pairs * args.seq * world
    if rank == 0:
        line.update({"value": tokens / (ms / 1e3), "ms_per_step": ms, "pairs_per_sec": args.pairs * world / (ms / 1e3),
                     "final_loss": float(loss.detach()),
                     "peak_mem_gib": torch.cuda.max_memory_allocated() / 2**30})
        print(json.dumps(line), flush=True)
    if _dist.is_available() and _dist.is_initialized():
        bench.barrier()
        _dist.destroy_process_group()


if __name__ == "__main__":
    os.environ.setdefault("MINT_PG_TIMEOUT_S", "300")
    main()
