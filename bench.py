#!/usr/bin/env python
"""Pretraining throughput benchmark (BASELINE.json metric: pretrain tokens/sec, device-timed, max over ranks).

Config (config 2): Gemma-style d12 decoder -- 12 layers, d_model 768, 6 heads x 128
(MHA), GeGLU ffn 3072, RoPE theta 10000, tied embeddings, vocab 65,536 -- seq 2048, micro-batch 32
per dp rank, next-token CE on uniform-random token ids (random-init weights), NorMuon (Polar
Express, 5 iterations) on block matrices and AdamW elsewhere, bf16 autocast, grad clip 1.0.
Every row holds two documents of seq/2 tokens (doc ids 0 and 1), the input the reference's own
benchmark worker gives its model (scripts/benchmark.py:258-263), so attention is causal within each
document on both arms.
Layouts: 1 GPU single; 2 GPUs tp=2 sp; 4 GPUs tp=2 sp ZeRO-2 dp=2; 8 GPUs tp=2 sp ZeRO-2 dp=4.

    python bench.py [--gpus 1] [--steps K] [--warmup W]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench.py --gpus N --steps K --warmup W
    python bench.py --impl reference ...      # the unmodified reference (baseline/_ref) on the same config

Timing: W untimed warm-up steps; then barrier + synchronize, CUDA events around exactly K full
training steps (forward, backward, gradient collectives, optimizer step), synchronize; the
reported step time is the max over ranks. Each step's working set (8.6 GB of logits alone) is far
larger than the 126 MB L2, so no step reuses the previous step's cache contents. ``e2e`` repeats
the measurement through the public training API with every step's token ids copied host->device
from pinned memory and the loss read back to the host.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

BASELINE_TOKS = None  # BASELINE.md publishes no number for this config
METRIC = "pretrain tokens/sec (device-timed, max over ranks)"
DOCS_PER_ROW = 2

MODELS = {
    "d12": dict(embed_dim=768, hidden_dim=3072, seq_length=2048, vocab_size=65536, n_layers=12, n_heads=6,
                n_kv_heads=6, head_dim=128, rope_base_theta=10000, micro_batch=32),
    "2b": dict(embed_dim=2048, hidden_dim=8192, seq_length=4096, vocab_size=65536, n_layers=24, n_heads=16,
               n_kv_heads=4, head_dim=128, rope_base_theta=10000, micro_batch=8),
}


def layout_for(n: int, model: str) -> dict:
    if model == "2b":
        return {"tp": min(4, n), "sp": n > 1, "ddp_level": 3 if n > 4 else 2}
    if n == 1:
        return {"tp": 1, "sp": False, "ddp_level": 0}
    return {"tp": 2, "sp": True, "ddp_level": 2}


def parallelism_name(n: int, lay: dict) -> str:
    if n == 1:
        return "single"
    dp = n // lay["tp"]
    name = f"tp{lay['tp']}" + ("_sp" if lay["sp"] else "")
    if dp > 1:
        name += f"_zero{lay['ddp_level']}_dp{dp}"
    return name


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self) -> None:
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            self.fh = os.fdopen(fd, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        sm, mx, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        Path(self.path).unlink(missing_ok=True)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "power_w_median": statistics.median(power) if power else None, "samples": len(sm),
                "reasons": sorted(reasons)}


def flops_per_token(cfg: dict) -> float:
    """Reference convention (scripts/benchmark.py:70-82): 6 x matmul params (incl. unpadded head) + attention."""
    d, f, L = cfg["embed_dim"], cfg["hidden_dim"], cfg["n_layers"]
    hq, hkv, hd = cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"]
    blocks = L * (d * hq * hd + 2 * d * hkv * hd + hq * hd * d + 3 * d * f)
    head = cfg["vocab_size"] * d
    attn = 4 * cfg["seq_length"] * hq * hd * L
    return 3 * (2 * (blocks + head) + attn)


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except json.JSONDecodeError:
            pass
    return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0, "fallback": True}


def dist_setup():  # noqa: ANN201
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local, dist


def max_over_ranks(x: float) -> float:
    import torch
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())
    return x


def barrier() -> None:
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        dist.barrier()


# ---------------------------------------------------------------------------------------------- ours
def build_ours(args, cfg: dict, lay: dict):  # noqa: ANN001, ANN201
    import torch

    from mint_b200.models.gemma import GemmaConfig, configure_optimizer
    from mint_b200.optim.muon_adamw import MuonAdamWConfig
    from mint_b200.scripts.common import build_model
    from mint_b200.trainer.base import BasetrainConfig
    from mint_b200.trainer.scheduler import SchedulerConfig
    from mint_b200.utils.device import Device, DeviceConfig

    os.environ.setdefault("MINT_PG_TIMEOUT_S", "300")
    device = Device(DeviceConfig(mixed_precision=True, tp_size=lay["tp"], ddp_level=lay["ddp_level"], sp=lay["sp"]))
    mcfg = GemmaConfig(**{k: v for k, v in cfg.items() if k != "micro_batch"})
    tcfg = BasetrainConfig(use_meta_device=True, compile_model=False, gradient_checkpointing=False)
    model = build_model(mcfg, tcfg, device, seed=1234)
    opt = configure_optimizer(model, mcfg, SchedulerConfig(), MuonAdamWConfig(matrix_optimizer=args.matrix_optimizer),
                              dp_group=device.parallel.dp_group)

    def step(x, y, m, doc):  # noqa: ANN001, ANN202
        with device.autocast():
            loss = model.loss(x, y, m, doc_ids=doc)
        device.backward(loss)
        device.optimizer_step(opt, grad_clip=1.0, params=None)
        opt.zero_grad()
        return loss

    return device, step, torch


# ---------------------------------------------------------------------------------------------- reference
def build_reference(args, cfg: dict, lay: dict):  # noqa: ANN001, ANN201
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "mint").exists():
        raise RuntimeError("reference not installed under baseline/_ref")
    sys.path.insert(0, str(ref))
    import torch
    from mint.models.gemma import Gemma, GemmaConfig, configure_optimizer
    from mint.optim.muon_adamw import MuonAdamWConfig
    from mint.trainer.base import _masked_cross_entropy
    from mint.trainer.scheduler import SchedulerConfig
    from mint.utils.device import Device, DeviceConfig

    device = Device(DeviceConfig(mixed_precision=True, tp_size=lay["tp"], ddp_level=lay["ddp_level"], sp=lay["sp"]))
    mcfg = GemmaConfig(**{k: v for k, v in cfg.items() if k != "micro_batch"})
    torch.manual_seed(1234)
    with torch.device("meta"):
        model = Gemma(mcfg, gradient_checkpointing=False)
    model = device.move_to_device(model, from_meta=True)
    model = device.setup_parallel(model, tp_plan=mcfg.tp_plan)
    model = device.compile_model(model, enabled=True)
    opt = configure_optimizer(model, mcfg, SchedulerConfig(), MuonAdamWConfig(), dp_group=device.parallel.dp_group)
    loss_fn = torch.compile(_masked_cross_entropy)

    def step(x, y, m, doc):  # noqa: ANN001, ANN202
        with device.autocast():
            logits = model(x, doc_ids=doc)
            loss = loss_fn(logits, y, m, None)
        device.backward(loss)
        device.optimizer_step(opt, grad_clip=1.0, params=model.parameters())
        opt.zero_grad(set_to_none=True)
        return loss

    return device, step, torch


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--model", choices=list(MODELS), default="d12")
    ap.add_argument("--micro-batch", type=int, default=0, help="override micro-batch per dp rank")
    ap.add_argument("--matrix-optimizer", choices=["muon", "adamw"], default="muon")
    ap.add_argument("--tp", type=int, default=0, help="override the layout's tensor-parallel size")
    ap.add_argument("--ddp-level", type=int, default=-1, help="override the layout's ZeRO level (0..3)")
    ap.add_argument("--sp", choices=["on", "off"], default=None, help="override sequence parallelism")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-same-optimizer", action="store_true",
                    help="skip the extra all-AdamW measurement (the reference arm's optimizer)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    world, rank, local, _dist = dist_setup()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    cfg = dict(MODELS[args.model])
    if args.micro_batch:
        cfg["micro_batch"] = args.micro_batch
    lay = layout_for(args.gpus, args.model)
    if args.tp:
        lay["tp"] = args.tp
    if args.ddp_level >= 0:
        lay["ddp_level"] = args.ddp_level
    if args.sp is not None:
        lay["sp"] = args.sp == "on"
    if lay["tp"] == 1:
        lay["sp"] = False
    dp = args.gpus // lay["tp"]
    mb, T, V = cfg["micro_batch"], cfg["seq_length"], cfg["vocab_size"]
    par_name = parallelism_name(args.gpus, lay)
    base_line = {"metric": METRIC, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
                 "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "dtype": "bf16",
                 "data": "synthetic (uniform-random token ids, random-init weights)",
                 "config": {"model": f"{args.model} (Gemma-style, {cfg['n_layers']}L d{cfg['embed_dim']} "
                                     f"{cfg['n_heads']}q/{cfg['n_kv_heads']}kv x{cfg['head_dim']}, ffn {cfg['hidden_dim']}, "
                                     f"V {V})",
                            "global_batch": mb * dp, "seq_len": T, "parallelism": par_name,
                            "micro_batch_per_dp_rank": mb,
                            "optimizer": ("NorMuon(matrices)+AdamW" if args.impl == "ours" and args.matrix_optimizer == "muon"
                                          else "AdamW (all groups; reference configure_optimizer)"),
                            "docs_per_row": DOCS_PER_ROW,
                            "tokens_per_gpu_per_step": mb * T * dp // args.gpus,
                            "attention_mask": "causal + same-document (2 docs per row, as the reference benchmark worker); "
                                              "even layers also a seq/4 sliding window",
                            "l2": "per-step working set >> 126 MB L2 (logits alone 8.6 GB); no flush needed"}}
    if args.impl == "reference":
        base_line["impl"] = "reference"
    try:
        builder = build_reference if args.impl == "reference" else build_ours
        device, step, torch = builder(args, cfg, lay)
    except Exception as exc:  # noqa: BLE001
        if rank == 0:
            print(json.dumps({"impl": args.impl, "unavailable": f"{type(exc).__name__}: {exc}"[:400]}), flush=True)
        raise

    gen = torch.Generator().manual_seed(4321 + rank // lay["tp"])
    pinned = []
    for _ in range(2):
        row = torch.randint(0, V, (mb, T + 1), generator=gen)
        pinned.append((row[:, :-1].contiguous().pin_memory(), row[:, 1:].contiguous().pin_memory()))
    dev_batches = [(x.cuda(), y.cuda()) for x, y in pinned]
    mask = torch.ones(mb, T, device="cuda", dtype=torch.float32)
    # two documents per row, as the reference's benchmark worker feeds its model (scripts/benchmark.py:258-263)
    doc = (torch.arange(T, device="cuda") // (T // DOCS_PER_ROW)).to(torch.int32).expand(mb, -1).contiguous()

    for i in range(args.warmup):
        x, y = dev_batches[i % 2]
        loss = step(x, y, mask, doc)
    torch.cuda.synchronize()
    barrier()

    ext = None
    if args.impl == "ours":
        from mint_b200.ops import _ext

        ext = _ext.require()
        _ext.check_device_status()
        _ext.reset_fallbacks()
    launches0 = ext.launch_count() if ext is not None else 0
    sampler = ClockSampler(int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[local])
                           if os.environ.get("CUDA_VISIBLE_DEVICES") else local)
    sampler.start()
    time.sleep(0.3)
    torch.cuda.synchronize()
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(args.steps):
        x, y = dev_batches[i % 2]
        loss = step(x, y, mask, doc)
    end.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    launches = (ext.launch_count() - launches0) if ext is not None else 0
    fallbacks = None
    if ext is not None:
        from mint_b200.ops import _ext

        fallbacks = sum(_ext.fallback_counts().values())  # PyTorch-fallback calls in the timed steps
    ms = start.elapsed_time(end) / args.steps
    ms = max_over_ranks(ms)
    last_loss = float(loss.detach())

    e2e = None
    if not args.no_e2e:
        xin = torch.empty(mb, T, dtype=torch.long, device="cuda")
        yin = torch.empty(mb, T, dtype=torch.long, device="cuda")
        torch.cuda.synchronize()
        barrier()
        s2, e2_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for i in range(args.steps):
            hx, hy = pinned[i % 2]
            xin.copy_(hx, non_blocking=True)
            yin.copy_(hy, non_blocking=True)
            loss = step(xin, yin, mask, doc)
            _ = loss.item()
        e2_.record()
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(s2.elapsed_time(e2_) / args.steps)
        e2e = {"value": mb * T * dp / (e2e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": 2 * mb * T * 8, "d2h_bytes_per_step": 4,
               "how": "H2D of the step's int64 input/target ids from pinned memory + fwd/bwd/optimizer + loss.item()"}
    if ext is not None:
        from mint_b200.ops import _ext

        _ext.check_device_status()

    same_opt = None
    if args.impl == "ours" and args.matrix_optimizer == "muon" and not args.no_same_optimizer:
        # the same step with the reference arm's optimizer (AdamW on every group), so that a ratio
        # against the reference compares identical work; the NorMuon number above stays the headline
        del step
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        args_a = argparse.Namespace(**{**vars(args), "matrix_optimizer": "adamw"})
        _dev2, step_a, _ = build_ours(args_a, cfg, lay)
        for i in range(args.warmup):
            x, y = dev_batches[i % 2]
            step_a(x, y, mask, doc)
        torch.cuda.synchronize()
        barrier()
        sa, ea = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        sa.record()
        for i in range(args.steps):
            x, y = dev_batches[i % 2]
            loss_a = step_a(x, y, mask, doc)
        ea.record()
        torch.cuda.synchronize()
        ms_a = max_over_ranks(sa.elapsed_time(ea) / args.steps)
        same_opt = {"matrix_optimizer": "adamw", "value": mb * T * dp / (ms_a / 1e3), "unit": "tokens/s",
                    "ms_per_step": ms_a, "final_loss": float(loss_a.detach()),
                    "how": "same model, data and timing; AdamW on every parameter group as the reference's "
                           "configure_optimizer (device-timed, max over ranks)"}
        if ext is not None:
            _ext.check_device_status()

    tok_s = mb * T * dp / (ms / 1e3)
    pk = peaks()
    fpt = flops_per_token(cfg)
    tflops_per_gpu = fpt * tok_s / 1e12 / args.gpus
    if rank == 0:
        line = dict(base_line)
        line.update({
            "value": tok_s, "ms_per_step": ms,
            "vs_baseline": (tok_s / BASELINE_TOKS) if BASELINE_TOKS else None,
            "mfu": tflops_per_gpu / 2250.0,
            "tflops_per_gpu": tflops_per_gpu,
            "frac_of_measured_bf16_sustained": tflops_per_gpu / pk.get("bf16_tflops_sustained", 1400.0),
            "clocks": clocks, "gpu_launches": launches, "final_loss": last_loss,
        })
        if fallbacks is not None:
            line["kernel_fallbacks"] = fallbacks
        if e2e is not None:
            line["e2e"] = e2e
        if same_opt is not None:
            line["same_optimizer_as_reference"] = same_opt
        print(json.dumps(line), flush=True)
    if _dist.is_available() and _dist.is_initialized():
        barrier()
        _dist.destroy_process_group()


if __name__ == "__main__":
    main()
