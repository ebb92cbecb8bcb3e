"""Worker for test_fused_tp.py, launched by torchrun with one rank per GPU.

Checks the fused tensor-parallel kernels against NCCL collectives + an fp32 reference GEMM:
  1. all-gather -> GEMM (weights K-major and MN-major), three calls in a row;
  2. GEMM -> reduce-scatter (both weight layouts), three calls in a row;
  3. GEMM -> all-reduce (tensor parallelism without SP), both weight layouts;
  4. a small Gemma (tp = world), with and without sequence parallelism: loss and every gradient
     with the fused kernels against the same model on the NCCL path.
Prints one line per check and exits non-zero on a mismatch.
"""

from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[2]))


def rel(a: torch.Tensor, b: torch.Tensor) -> float:
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


def main() -> None:
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120))
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)
    from mint_b200.ops import _ext
    from mint_b200.parallel import fused

    comm = fused.TPComm(dist.group.WORLD, dev)
    failures = 0
    B, seg, K, N = 2, 512, 768, 1152
    T = seg * world
    for it in range(3):
        g = torch.Generator(device="cuda").manual_seed(100 + it)
        w = torch.randn(N, K, device=dev, dtype=torch.bfloat16, generator=g) * 0.05
        torch.manual_seed(1000 * it + rank)
        x_local = torch.randn(B, seg, K, device=dev, dtype=torch.bfloat16)
        parts = [torch.empty_like(x_local) for _ in range(world)]
        dist.all_gather(parts, x_local)
        full = torch.cat(parts, dim=1)  # [B, T, K]
        for kmajor in (True, False):
            slot, buf = comm.acquire(B * T * K * 2)
            buf.view((B, world, seg, K), torch.bfloat16)[:, rank].copy_(x_local)
            wb = w if kmajor else w.t().contiguous()
            y = comm.gemm_ag(buf, B * T, K, wb, kmajor, seg)
            comm.mark_read_by_peers(slot)
            comm.release(slot)
            ref = full.reshape(B * T, K).float() @ w.float().t()
            e = rel(y, ref)
            ok = e < 1e-2
            failures += not ok
            print(f"[rank {rank}] all-gather->GEMM call {it} kmajor={kmajor}: rel err {e:.2e} {'OK' if ok else 'FAIL'}",
                  flush=True)
        # GEMM -> reduce-scatter: every rank's A differs; the sum is taken over ranks
        a = torch.randn(B * T, K, device=dev, dtype=torch.bfloat16)
        total = (a.float() @ w.float().t())
        dist.all_reduce(total)
        want = total.view(B, world, seg, N)[:, rank].reshape(B * seg, N)
        for kmajor in (True, False):
            wb = w if kmajor else w.t().contiguous()
            out = comm.gemm_rs(a, wb, kmajor, seg)
            e = rel(out, want)
            ok = e < 1e-2
            failures += not ok
            print(f"[rank {rank}] GEMM->reduce-scatter call {it} kmajor={kmajor}: rel err {e:.2e} "
                  f"{'OK' if ok else 'FAIL'}", flush=True)
            # GEMM -> all-reduce (no SP): the full sum on every rank
            full_out = comm.gemm_ar(a, wb, kmajor)
            e = rel(full_out, total)
            ok = e < 1e-2
            failures += not ok
            print(f"[rank {rank}] GEMM->all-reduce call {it} kmajor={kmajor}: rel err {e:.2e} "
                  f"{'OK' if ok else 'FAIL'}", flush=True)
    torch.cuda.synchronize()
    _ext.check_device_status()

    # NorMuon on tensor-parallel shards (norms all-reduced, bf16 shards all-gathered, each rank
    # updating its slice) against the same update of the whole matrices on one rank
    from mint_b200.optim.functional import NorMuonStack

    for tp_dim, shape in ((0, (512, 256)), (1, (256, 512))):
        torch.manual_seed(5)
        full_p = [torch.randn(shape, device=dev) * 0.02 for _ in range(3)]
        full_g = [torch.randn(shape, device=dev) * 1e-3 for _ in range(3)]
        rows, cols = shape
        J = rows if rows >= cols else cols
        ref_p = [t.clone() for t in full_p]
        ref = NorMuonStack(ref_p, [t.clone() for t in full_g], torch.zeros(3, rows, cols, device=dev),
                           torch.zeros(3, J, device=dev))
        ref.step(lr=0.02, momentum=0.95, beta2=0.9, wd=0.1, ns_steps=5)
        # clones: a dim-0 chunk of a contiguous tensor is already contiguous (a view, not a copy)
        sh_p = [t.chunk(world, dim=tp_dim)[rank].clone().contiguous() for t in full_p]
        sh_g = [t.chunk(world, dim=tp_dim)[rank].clone().contiguous() for t in full_g]
        st = NorMuonStack(sh_p, sh_g, torch.zeros(3, *sh_p[0].shape, device=dev), torch.zeros(3, J, device=dev),
                          tp_group=dist.group.WORLD, tp_dim=tp_dim)
        st.step(lr=0.02, momentum=0.95, beta2=0.9, wd=0.1, ns_steps=5)
        torch.cuda.synchronize()
        worst = max(rel(got - full_p[i].chunk(world, dim=tp_dim)[rank],
                        ref_p[i].chunk(world, dim=tp_dim)[rank] - full_p[i].chunk(world, dim=tp_dim)[rank])
                    for i, got in enumerate(sh_p))
        ok = worst < 1e-2
        failures += not ok
        print(f"[rank {rank}] NorMuon tp_dim={tp_dim}: update rel err {worst:.2e} {'OK' if ok else 'FAIL'}", flush=True)

    # model-level: fused vs NCCL path on the same weights and batch
    from mint_b200.models.gemma import GemmaConfig
    from mint_b200.scripts.common import build_model
    from mint_b200.trainer.base import BasetrainConfig
    from mint_b200.utils.device import Device, DeviceConfig

    cfg = GemmaConfig(embed_dim=256, hidden_dim=512, seq_length=256 * world, vocab_size=1024, n_layers=2, n_heads=2 * world,
                      n_kv_heads=2 * world, head_dim=128, rope_base_theta=10000)
    tcfg = BasetrainConfig(use_meta_device=True, compile_model=False, gradient_checkpointing=False)
    for sp in (True, False):
        device = Device(DeviceConfig(mixed_precision=True, tp_size=world, ddp_level=0, sp=sp))
        results = {}
        for mode in ("0", "1"):
            os.environ["MINT_FUSED_TP"] = mode
            model = build_model(cfg, tcfg, device, seed=7)
            torch.manual_seed(11)
            x = torch.randint(0, cfg.vocab_size, (2, cfg.seq_length), device=dev)
            y = torch.randint(0, cfg.vocab_size, (2, cfg.seq_length), device=dev)
            m = torch.ones(2, cfg.seq_length, device=dev)
            with device.autocast():
                loss = model.loss(x, y, m)
            loss.backward()
            grads = {n: p.grad.detach().float().clone() for n, p in model.named_parameters() if p.grad is not None}
            results[mode] = (float(loss.detach()), grads)
        l0, g0 = results["0"]
        l1, g1 = results["1"]
        ok = abs(l0 - l1) < 2e-2 * abs(l0)
        failures += not ok
        print(f"[rank {rank}] model sp={sp} loss NCCL {l0:.5f} fused {l1:.5f} {'OK' if ok else 'FAIL'}", flush=True)
        worst = max(rel(g1[n], g0[n]) for n in g0)
        ok = worst < 5e-2 and set(g0) == set(g1)
        failures += not ok
        print(f"[rank {rank}] model sp={sp} grads worst rel err {worst:.2e} over {len(g0)} params "
              f"{'OK' if ok else 'FAIL'}", flush=True)
    torch.cuda.synchronize()
    _ext.check_device_status()
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(1 if failures else 0)


if __name__ == "__main__":
    main()
