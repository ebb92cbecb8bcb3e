#!/usr/bin/env python
"""Fused tensor-parallel GEMMs vs the NCCL path (BASELINE config 5 sweep), one rank per GPU:

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 benchmarks/tp_fused.py [--M 8192 32768 131072]

For each M (tokens, sharded over the tp ranks), K = 2048 and N in {2048, 8192}:
  all-gather -> GEMM:  fused kernel  vs  NCCL all_gather_into_tensor + our GEMM  vs  NCCL + cuBLAS
  GEMM -> reduce-scatter: fused kernel vs  our GEMM + NCCL reduce_scatter_tensor  vs  cuBLAS + NCCL
Times are CUDA-event times on each rank's stream, median of --iters, max over ranks. The roofline of
a fused call is the slower of its FLOPs at the measured GEMM peak and the bytes it must move over
NVLink per GPU at the measured 770 GB/s peer bandwidth; `frac` = roofline / achieved.
Rank 0 prints one JSON line per case.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

NVLINK_GBS = 770.0  # measured peer copy bandwidth per direction per GPU on this pool


def gemm_peak_tflops() -> float:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops"])
        except (KeyError, ValueError):
            pass
    return 1590.0


def timed(fn, iters: int) -> float:  # noqa: ANN001
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    ts = []
    for _ in range(iters):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        ts.append(s.elapsed_time(e))
    t = torch.tensor([statistics.median(ts)], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--M", type=int, nargs="+", default=[8192, 32768, 131072])
    ap.add_argument("--N", type=int, nargs="+", default=[2048, 8192])
    ap.add_argument("--K", type=int, default=2048)
    ap.add_argument("--iters", type=int, default=10)
    args = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120))
    rank, world = dist.get_rank(), dist.get_world_size()
    from mint_b200.ops.gemm import matmul
    from mint_b200.parallel import fused

    comm = fused.TPComm(dist.group.WORLD, torch.device("cuda", local))
    peak = gemm_peak_tflops()
    K = args.K
    for M in args.M:
        seg = M // world
        for N in args.N:
            torch.manual_seed(rank)
            w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.02
            x_local = torch.randn(seg, K, device="cuda", dtype=torch.bfloat16) * 0.02
            # all-gather -> GEMM (column-parallel: each rank holds N / world output columns)
            wl = w[: N // world].contiguous()
            # held for the whole measurement: every timed call re-reads the same unchanged shard
            _slot, buf = comm.acquire(M * K * 2)
            buf.view((M, K), torch.bfloat16)[rank * seg : (rank + 1) * seg].copy_(x_local)
            gathered = torch.empty(M, K, device="cuda", dtype=torch.bfloat16)

            def ag_fused():  # noqa: ANN202
                return comm.gemm_ag(buf, M, K, wl, True, seg)

            def ag_nccl_ours():  # noqa: ANN202
                dist.all_gather_into_tensor(gathered, x_local)
                return matmul(gathered, wl, trans_b=True)

            def ag_nccl_cublas():  # noqa: ANN202
                dist.all_gather_into_tensor(gathered, x_local)
                return gathered @ wl.t()

            flop = 2.0 * M * K * (N // world)
            moved = (world - 1) * seg * K * 2  # bytes pulled in per GPU
            roof = max(flop / (peak * 1e12), moved / (NVLINK_GBS * 1e9)) * 1e3
            res = {"op": "allgather_gemm", "tp": world, "M": M, "K": K, "N": N}
            for name, fn in (("fused", ag_fused), ("nccl_ours", ag_nccl_ours), ("nccl_cublas", ag_nccl_cublas)):
                res[f"{name}_ms"] = timed(fn, args.iters)
            res["roofline_ms"] = roof
            res["fused_frac"] = roof / res["fused_ms"]
            res["fused_tflops"] = flop / res["fused_ms"] / 1e9
            if rank == 0:
                print(json.dumps(res), flush=True)
            # GEMM -> reduce-scatter (row-parallel: each rank holds K / world input columns)
            kl = K // world
            a = torch.randn(M, kl, device="cuda", dtype=torch.bfloat16) * 0.02
            wr = torch.randn(N, kl, device="cuda", dtype=torch.bfloat16) * 0.02
            out = torch.empty(seg, N, device="cuda", dtype=torch.bfloat16)

            def rs_fused():  # noqa: ANN202
                return comm.gemm_rs(a, wr, True, seg)

            def rs_nccl_ours():  # noqa: ANN202
                part = matmul(a, wr, trans_b=True)
                dist.reduce_scatter_tensor(out, part)
                return out

            def rs_nccl_cublas():  # noqa: ANN202
                part = a @ wr.t()
                dist.reduce_scatter_tensor(out, part)
                return out

            flop = 2.0 * M * kl * N
            moved = (world - 1) * seg * N * 2  # partial rows pushed out per GPU
            roof = max(flop / (peak * 1e12), moved / (NVLINK_GBS * 1e9)) * 1e3
            res = {"op": "gemm_reducescatter", "tp": world, "M": M, "K": K, "N": N}
            for name, fn in (("fused", rs_fused), ("nccl_ours", rs_nccl_ours), ("nccl_cublas", rs_nccl_cublas)):
                res[f"{name}_ms"] = timed(fn, args.iters)
            res["roofline_ms"] = roof
            res["fused_frac"] = roof / res["fused_ms"]
            res["fused_tflops"] = flop / res["fused_ms"] / 1e9
            if rank == 0:
                print(json.dumps(res), flush=True)
    torch.cuda.synchronize()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
