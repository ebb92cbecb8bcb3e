#!/usr/bin/env python
"""ZeRO data-parallel collectives over NVLink peer memory vs NCCL, one rank per GPU:

    torchrun --nproc-per-node N --master-addr 127.0.0.1 benchmarks/zero_fused.py [--mb 64 256]

For each fp32 bucket size (MiB per rank, full bucket):
  reduce-scatter: fused kernel (sum over peers + 1/dp scale + squared norm, then a group barrier)
                  vs NCCL reduce_scatter_tensor + scale + norm
  all-gather:     push kernel + barrier  vs  NCCL all_gather_into_tensor
Times are CUDA-event times, median of --iters, max over ranks. Roofline: the bytes each GPU must
receive over NVLink ((dp - 1) / dp of the bucket) at the measured 770 GB/s per direction;
`frac` = roofline / achieved. Rank 0 prints one JSON line per case.
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
    ap.add_argument("--mb", type=int, nargs="+", default=[16, 64, 256])
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120))
    rank, world = dist.get_rank(), dist.get_world_size()
    from mint_b200.ops import _ext
    from mint_b200.parallel.fused import _Symm

    C = _ext.require()
    ctrl = _Symm(256, dist.group.WORLD, dev)
    flags = ctrl.view((world,), torch.int32)
    seq = [0]

    def nxt() -> int:
        seq[0] += 1
        return seq[0]

    for mb in args.mb:
        size = (mb * 1024 * 1024 // 4) // (4 * world) * (4 * world)
        shard = size // world
        buf = _Symm(size * 4, dist.group.WORLD, dev)
        bv = buf.view((size,), torch.float32)
        bv.normal_()
        plain = bv.clone()
        out = torch.empty(shard, device=dev)
        sumsq = torch.zeros(1, device=dev)

        def rs_fused():  # noqa: ANN202
            C.zero_reduce_scatter(buf.ptrs, out, 1.0 / world, sumsq, ctrl.ptrs, flags, rank, world, nxt())
            C.zero_barrier(ctrl.ptrs, flags, rank, world, nxt())

        def rs_nccl():  # noqa: ANN202
            dist.reduce_scatter_tensor(out, plain)
            out.mul_(1.0 / world)
            sumsq.add_(out.square().sum())

        def ag_fused():  # noqa: ANN202
            C.zero_all_gather(out, buf.ptrs, rank, world)
            C.zero_barrier(ctrl.ptrs, flags, rank, world, nxt())

        def ag_nccl():  # noqa: ANN202
            dist.all_gather_into_tensor(plain, out)

        moved = (world - 1) * shard * 4
        roof = moved / (NVLINK_GBS * 1e9) * 1e3
        for op, fused, nccl in (("reduce_scatter", rs_fused, rs_nccl), ("all_gather", ag_fused, ag_nccl)):
            res = {"op": op, "dp": world, "bucket_mib": mb, "fused_ms": timed(fused, args.iters),
                   "nccl_ms": timed(nccl, args.iters), "roofline_ms": roof}
            res["fused_frac"] = roof / res["fused_ms"]
            res["nccl_frac"] = roof / res["nccl_ms"]
            if rank == 0:
                print(json.dumps(res), flush=True)
        del buf
    torch.cuda.synchronize()
    _ext.check_device_status()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
