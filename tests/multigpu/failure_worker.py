"""Worker for test_failure_detection.py, launched by torchrun with one rank per GPU.

1. Both ranks run one fused all-gather -> GEMM call: no status bit is set.
2. Rank 1 skips the next fused call. Rank 0's kernel waits for rank 1 to enter the call, gives up
   after the wait limit (set to 0.2 s here), records the peer-timeout bit, drains and returns; the
   host then raises DeviceStatusError. Nothing waits without a bound, no rank exits while a kernel
   or collective of it is in flight, and the communicator is not used after the skipped call.
3. A ZeRO-2 style update after the failure: AdamW on the GPU leaves the parameters unchanged
   while the status word is set (the device-side gate of the update kernels).
Prints one line per check and exits non-zero on a mismatch.
"""

from __future__ import annotations

import os
import sys
import time
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[2]))


def main() -> None:
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60))
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)
    from mint_b200.ops import _ext
    from mint_b200.optim.functional import adamw_update
    from mint_b200.parallel import fused

    _ext.check_device_status()
    _ext.set_wait_limit(0.2)
    comm = fused.TPComm(dist.group.WORLD, dev)
    B, seg, K, N = 1, 256, 256, 512
    T = seg * world
    torch.manual_seed(rank)
    x = torch.randn(B, seg, K, device=dev, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=dev, dtype=torch.bfloat16) * 0.05
    failures = 0

    # one gathered buffer for both calls, allocated (collectively) while both ranks take part;
    # its content does not change between the calls, so reusing it needs no reuse distance
    _slot, buf = comm.acquire(B * T * K * 2)
    buf.view((B, world, seg, K), torch.bfloat16)[:, rank].copy_(x)

    def fused_call() -> torch.Tensor:
        return comm.gemm_ag(buf, B * T, K, w, True, seg)

    fused_call()
    torch.cuda.synchronize()
    try:
        _ext.check_device_status()
        print(f"[rank {rank}] matched call: status clean OK", flush=True)
    except _ext.DeviceStatusError as exc:
        failures += 1
        print(f"[rank {rank}] matched call: unexpected status {exc} FAIL", flush=True)
    dist.barrier()

    if rank == 0:
        t0 = time.perf_counter()
        fused_call()  # rank 1 never enters this call
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        try:
            _ext.check_device_status()
            failures += 1
            print(f"[rank 0] skipped peer: no status bit after {dt:.2f} s FAIL", flush=True)
        except _ext.DeviceStatusError as exc:
            ok = "peer" in str(exc) and dt < 5.0
            failures += not ok
            print(f"[rank 0] skipped peer: raised after {dt:.2f} s ({exc}) {'OK' if ok else 'FAIL'}", flush=True)
        # the update kernels leave parameters alone while the status word is set
        C = _ext.require()
        C.status_tensor().fill_(1 << 4)
        p, g = torch.randn(4096, device=dev), torch.randn(4096, device=dev)
        m, v = torch.zeros_like(p), torch.zeros_like(p)
        before = p.clone()
        adamw_update(p, g, m, v, 1, 1e-2, 0.9, 0.95, 1e-8, 0.0)
        torch.cuda.synchronize()
        ok = torch.equal(p, before)
        failures += not ok
        print(f"[rank 0] update gated by the status word: {'OK' if ok else 'FAIL'}", flush=True)
        C.read_status(True)
    # both ranks meet on the host (NCCL barrier) only after rank 0's kernel has returned
    dist.barrier()
    flag = torch.tensor([float(failures)], device=dev)
    dist.all_reduce(flag)
    dist.destroy_process_group()
    sys.exit(1 if flag.item() > 0 else 0)


if __name__ == "__main__":
    main()
