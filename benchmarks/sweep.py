#!/usr/bin/env python
"""Benchmark sweep over the BASELINE.json configurations, one isolated subprocess per cell.

    python benchmarks/sweep.py [--gpus 8] [--only d12,attn] [--impl ours,reference] [--out DIR]

Cells (each skipped when it needs more GPUs than ``--gpus``):
  d12      pretraining tokens/s, tp=2 sp + ZeRO-2 layouts at 1/2/4/8 GPUs (bench.py), ours and the
           reference arm
  2b       ~2B decoder, tp=4 sp + ZeRO-3 dp=2 on 8 GPUs (bench.py --model 2b)
  tpfused  all-gather->GEMM and GEMM->reduce-scatter vs NCCL + cuBLAS at tp = 2/4/8
           (benchmarks/tp_fused.py; M in {8k, 32k, 128k}, K 2048, N in {2048, 8192})
  attn     GQA FlashAttention forward/backward, 16q/4kv heads x 128, seq 1k..16k vs torch SDPA
           (benchmarks/kernels.py attn)
  zero     ZeRO-2 reduce-scatter / all-gather over NVLink peer memory vs NCCL (benchmarks/zero_fused.py)

Every cell runs in its own process group with a time limit (the group is killed on expiry) and is
classified ok / oom / timeout / fail from its exit status and output. Results go to
``<out>/results.json`` (one record per cell: command, status, seconds, parsed JSON lines, log tail)
and ``<out>/report.md`` (a table per cell family).
"""

from __future__ import annotations

import argparse
import json
import os
import signal
import subprocess
import sys
import time
from dataclasses import asdict, dataclass, field
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
PY = sys.executable


@dataclass
class Cell:
    family: str
    name: str
    gpus: int
    cmd: list[str]
    timeout: float
    env: dict = field(default_factory=dict)


def torchrun(n: int, port: int, script: str, *args: str) -> list[str]:
    if n == 1:
        return [PY, script, *args]
    return ["timeout", "-k", "60", "1500", PY, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
            "--master-addr=127.0.0.1", f"--master-port={port}", script, *args]


def build_cells(max_gpus: int, impls: list[str]) -> list[Cell]:
    cells: list[Cell] = []
    port = 29600
    for n in (1, 2, 4, 8):
        for impl in impls:
            port += 1
            cells.append(Cell("d12", f"d12 {impl} {n}gpu", n,
                              torchrun(n, port, "bench.py", "--gpus", str(n), "--steps", "10", "--warmup", "3",
                                       "--impl", impl, "--no-same-optimizer"), 900))
    for impl in impls:
        port += 1
        cells.append(Cell("2b", f"2b {impl} 8gpu", 8,
                          torchrun(8, port, "bench.py", "--gpus", "8", "--model", "2b", "--steps", "5", "--warmup", "3",
                                   "--impl", impl, "--no-same-optimizer"), 1500))
    for n in (2, 4, 8):
        port += 1
        cells.append(Cell("tpfused", f"tp_fused tp={n}", n,
                          torchrun(n, port, "benchmarks/tp_fused.py", "--M", "8192", "32768", "131072", "--N", "2048",
                                   "8192", "--K", "2048"), 900))
    for t in (1024, 2048, 4096, 8192, 16384):
        b = max(1, 32768 // t)
        cells.append(Cell("attn", f"attn gqa T={t}", 1,
                          [PY, "benchmarks/kernels.py", "attn", "--B", str(b), "--T", str(t), "--hq", "16", "--hkv", "4",
                           "--iters", "10"], 600))
    for n in (2, 4, 8):
        port += 1
        cells.append(Cell("zero", f"zero_fused dp={n}", n, torchrun(n, port, "benchmarks/zero_fused.py"), 600))
    for n in (1, 8):
        for impl in impls:
            port += 1
            cells.append(Cell("dpo", f"dpo {impl} {n}gpu", n,
                              torchrun(n, port, "benchmarks/dpo_step.py", "--gpus", str(n), "--impl", impl,
                                       "--ddp-level", "3" if n > 1 else "0"), 900))
    return [c for c in cells if c.gpus <= max_gpus]


def classify(rc: int | None, text: str, timed_out: bool) -> str:
    if timed_out:
        return "timeout"
    if rc == 0:
        return "ok"
    low = text.lower()
    if "out of memory" in low or "cuda error: out of memory" in low:
        return "oom"
    return "fail"


def json_lines(text: str) -> list[dict]:
    out = []
    for line in text.splitlines():
        line = line.strip()
        if line.startswith("{") and line.endswith("}"):
            try:
                out.append(json.loads(line))
            except json.JSONDecodeError:
                continue
    return out


def run_cell(cell: Cell) -> dict:
    t0 = time.monotonic()
    env = {**os.environ, **cell.env, "NCCL_NVLS_ENABLE": os.environ.get("NCCL_NVLS_ENABLE", "0")}
    proc = subprocess.Popen(cell.cmd, cwd=ROOT, env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True,
                            start_new_session=True)
    timed_out = False
    try:
        text, _ = proc.communicate(timeout=cell.timeout)
    except subprocess.TimeoutExpired:
        timed_out = True
        try:
            os.killpg(proc.pid, signal.SIGTERM)  # the cell's own process group (new session)
            text, _ = proc.communicate(timeout=60)
        except (subprocess.TimeoutExpired, ProcessLookupError):
            os.killpg(proc.pid, signal.SIGKILL)
            text, _ = proc.communicate()
    rec = asdict(cell)
    rec.update(status=classify(proc.returncode, text or "", timed_out), returncode=proc.returncode,
               seconds=round(time.monotonic() - t0, 1), results=json_lines(text or ""),
               log_tail=(text or "")[-3000:])
    return rec


def _fmt(v: object) -> str:
    if isinstance(v, float):
        return f"{v:,.1f}" if abs(v) >= 100 else f"{v:.4g}"
    return str(v)


def report(records: list[dict]) -> str:
    lines = ["# Benchmark sweep", ""]
    for fam in dict.fromkeys(r["family"] for r in records):
        lines += [f"## {fam}", "", "| cell | status | s | result |", "|---|---|---|---|"]
        for r in records:
            if r["family"] != fam:
                continue
            if r["results"]:
                res = r["results"][-1]
                keys = [k for k in ("value", "unit", "ms_per_step", "fused_ms", "nccl_ms", "fwd_ms", "bwd_ms",
                                    "sdpa_fwd_ms", "sdpa_bwd_ms", "frac_of_roofline") if k in res]
                summary = ", ".join(f"{k}={_fmt(res[k])}" for k in keys) or json.dumps(res)[:200]
            else:
                summary = ""
            lines.append(f"| {r['name']} | {r['status']} | {r['seconds']} | {summary} |")
        lines.append("")
    return "\n".join(lines)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=8, help="GPUs available to the sweep")
    ap.add_argument("--only", default="", help="comma-separated cell families (default: all)")
    ap.add_argument("--impl", default="ours,reference")
    ap.add_argument("--out", default="")
    ap.add_argument("--list", action="store_true", help="print the cells and exit")
    args = ap.parse_args()
    cells = build_cells(args.gpus, [i for i in args.impl.split(",") if i])
    if args.only:
        keep = set(args.only.split(","))
        cells = [c for c in cells if c.family in keep]
    if args.list:
        for c in cells:
            print(f"{c.family:8s} {c.name:24s} gpus={c.gpus} {' '.join(c.cmd)}")
        return
    out = Path(args.out or ROOT / "benchmarks" / "runs" / time.strftime("%Y%m%d_%H%M%S"))
    out.mkdir(parents=True, exist_ok=True)
    records = []
    for cell in cells:
        print(f"[sweep] {cell.name} ...", flush=True)
        rec = run_cell(cell)
        records.append(rec)
        print(f"[sweep] {cell.name}: {rec['status']} in {rec['seconds']} s", flush=True)
        (out / "results.json").write_text(json.dumps(records, indent=1))
        (out / "report.md").write_text(report(records))
    print(report(records))


if __name__ == "__main__":
    main()
