#!/usr/bin/env python
"""Kernel microbenchmarks: the framework's sm_100a kernels against the PyTorch library path
(cuBLAS for GEMMs, torch SDPA -- flash / cuDNN backends -- for attention) on one GPU.

    python benchmarks/kernels.py attn --B 8 --T 4096 --hq 16 --hkv 4          # GQA fwd + bwd
    python benchmarks/kernels.py attn --B 4 --T 2048 --hq 6 --hkv 6 --docs 2  # packed documents
    python benchmarks/kernels.py gemm --M 65536 --N 2304 --K 768              # y = x W^T
    python benchmarks/kernels.py gemm --M 768 --N 2304 --K 65536 --layout wgrad
    python benchmarks/kernels.py gemm --M 768 --N 3072 --K 768 --batch 24     # batched (Polar Express)
    python benchmarks/kernels.py norm --M 65536 --D 768                       # QK-norm+RoPE, add+RMSNorm
    python benchmarks/kernels.py attn ... --once       # one untimed call per kernel (for ncu captures)
    python benchmarks/kernels.py gemm ... --once-lib   # the same for the library path

Timing: CUDA events on the launching stream, after warm-up, a synchronize on both sides, median
of ``--iters`` runs; before each run a 256 MB buffer is rewritten so no run starts with the
previous run's operands in L2. Attention FLOPs count only the unmasked work
(``4 * B * Hq * D * kept_pairs`` forward, 2.5x that backward), so causal / window / document
masks do not inflate the rate.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
from pathlib import Path

import torch
import torch.nn.functional as F  # noqa: N812

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from mint_b200.ops import _ext  # noqa: E402
from mint_b200.ops.gemm import matmul  # noqa: E402

_FLUSH: torch.Tensor | None = None


def flush_l2() -> None:
    global _FLUSH
    if _FLUSH is None:
        _FLUSH = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")
    _FLUSH.fill_(1.0)


REPEAT = 1  # calls per timed sample (--repeat): > 1 hides the host-side launch cost of one call


def time_fn(fn, iters: int, warmup: int = 3) -> float:  # noqa: ANN001
    """Median milliseconds per call of ``fn()`` over ``iters`` samples of REPEAT back-to-back calls,
    L2 flushed before each sample."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        flush_l2()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(REPEAT):
            fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e) / REPEAT)
    return statistics.median(times)


def kept_pairs(T: int, causal: bool, window: int, docs: int) -> int:
    """Number of (query, key) pairs the mask keeps, per batch row and head."""
    seg = T // docs
    total = 0
    for d in range(docs):
        n = seg if d < docs - 1 else T - seg * (docs - 1)
        for i in range(n):
            lo = max(0, i - window) if window >= 0 else 0
            hi = i if causal else n - 1
            total += hi - lo + 1
    return total


def run_attn(a: argparse.Namespace) -> dict:
    C = _ext.require()
    torch.manual_seed(0)
    B, T, Hq, Hkv, D = a.B, a.T, a.hq, a.hkv, 128
    q = torch.randn(B, T, Hq, D, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(B, T, Hkv, D, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(B, T, Hkv, D, device="cuda", dtype=torch.bfloat16)
    do = torch.randn_like(q)
    doc = bounds = None
    if a.docs > 1:
        doc = (torch.arange(T, device="cuda") // (T // a.docs)).clamp_max(a.docs - 1).int().expand(B, -1).contiguous()
        bounds = C.doc_bounds(doc) if hasattr(C, "doc_bounds") else None
    scale = 1.0 / math.sqrt(D)
    causal = not a.no_causal
    extra = (bounds,) if bounds is not None else ()
    o, lse = C.flash_attn_fwd(q, k, v, doc, causal, a.window, scale, *extra)
    if os.environ.get("MINT_FA_TRACE"):
        # per-phase clock64 deltas of the longest query tile (diagnostic build path), median over tiles
        for _ in range(3):
            C.flash_attn_fwd(q, k, v, doc, causal, a.window, scale, *extra)
        torch.cuda.synchronize()
        tr = C.flash_attn_fwd_trace().view(-1).tolist()
        steps, tiles = 10, 64
        n = min(tiles, (T + 127) // 128)
        names = ["s_wait", "tmem_ld", "max", "mx_xchg", "rescale", "exp", "pv_wait", "p_store", "fence_arrive"]
        out = {}
        for half in range(2):
            base = half * tiles * steps
            rows = [tr[base + t * steps: base + (t + 1) * steps] for t in range(n)]
            for i, nm in enumerate(names):
                out[f"h{half}_{nm}"] = statistics.median(r[i + 1] - r[i] for r in rows)
            out[f"h{half}_tile"] = statistics.median(rows[t + 1][0] - rows[t][0] for t in range(n - 1))
        mb = 2 * tiles * steps
        mrows = [tr[mb + t * 4: mb + t * 4 + 4] for t in range(n)]
        out["mma_issue_s"] = statistics.median(r[1] - r[0] for r in mrows)
        out["mma_wait_p"] = statistics.median(r[2] - r[1] for r in mrows)
        out["mma_issue_pv"] = statistics.median(r[3] - r[2] for r in mrows)
        print(json.dumps({"fa_fwd_trace_cycles": out, "tiles": n}), flush=True)
        for _ in range(3):
            C.flash_attn_bwd(do, q, k, v, o, lse, doc, causal, a.window, scale, *extra)
        torch.cuda.synchronize()
        tr = C.flash_attn_bwd_trace().view(-1).tolist()
        steps = 12
        nb = min(tiles, (T + 127) // 128) * (Hq // Hkv)
        bnames = ["stage_lse", "s_wait", "s_load", "mask_exp", "p_store_arrive", "dp_wait", "dp_load_ds",
                  "dv_wait", "ds_store_arrive", "dq_wait", "dq_drain"]
        rows = [tr[t * steps: (t + 1) * steps] for t in range(nb)]
        outb = {nm: statistics.median(r[i + 1] - r[i] for r in rows) for i, nm in enumerate(bnames)}
        outb["tile"] = statistics.median(rows[t + 1][0] - rows[t][0] for t in range(nb - 1))
        mb = tiles * steps
        mrows = [tr[mb + t * 4: mb + t * 4 + 4] for t in range(nb - 1)]
        outb["mma_wait_p"] = statistics.median(r[1] - r[0] for r in mrows)
        outb["mma_dv_s_wait_ds"] = statistics.median(r[2] - r[1] for r in mrows)
        outb["mma_dkdq_wait_dqfree"] = statistics.median(r[3] - r[2] for r in mrows)
        print(json.dumps({"fa_bwd_trace_cycles": outb, "tiles": nb}), flush=True)
    if a.once:
        C.flash_attn_bwd(do, q, k, v, o, lse, doc, causal, a.window, scale, *extra)
        torch.cuda.synchronize()
        return {"once": True}
    if a.once_lib:  # the library path once (torch SDPA forward + backward), for profiler captures
        qt, kt, vt = (t.transpose(1, 2).detach().requires_grad_() for t in (q, k, v))
        ot = F.scaled_dot_product_attention(qt, kt, vt, is_causal=causal, enable_gqa=Hq != Hkv)
        torch.autograd.grad(ot, (qt, kt, vt), do.transpose(1, 2))
        torch.cuda.synchronize()
        return {"once_lib": True}
    pairs = kept_pairs(T, causal, a.window, a.docs)
    fwd_flop = 4.0 * B * Hq * D * pairs
    res = {"B": B, "T": T, "Hq": Hq, "Hkv": Hkv, "causal": causal, "window": a.window, "docs": a.docs}
    t_fwd = time_fn(lambda: C.flash_attn_fwd(q, k, v, doc, causal, a.window, scale, *extra), a.iters)
    t_bwd = time_fn(lambda: C.flash_attn_bwd(do, q, k, v, o, lse, doc, causal, a.window, scale, *extra), a.iters)
    res.update(ours_fwd_ms=t_fwd, ours_bwd_ms=t_bwd, ours_fwd_tflops=fwd_flop / t_fwd / 1e9,
               ours_bwd_tflops=2.5 * fwd_flop / t_bwd / 1e9)
    if a.window < 0 and a.docs == 1:
        # library reference: torch SDPA (flash / cuDNN backends pick themselves), GQA native
        qt, kt, vt = (t.transpose(1, 2).detach().requires_grad_() for t in (q, k, v))
        gqa = Hq != Hkv

        def sdpa_fwd():  # noqa: ANN202
            return F.scaled_dot_product_attention(qt, kt, vt, is_causal=causal, enable_gqa=gqa)

        ot = sdpa_fwd()
        dot = do.transpose(1, 2)
        t_sf = time_fn(sdpa_fwd, a.iters)
        t_sb = time_fn(lambda: torch.autograd.grad(ot, (qt, kt, vt), dot, retain_graph=True), a.iters)
        res.update(sdpa_fwd_ms=t_sf, sdpa_bwd_ms=t_sb, sdpa_fwd_tflops=fwd_flop / t_sf / 1e9,
                   sdpa_bwd_tflops=2.5 * fwd_flop / t_sb / 1e9)
        try:  # the flash-attn package: what the reference's attention dispatches to on this box
            from flash_attn import flash_attn_func  # noqa: PLC0415
        except ImportError:
            flash_attn_func = None
        if flash_attn_func is not None:
            qf, kf, vf = (t.detach().requires_grad_() for t in (q, k, v))

            def fa2_fwd():  # noqa: ANN202
                return flash_attn_func(qf, kf, vf, causal=causal)

            of = fa2_fwd()
            t_ff = time_fn(fa2_fwd, a.iters)
            t_fb = time_fn(lambda: torch.autograd.grad(of, (qf, kf, vf), do, retain_graph=True), a.iters)
            res.update(flash_attn_fwd_ms=t_ff, flash_attn_bwd_ms=t_fb)
    return res


def run_gemm(a: argparse.Namespace) -> dict:
    _ext.require()
    torch.manual_seed(0)
    M, N, K, nb = a.M, a.N, a.K, a.batch
    lead = (nb,) if nb > 1 else ()
    if a.layout == "fwd":  # y[M,N] = x[M,K] @ W[N,K]^T
        x = torch.randn(*lead, M, K, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(*lead, N, K, device="cuda", dtype=torch.bfloat16)

        def ours():  # noqa: ANN202
            return matmul(x, w, trans_b=True, out_dtype=torch.bfloat16)

        def lib():  # noqa: ANN202
            return x @ w.mT
    elif a.layout == "dgrad":  # dx[M,N] = dy[M,K] @ W[K,N]
        x = torch.randn(*lead, M, K, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(*lead, K, N, device="cuda", dtype=torch.bfloat16)

        def ours():  # noqa: ANN202
            return matmul(x, w, out_dtype=torch.bfloat16)

        def lib():  # noqa: ANN202
            return x @ w
    else:  # wgrad: dW[M,N] (fp32, accumulated) += dy[K,M]^T @ x[K,N]
        dy = torch.randn(*lead, K, M, device="cuda", dtype=torch.bfloat16)
        x = torch.randn(*lead, K, N, device="cuda", dtype=torch.bfloat16)
        out = torch.zeros(*lead, M, N, device="cuda", dtype=torch.float32)

        def ours():  # noqa: ANN202
            return matmul(dy, x, trans_a=True, out=out, accumulate=True)

        def lib():  # noqa: ANN202  (cuBLAS bf16 GEMM of the same shape, fp32 accumulation inside)
            return dy.mT @ x
    if a.once or a.once_lib:
        (lib if a.once_lib else ours)()
        torch.cuda.synchronize()
        return {"once": True}
    flop = 2.0 * M * N * K * nb
    t_o = time_fn(ours, a.iters)
    t_l = time_fn(lib, a.iters)
    return {"M": M, "N": N, "K": K, "batch": nb, "layout": a.layout, "ours_ms": t_o, "cublas_ms": t_l,
            "ours_tflops": flop / t_o / 1e9, "cublas_tflops": flop / t_l / 1e9}


def hbm_peak_gbs() -> tuple[float, str]:
    p = Path(__file__).resolve().parent.parent / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except (KeyError, ValueError):
            pass
    return 6650.0, "fallback"


def run_norm(a: argparse.Namespace) -> dict:
    """QK-norm + RoPE and residual-add + RMSNorm, forward and backward, on the d12 shapes."""
    C = _ext.require()
    torch.manual_seed(0)
    M, D, hq, hkv, dh = a.M, a.D, a.hq, a.hkv, 128
    H = hq + 2 * hkv
    T = a.T
    qkv = torch.randn(M // T, T, H * dh, device="cuda", dtype=torch.bfloat16)
    qs, ks = torch.zeros(dh, device="cuda"), torch.zeros(dh, device="cuda")
    pos = torch.arange(T, device="cuda", dtype=torch.float32)[:, None]
    inv = 1.0 / (10000.0 ** (torch.arange(0, dh, 2, device="cuda", dtype=torch.float32) / dh))
    cos, sin = torch.cos(pos * inv).contiguous(), torch.sin(pos * inv).contiguous()
    q, k, v, rq, rk = C.qk_norm_rope_fwd(qkv, hq, hkv, dh, qs, ks, cos, sin, 0, 1e-6, True)
    dq, dk, dv = torch.randn_like(q), torch.randn_like(k), torch.randn_like(v)
    res = torch.randn(M, D, device="cuda", dtype=torch.float32)
    x = torch.randn(M, D, device="cuda", dtype=torch.bfloat16)
    post, pre = torch.zeros(D, device="cuda"), torch.zeros(D, device="cuda")
    h, y, ra, rh = C.add_rmsnorm_fwd(res, x, post, pre, 1e-6, 1)
    dh_, dy = torch.randn_like(h), torch.randn_like(y)
    if a.once:
        C.qk_norm_rope_bwd(dq, dk, dv, qkv, rq, rk, qs, ks, cos, sin, hq, hkv, dh, 0, True)
        C.add_rmsnorm_bwd(dh_, dy, x, h, ra, rh, post, pre)
        torch.cuda.synchronize()
        return {"once": True}
    peak, kind = hbm_peak_gbs()
    e2, e4 = 2, 4
    rows_qk = M * (hq + hkv)
    cases = {
        "qk_norm_rope_fwd": (lambda: C.qk_norm_rope_fwd(qkv, hq, hkv, dh, qs, ks, cos, sin, 0, 1e-6, True),
                             2 * M * H * dh * e2 + rows_qk * e4),
        "qk_norm_rope_bwd": (lambda: C.qk_norm_rope_bwd(dq, dk, dv, qkv, rq, rk, qs, ks, cos, sin, hq, hkv, dh, 0, True),
                             2 * M * H * dh * e2 + rows_qk * dh * e2 + rows_qk * e4),
        "add_rmsnorm_fwd": (lambda: C.add_rmsnorm_fwd(res, x, post, pre, 1e-6, 1),
                            M * D * (e4 + e2) + M * D * (e4 + e2) + 2 * M * e4),
        "add_rmsnorm_bwd": (lambda: C.add_rmsnorm_bwd(dh_, dy, x, h, ra, rh, post, pre),
                            M * D * (e4 + e2 + e2 + e4) + M * D * (e4 + e2) + 2 * M * e4),
    }
    V = a.V
    logits = torch.randn(M, V, device="cuda", dtype=torch.bfloat16)
    tgt = torch.randint(0, V, (M,), device="cuda")
    cmask = torch.ones(M, device="cuda")
    denom = torch.full((1,), float(M), device="cuda")
    # in place: every timed call rewrites the logits with gradients (same traffic, values irrelevant)
    cases["ce_fused_fwd_bwd"] = (lambda: C.ce_fused_fwd_bwd(logits, tgt, cmask, denom, V, 0), 2 * M * V * e2)
    out = {"M": M, "D": D, "hq": hq, "hkv": hkv, "V": V, "peak_gbs": peak, "peak": kind}
    for name, (fn, nbytes) in cases.items():
        t = time_fn(fn, a.iters)
        out[f"{name}_ms"] = t
        out[f"{name}_frac"] = nbytes / (t * 1e-3) / 1e9 / peak
    return out


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    at = sub.add_parser("attn")
    at.add_argument("--B", type=int, default=4)
    at.add_argument("--T", type=int, default=2048)
    at.add_argument("--hq", type=int, default=6)
    at.add_argument("--hkv", type=int, default=6)
    at.add_argument("--window", type=int, default=-1)
    at.add_argument("--docs", type=int, default=1)
    at.add_argument("--no-causal", action="store_true")
    gm = sub.add_parser("gemm")
    gm.add_argument("--M", type=int, default=65536)
    gm.add_argument("--N", type=int, default=2304)
    gm.add_argument("--K", type=int, default=768)
    gm.add_argument("--batch", type=int, default=1)
    gm.add_argument("--layout", choices=["fwd", "dgrad", "wgrad"], default="fwd")
    nm = sub.add_parser("norm")
    nm.add_argument("--M", type=int, default=65536)
    nm.add_argument("--T", type=int, default=2048)
    nm.add_argument("--D", type=int, default=768)
    nm.add_argument("--hq", type=int, default=6)
    nm.add_argument("--hkv", type=int, default=6)
    nm.add_argument("--V", type=int, default=65536)
    for p in (at, gm, nm):
        p.add_argument("--iters", type=int, default=10)
        p.add_argument("--repeat", type=int, default=1,
                       help="back-to-back calls per timed sample (the first reads a flushed L2, the rest a warm one)")
        p.add_argument("--once", action="store_true")
        p.add_argument("--once-lib", action="store_true", help="run the library (cuBLAS / SDPA) path once")
    a = ap.parse_args()
    global REPEAT
    REPEAT = max(1, a.repeat)
    res = {"attn": run_attn, "gemm": run_gemm, "norm": run_norm}[a.cmd](a)
    _ext.check_device_status()
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
