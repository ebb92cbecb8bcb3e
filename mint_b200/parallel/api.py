"""``setup_parallel`` = tensor-parallel plan + gradient engine (mint/utils/parallel.py:526-533)."""

from __future__ import annotations

from torch import nn

from mint_b200.parallel.context import ParallelContext
from mint_b200.parallel.tensor_parallel import apply_tp
from mint_b200.parallel.zero import apply_ddp


def setup_parallel(
    model: nn.Module,
    parallel: ParallelContext,
    tp_plan: dict[str, str] | None = None,
    bucket_cap_mb: float = 256.0,
) -> nn.Module:
    model = apply_tp(model, parallel, tp_plan=tp_plan)
    return apply_ddp(model, parallel, bucket_cap_mb=bucket_cap_mb)
