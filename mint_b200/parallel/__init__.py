"""Parallel runtime: dp x tp mesh, tensor/sequence-parallel collectives, ZeRO gradient engine.

Submodules are imported lazily so that ``mint_b200.nn`` can depend on ``parallel.tp``.
"""

from __future__ import annotations

import importlib
from typing import Any

_LAZY = {
    "setup_parallel": "mint_b200.parallel.api",
    "ParallelContext": "mint_b200.parallel.context",
    "dp_tp_ranks": "mint_b200.parallel.context",
    "apply_tp": "mint_b200.parallel.tensor_parallel",
    "GradEngine": "mint_b200.parallel.zero",
    "apply_ddp": "mint_b200.parallel.zero",
    "get_engine": "mint_b200.parallel.zero",
}


def __getattr__(name: str) -> Any:  # noqa: ANN401
    if name in _LAZY:
        return getattr(importlib.import_module(_LAZY[name]), name)
    raise AttributeError(name)


__all__ = list(_LAZY)
