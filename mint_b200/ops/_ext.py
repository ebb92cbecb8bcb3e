"""Loader for the in-tree sm_100a extension ``mint_b200._C``.

CUDA tensors always run through the extension's kernels; when the extension is missing
on a machine with a GPU, ``require()`` raises instead of silently using PyTorch ops.
CPU tensors (unit tests, gloo ranks) use the plain PyTorch reference implementation
that lives next to each op.
"""

from __future__ import annotations

import importlib
import os
from types import ModuleType

_C: ModuleType | None = None
_LOAD_ERROR: BaseException | None = None


def _try_load() -> ModuleType | None:
    global _C, _LOAD_ERROR
    if _C is not None or _LOAD_ERROR is not None:
        return _C
    try:
        import torch  # noqa: F401  (the extension links against libtorch)

        _C = importlib.import_module("mint_b200._C")
    except ImportError as exc:  # not built
        _LOAD_ERROR = exc
    return _C


def available() -> bool:
    return _try_load() is not None


def require() -> ModuleType:
    mod = _try_load()
    if mod is None:
        raise RuntimeError(
            "mint_b200._C (sm_100a kernels) is not built or failed to load: "
            f"{_LOAD_ERROR!r}. Build it with `python -m mint_b200.csrc.build`."
        )
    return mod


def kernels_enabled() -> bool:
    """Kernels are on unless MINT_DISABLE_KERNELS=1 (used only by A/B numerics tests)."""
    return os.environ.get("MINT_DISABLE_KERNELS", "0") != "1"


def use_cuda_kernels(t) -> bool:  # noqa: ANN001
    """True when ``t`` lives on a GPU: then the extension is mandatory."""
    if not t.is_cuda:
        return False
    if not kernels_enabled():
        return False
    require()
    return True


def check_device_status() -> None:
    """Raise if any kernel recorded an error (timed-out wait, bad shape) in the device status word."""
    mod = _try_load()
    if mod is None:
        return
    code = int(mod.read_status(False))
    if code != 0:
        mod.read_status(True)
        raise RuntimeError(f"mint_b200 kernel reported device status 0x{code:x} (see kernel error codes)")
