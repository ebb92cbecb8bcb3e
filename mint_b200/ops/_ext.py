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


_FALLBACKS: dict[tuple[str, str], int] = {}


def fallback(op: str, reason: str) -> None:
    """Record that a call of ``op`` on CUDA tensors ran its PyTorch implementation instead of a
    kernel (an operand the kernel cannot take). The first occurrence of each (op, reason) warns;
    with ``MINT_STRICT_KERNELS=1`` every occurrence raises, so a hot path cannot silently move onto
    PyTorch / cuBLAS. ``fallback_counts()`` reports them (``bench.py`` prints the total)."""
    key = (op, reason)
    _FALLBACKS[key] = _FALLBACKS.get(key, 0) + 1
    if os.environ.get("MINT_STRICT_KERNELS", "0") == "1":
        raise RuntimeError(f"mint_b200: {op} has no kernel path for this call ({reason}); MINT_STRICT_KERNELS=1")
    if _FALLBACKS[key] == 1:
        import warnings  # noqa: PLC0415

        warnings.warn(f"mint_b200: {op} ran its PyTorch fallback on CUDA ({reason})", RuntimeWarning, stacklevel=3)


def fallback_counts() -> dict[str, int]:
    return {f"{op}: {reason}": n for (op, reason), n in _FALLBACKS.items()}


def reset_fallbacks() -> None:
    _FALLBACKS.clear()


def use_cuda_kernels(t) -> bool:  # noqa: ANN001
    """True when ``t`` lives on a GPU: then the extension is mandatory."""
    if not t.is_cuda:
        return False
    if not kernels_enabled():
        return False
    require()
    return True


STATUS_BITS = {
    1 << 0: "timed-out wait in a GEMM producer",
    1 << 1: "timed-out wait in a GEMM MMA issuer",
    1 << 2: "timed-out wait in a GEMM epilogue",
    1 << 3: "bad kernel argument",
    1 << 4: "timed-out wait for a peer GPU (fused collective)",
    1 << 5: "timed-out wait in attention",
}


class DeviceStatusError(RuntimeError):
    """A kernel recorded an error in the device status word: its outputs (and every parameter
    update that would have used them) are not to be trusted."""


def _describe(code: int) -> str:
    names = [txt for bit, txt in STATUS_BITS.items() if code & bit]
    return f"0x{code:x} ({'; '.join(names) or 'unknown bits'})"


def check_device_status() -> None:
    """Raise if any kernel recorded an error (timed-out wait, bad shape) in the device status word.

    Synchronizes with the device (a 4-byte device-to-host copy)."""
    mod = _try_load()
    if mod is None:
        return
    code = int(mod.read_status(False))
    if code != 0:
        mod.read_status(True)
        raise DeviceStatusError(f"mint_b200 kernel reported device status {_describe(code)}")


def set_wait_limit(seconds: float) -> None:
    """Bound every spin-wait of this device's kernels (default 4 s). On expiry a kernel records a
    status bit, drains its in-flight work and returns; the parameter-update kernels then skip
    their updates until the host has read the word."""
    require().set_wait_limit_ns(max(1, int(seconds * 1e9)))


def wait_limit() -> float:
    return require().wait_limit_ns() / 1e9


class StatusWatch:
    """Per-step check of the device status word without stalling the host.

    ``poll()`` raises :class:`DeviceStatusError` if the snapshot taken by the previous ``poll()``
    (an asynchronous copy into pinned memory, enqueued after that step's work) shows an error,
    then enqueues a new snapshot. A failed step is therefore reported one step later at most; the
    update kernels (AdamW, NorMuon) already skipped their updates on the device, so no parameter
    was changed with data from a timed-out collective. ``flush()`` checks synchronously."""

    def __init__(self) -> None:
        import torch  # noqa: PLC0415

        self._torch = torch
        self._host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self._event = None

    def poll(self) -> None:
        torch = self._torch
        if self._event is not None:
            self._event.synchronize()
            code = int(self._host[0])
            if code != 0:
                self._event = None
                check_device_status()  # clears the word and raises with the decoded bits
                raise DeviceStatusError(f"mint_b200 kernel reported device status {_describe(code)}")
        self._host.copy_(require().status_tensor(), non_blocking=True)
        self._event = torch.cuda.Event()
        self._event.record()

    def flush(self) -> None:
        self._event = None
        check_device_status()


_WATCHES: dict[int, StatusWatch] = {}


def status_watch(device_index: int) -> StatusWatch:
    w = _WATCHES.get(device_index)
    if w is None:
        w = StatusWatch()
        _WATCHES[device_index] = w
    return w


PIECE_ELEMS = 1 << 16  # elements per row of the multi-tensor kernels' work tables


def piece_table(segments: list[tuple[int, ...]], elem_bytes: tuple[int, ...]) -> list[tuple[int, ...]]:
    """Split ``(ptr_0, ..., ptr_k, numel)`` segments into rows of at most PIECE_ELEMS elements, each
    pointer advanced by its own element size, so one block per row gives balanced work."""
    rows = []
    for seg in segments:
        *ptrs, n = seg
        for off in range(0, n, PIECE_ELEMS):
            rows.append((*(p + off * eb for p, eb in zip(ptrs, elem_bytes)), min(PIECE_ELEMS, n - off)))
    return rows
