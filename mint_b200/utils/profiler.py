"""torch.profiler wrapper with a wait/warmup/active/repeat schedule (mint/utils/profiler.py:15-95)
plus NVTX ranges (``nvtx_range``) that show up in ncu/nsys timelines."""

from __future__ import annotations

import contextlib
import os
from collections.abc import Iterator
from dataclasses import dataclass, field
from datetime import datetime
from pathlib import Path

import torch
import torch.profiler as tp

from mint_b200.config.base import Config
from mint_b200.utils.logger import logger


@dataclass
class ProfilerConfig(Config):
    enabled: bool = False
    output_dir: str = "./profiles_torch"
    schedule_wait: int = 1
    schedule_warmup: int = 1
    schedule_active: int = 3
    schedule_repeat: int = 0
    record_shapes: bool = True
    profile_memory: bool = True
    with_stack: bool = False
    with_flops: bool = True
    activities: list[str] = field(default_factory=lambda: ["cpu", "cuda"])
    trace_prefix: str = "trace"
    run_name: str = ""


class TorchProfiler:
    def __init__(self, config: ProfilerConfig | None = None) -> None:
        self.config = config or ProfilerConfig()
        self._profiler: tp.profile | None = None

    def start(self) -> None:
        if not self.config.enabled:
            return
        self._profiler = self._build()
        self._profiler.start()
        logger.info(f"[profiler] started -> {self.config.output_dir}")

    def stop(self) -> None:
        if self._profiler is None:
            return
        self._profiler.stop()
        self._profiler = None

    def step(self) -> None:
        if self._profiler is not None:
            self._profiler.step()

    def __enter__(self) -> TorchProfiler:
        self.start()
        return self

    def __exit__(self, *_: object) -> None:
        self.stop()

    def _build(self) -> tp.profile:
        acts = []
        for name in self.config.activities:
            a = name.strip().lower()
            if a == "cpu":
                acts.append(tp.ProfilerActivity.CPU)
            elif a == "cuda" and torch.cuda.is_available():
                acts.append(tp.ProfilerActivity.CUDA)
        run = self.config.run_name or datetime.now().strftime("%Y%m%d_%H%M%S")
        out = Path(self.config.output_dir) / run
        out.mkdir(parents=True, exist_ok=True)
        return tp.profile(
            activities=acts,
            schedule=tp.schedule(wait=self.config.schedule_wait, warmup=self.config.schedule_warmup,
                                 active=self.config.schedule_active, repeat=self.config.schedule_repeat),
            on_trace_ready=tp.tensorboard_trace_handler(
                str(out), worker_name=f"{self.config.trace_prefix}_rank{os.getenv('RANK', '0')}"),
            record_shapes=self.config.record_shapes,
            profile_memory=self.config.profile_memory,
            with_stack=self.config.with_stack,
            with_flops=self.config.with_flops,
        )


@contextlib.contextmanager
def nvtx_range(name: str) -> Iterator[None]:
    """NVTX range on CUDA builds (no-op elsewhere)."""
    if torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield
