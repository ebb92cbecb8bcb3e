"""Step-windowed torch.profiler capture and NVTX ranges.

The ``[train.profiler]`` TOML table is the reference's (mint/utils/profiler.py:15-34): skip
``schedule_wait`` steps, warm up for ``schedule_warmup``, record ``schedule_active``, repeat
``schedule_repeat`` times (0 = until training ends). The mechanism is this framework's own: the
trainer calls ``step()`` once per optimizer step and :class:`StepProfiler` opens a fresh
``torch.profiler.profile`` for each recording window itself (no torch schedule object, no
TensorBoard plugin). When a window closes it writes, per rank,

* ``<output_dir>/<run_name>/<trace_prefix>_rank<R>_w<N>.json`` -- a Chrome / Perfetto trace;
* ``..._w<N>.kernels.txt`` -- device time per kernel name summed over the window, largest first,
  which is usually the first thing to read for a GPU step.

``nvtx_range`` marks host phases for device timelines.
"""

from __future__ import annotations

import contextlib
import os
from collections import defaultdict
from collections.abc import Iterator
from dataclasses import dataclass, field
from datetime import datetime
from pathlib import Path

import torch
from torch import profiler as tprof

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


def _activities(names: list[str]) -> list[tprof.ProfilerActivity]:
    table = {"cpu": tprof.ProfilerActivity.CPU, "cuda": tprof.ProfilerActivity.CUDA}
    acts = []
    for name in names:
        act = table.get(name.strip().lower())
        if act is tprof.ProfilerActivity.CUDA and not torch.cuda.is_available():
            continue
        if act is not None and act not in acts:
            acts.append(act)
    return acts


class StepProfiler:
    """Records windows of ``schedule_active`` steps; see the module docstring for the cadence."""

    def __init__(self, config: ProfilerConfig | None = None) -> None:
        self.config = config or ProfilerConfig()
        self._step = 0
        self._windows = 0
        self._prof: tprof.profile | None = None
        self._recorded = False
        run = self.config.run_name or datetime.now().strftime("%Y%m%d_%H%M%S")
        self.out_dir = Path(self.config.output_dir) / run
        self.rank = int(os.getenv("RANK", "0"))

    # ---------------------------------------------------------------- cadence
    def _phase(self, step: int) -> str:
        """'record' when ``step`` falls in a recording window, 'warmup' right before one, else 'idle'."""
        c = self.config
        cycle = c.schedule_wait + c.schedule_warmup + c.schedule_active
        if cycle <= 0 or c.schedule_active <= 0:
            return "idle"
        k, pos = divmod(step, cycle)
        if c.schedule_repeat and k >= c.schedule_repeat:
            return "idle"
        if pos < c.schedule_wait:
            return "idle"
        return "warmup" if pos < c.schedule_wait + c.schedule_warmup else "record"

    # ---------------------------------------------------------------- control
    def start(self) -> None:
        if self.config.enabled:
            self.out_dir.mkdir(parents=True, exist_ok=True)
            logger.info(f"[profiler] recording windows of {self.config.schedule_active} steps into {self.out_dir}")
            self._transition(self._phase(0))

    def step(self) -> None:
        if not self.config.enabled:
            return
        self._step += 1
        self._transition(self._phase(self._step))

    def stop(self) -> None:
        if self._prof is not None:
            self._close()

    def __enter__(self) -> StepProfiler:
        self.start()
        return self

    def __exit__(self, *_: object) -> None:
        self.stop()

    def _transition(self, phase: str) -> None:
        # warm-up steps run under the profiler too (its own start-up cost stays out of the window),
        # so a profile opens at the first warm-up or record step and closes after the last record step
        want_open = phase in ("warmup", "record")
        if self._prof is not None and (not want_open or (phase == "warmup" and self._recorded)):
            self._close()
        if want_open and self._prof is None:
            self._open()
        if phase == "record":
            self._recorded = True

    def _open(self) -> None:
        c = self.config
        self._recorded = False
        self._prof = tprof.profile(activities=_activities(c.activities), record_shapes=c.record_shapes,
                                   profile_memory=c.profile_memory, with_stack=c.with_stack, with_flops=c.with_flops)
        self._prof.__enter__()

    def _close(self) -> None:
        prof, self._prof = self._prof, None
        prof.__exit__(None, None, None)
        if not self._recorded:
            return
        stem = self.out_dir / f"{self.config.trace_prefix}_rank{self.rank}_w{self._windows}"
        self._windows += 1
        prof.export_chrome_trace(str(stem) + ".json")
        (Path(str(stem) + ".kernels.txt")).write_text(kernel_summary(prof))
        logger.info(f"[profiler] wrote {stem}.json")


def kernel_summary(prof: tprof.profile, limit: int = 40) -> str:
    """Device time per kernel name over a finished profile, largest first."""
    per: dict[str, list[float]] = defaultdict(lambda: [0.0, 0])
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA:
            rec = per[ev.name]
            rec[0] += ev.device_time_total / 1e3
            rec[1] += 1
    total = sum(v[0] for v in per.values()) or 1e-9
    lines = [f"device time {total:.3f} ms over {sum(int(v[1]) for v in per.values())} kernels"]
    for name, (ms, n) in sorted(per.items(), key=lambda kv: -kv[1][0])[:limit]:
        lines.append(f"{ms:10.3f} ms {int(n):6d}x {100 * ms / total:5.1f} %  {name[:160]}")
    return "\n".join(lines) + "\n"


# the trainers' original name for the profiler object
TorchProfiler = StepProfiler


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
