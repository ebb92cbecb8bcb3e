"""Training-recipe schedules: LR multiplier, Muon momentum and Muon weight decay per step.

The config fields (the ``[train.sched]`` TOML table) and the curves are the reference recipe's
(mint/trainer/scheduler.py:9-87): a linear LR warmup, a flat phase, a linear warmdown to
``final_lr_frac``; Muon momentum ramping from ``muon_momentum_start`` to ``muon_momentum_peak``
and easing to ``muon_momentum_final`` during the warmdown; a cosine weight-decay decay to zero.

Here each curve is data: an ordered list of segments, each a half-open step range with a shape
(constant, linear ramp, cosine), evaluated by one generic function. ``Scheduler.step`` writes the
values into the optimizer's param groups by group kind, so adding a curve or a group kind is a
table entry rather than a new method. One deliberate difference: a zero-length warmdown
(``warmdown_ratio = 0``) is a flat LR instead of the reference's division by zero.
"""

from __future__ import annotations

import math
from collections.abc import Callable
from dataclasses import dataclass

import torch

from mint_b200.config.base import Config


@dataclass
class SchedulerConfig(Config):
    weight_decay: float = 0.0
    weight_decay_lm_head: float = 0.01
    weight_decay_embedding: float = 0.001
    weight_decay_scalar: float = 0.05
    scalar_lr_multiplier: float = 0.01
    warmup_steps: int = 0
    warmdown_ratio: float = 0.0
    final_lr_frac: float = 0.1
    muon_momentum_warmup_steps: int = 400
    muon_momentum_start: float = 0.85
    muon_momentum_peak: float = 0.97
    muon_momentum_final: float = 0.90
    unembedding_lr: float = 0.004
    embedding_lr: float = 0.2
    matrix_lr: float = 0.02
    scalar_lr: float = 0.5


@dataclass(frozen=True)
class Segment:
    """``shape`` over steps ``[lo, hi)``: value(step) for step in range (None: unbounded above)."""

    lo: int
    hi: int | None
    shape: Callable[[int], float]

    def covers(self, step: int) -> bool:
        return step >= self.lo and (self.hi is None or step < self.hi)


def linear(x0: float, y0: float, x1: float, y1: float) -> Callable[[int], float]:
    """The line through (x0, y0) and (x1, y1); a degenerate span is the constant y1."""
    if x1 == x0:
        return lambda _s: y1
    return lambda s: y0 + (y1 - y0) * (s - x0) / (x1 - x0)


def constant(y: float) -> Callable[[int], float]:
    return lambda _s: y


def evaluate(curve: list[Segment], step: int, default: float) -> float:
    """The first segment covering ``step`` decides (earlier segments take precedence)."""
    for seg in curve:
        if seg.covers(step):
            return seg.shape(step)
    return default


def lr_curve(total: int, warmup: int, warmdown: int, final_frac: float) -> list[Segment]:
    start = total - warmdown
    curve = []
    if warmup > 0:
        curve.append(Segment(0, warmup, lambda s: (s + 1) / warmup))
    curve.append(Segment(-(1 << 62), start + 1, constant(1.0)))
    if warmdown > 0:
        curve.append(Segment(start + 1, None, linear(start, 1.0, total, final_frac)))
    return curve


def momentum_curve(total: int, ramp: int, warmdown: int, start: float, peak: float, final: float) -> list[Segment]:
    wd_start = total - warmdown
    curve = []
    if ramp > 0:
        curve.append(Segment(0, ramp, linear(0, start, ramp, peak)))
    if warmdown > 0:
        curve.append(Segment(wd_start, None, linear(wd_start, peak, total, final)))
    return curve


def cosine_to_zero(total: int, peak: float) -> list[Segment]:
    return [Segment(-(1 << 62), None, lambda s: peak * 0.5 * (1.0 + math.cos(math.pi * s / total)))]


class Scheduler:
    """Per-step values of the recipe's curves, applied to optimizer param groups by kind."""

    # group kind -> {param-group key: curve name}; "lr" is a multiplier of the group's initial_lr
    APPLY: dict[str, dict[str, str]] = {
        "adamw": {"lr": "lr_multiplier"},
        "muon": {"lr": "lr_multiplier", "momentum": "muon_momentum", "weight_decay": "muon_weight_decay"},
    }

    def __init__(self, num_iterations: int, config: SchedulerConfig) -> None:
        self.num_iterations = num_iterations
        warmdown = round(config.warmdown_ratio * num_iterations)
        self.curves: dict[str, tuple[list[Segment], float]] = {
            "lr_multiplier": (lr_curve(num_iterations, config.warmup_steps, warmdown, config.final_lr_frac), 1.0),
            "muon_momentum": (momentum_curve(num_iterations, config.muon_momentum_warmup_steps, warmdown,
                                             config.muon_momentum_start, config.muon_momentum_peak,
                                             config.muon_momentum_final), config.muon_momentum_peak),
            "muon_weight_decay": (cosine_to_zero(num_iterations, config.weight_decay), config.weight_decay),
        }

    def values(self, step: int) -> dict[str, float]:
        return {name: evaluate(curve, step, default) for name, (curve, default) in self.curves.items()}

    def get_lr_multiplier(self, step: int) -> float:
        return self.values(step)["lr_multiplier"]

    def get_muon_momentum(self, step: int) -> float:
        return self.values(step)["muon_momentum"]

    def get_weight_decay(self, step: int) -> float:
        return self.values(step)["muon_weight_decay"]

    def step(self, optimizer: torch.optim.Optimizer, step: int) -> dict[str, float]:
        vals = self.values(step)
        for group in optimizer.param_groups:
            for key, name in self.APPLY.get(group.get("kind", "adamw"), self.APPLY["adamw"]).items():
                group[key] = group["initial_lr"] * vals[name] if key == "lr" else vals[name]
        return vals
