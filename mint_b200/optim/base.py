"""Optimizer config marker (mint/optim/base.py:6-7)."""

from __future__ import annotations

from dataclasses import dataclass

from mint_b200.config.base import Config


@dataclass
class OptimConfig(Config): ...
