"""Adapter ABC (mint/sft/peft/base.py:7-11)."""

from __future__ import annotations

from abc import ABC, abstractmethod
from typing import Any

from torch import nn


class Adapter(ABC):
    @classmethod
    @abstractmethod
    def apply(cls, model: nn.Module, **kwargs: Any) -> None: ...  # noqa: ANN401
