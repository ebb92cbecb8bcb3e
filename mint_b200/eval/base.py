"""Evaluation task types, ``[train.eval]`` config and the Evaluator ABC (mint/eval/base.py:12-33)."""

from __future__ import annotations

from abc import ABC, abstractmethod
from dataclasses import dataclass
from enum import Enum
from typing import Any

from torch import nn

from mint_b200.config.base import Config


class Task(Enum):
    MC = "multiple_choice"
    SCHEMA = "schema"
    LM = "language_modeling"


@dataclass
class EvalConfig(Config):
    seq_length: int = 512
    max_new_tokens: int = 256


class Evaluator(ABC):
    def __init__(self, model: nn.Module, config: EvalConfig, device: Any) -> None:  # noqa: ANN401
        self.model: Any = model
        self.config = config
        self.device = device
        self.process_info = device.process_info()

    @abstractmethod
    def evaluate(self, *args: Any, **kwargs: Any) -> dict[str, Any]: ...  # noqa: ANN401
