"""Model config marker and HF-output unwrapping wrapper (mint/nn/base.py:10-24)."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch
from torch import nn

from mint_b200.config.base import Config


@dataclass
class ModelConfig(Config): ...


class LogitsWrapper(nn.Module):
    """Returns ``.logits`` for HF-style outputs and forwards ``generate``."""

    def __init__(self, model: nn.Module) -> None:
        super().__init__()
        self._model: Any = model

    def forward(self, *args: Any, **kwargs: Any) -> torch.Tensor:  # noqa: ANN401
        output = self._model(*args, **kwargs)
        return output.logits if hasattr(output, "logits") else output

    def generate(self, *args: Any, **kwargs: Any) -> torch.Tensor:  # noqa: ANN401
        return self._model.generate(*args, **kwargs)

    def __getattr__(self, name: str) -> Any:  # noqa: ANN401
        # ``token_logps`` (fused DPO log-probs) and other model methods pass through
        try:
            return super().__getattr__(name)
        except AttributeError:
            if name == "_model":
                raise
            return getattr(self._modules["_model"] if "_model" in self._modules else self.__dict__["_model"], name)


def compute_dtype(t: torch.Tensor) -> torch.dtype:
    """The dtype GEMMs should run in: the autocast dtype when autocast is on, else ``t.dtype``."""
    dev = t.device.type
    if dev in ("cuda", "cpu") and torch.is_autocast_enabled(dev):
        return torch.get_autocast_dtype(dev)
    return t.dtype
