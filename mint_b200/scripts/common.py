"""Model construction shared by the entry scripts (scripts/pretrain.py:59-99 in the reference)."""

from __future__ import annotations

from typing import Any

import torch
from torch import nn

from mint_b200.models.gemma import Gemma, GemmaConfig
from mint_b200.utils.device import Device
from mint_b200.utils.logger import logger


def build_model(config: GemmaConfig, train_cfg: Any, device: Device, *, seed: int = 1337) -> nn.Module:  # noqa: ANN401
    """Same seed on every rank (identical init), meta-device init when configured, then TP/ZeRO setup."""
    torch.manual_seed(seed)
    if getattr(train_cfg, "use_meta_device", False):
        with torch.device("meta"):
            model = Gemma(config, gradient_checkpointing=train_cfg.gradient_checkpointing)
        logger.info(f"Model parameters: {model.get_num_params():,} non-embedding | "
                    f"{model.get_num_params(non_embedding=False):,} total")
        model = device.move_to_device(model, from_meta=True)
    else:
        model = Gemma(config, gradient_checkpointing=train_cfg.gradient_checkpointing)
        model = device.move_to_device(model, from_meta=False)
    model = device.setup_parallel(model, tp_plan=getattr(config, "tp_plan", None))
    if getattr(train_cfg, "compile_model", False):
        model = device.compile_model(model, enabled=True)
    return model


def check_vocab(config: GemmaConfig, tokenizer: Any) -> None:  # noqa: ANN401
    if tokenizer is not None and config.vocab_size != tokenizer.vocab_size:
        raise ValueError(f"Vocab size mismatch: config={config.vocab_size}, tokenizer={tokenizer.vocab_size}")
