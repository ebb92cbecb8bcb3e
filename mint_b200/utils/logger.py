"""loguru logger on stderr at INFO, plus the W&B ``LoggerConfig`` table (mint/utils/logger.py:12-34)."""

from __future__ import annotations

import os
import sys
from dataclasses import dataclass

from loguru import logger

from mint_b200.config.base import Config

__all__ = ["LoggerConfig", "logger"]

logger.remove()
logger.add(
    sys.stderr,
    format=(
        "<green>{time:YYYY-MM-DD HH:mm:ss}</green> | <level>{level: <8}</level> | "
        "<cyan>{name}</cyan>:<cyan>{function}</cyan>:<cyan>{line}</cyan> - <level>{message}</level>"
    ),
    level=os.environ.get("MINT_LOG_LEVEL", "INFO"),
    colorize=True,
)


@dataclass
class LoggerConfig(Config):
    wandb_enabled: bool = True
    wandb_project: str = "goda"
    wandb_run_name: str | None = None
    wandb_entity: str | None = None
