"""Distributed dataloader ABC and ``[dl]`` config table (mint/data/dataloader.py:13-50)."""

from __future__ import annotations

from abc import ABC, abstractmethod
from collections.abc import Iterator
from dataclasses import dataclass
from pathlib import Path
from typing import Any

from mint_b200.config.base import Config
from mint_b200.data.sampler import Sampler


@dataclass
class DataloaderConfig(Config):
    data_dir: str = "data/climbmix"
    batch_size: int = 4
    buffer_size: int = 1000
    tokenizer_batch_size: int = 128
    seq_length: int = 512
    # extension: "parquet" (BOS best-fit packing of text shards) or "synthetic" (uniform random ids)
    source: str = "parquet"
    synthetic_vocab_size: int = 0
    seed: int = 4321


class DistributedDataloader(Sampler, ABC):
    def __init__(self, device: Any, data_dir: str, batch_size: int, seq_len: int, tokenizer: Any,  # noqa: ANN401
                 *args: Any, **kwargs: Any) -> None:  # noqa: ANN401, ARG002
        super().__init__()
        self.device = device
        self.data_dir = Path(data_dir)
        self.B = batch_size
        self.T = seq_len
        self.tokenizer = tokenizer

    @abstractmethod
    def batch_loader(self, split: str = "train", resume_state: dict | None = None) -> Iterator[Any]: ...

    @abstractmethod
    def get_state(self) -> dict: ...

    @abstractmethod
    def set_state(self, state: dict) -> None: ...
