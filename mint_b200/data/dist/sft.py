"""SFT dataloader (mint/data/dist/sft.py:12-139): seeded mixture shuffle, dp-strided, chat rendering,
right-padded rows of ``T + 1`` tokens split into inputs / targets / loss mask."""

from __future__ import annotations

import random
from collections.abc import Iterator
from typing import Any

import torch

from mint_b200.data.dataloader import DataloaderConfig, DistributedDataloader


class DistributedSFTDataloader(DistributedDataloader):
    def __init__(self, device: Any, config: DataloaderConfig, tokenizer: Any, datasets: list,  # noqa: ANN401
                 shuffle: bool = True, *args: Any, **kwargs: Any) -> None:  # noqa: ANN401, FBT001, FBT002
        super().__init__(device, config.data_dir, config.batch_size, config.seq_length, tokenizer, *args, **kwargs)
        self.datasets = datasets
        self.max_tokens = config.seq_length
        self.shuffle = shuffle
        info = device.process_info()
        self.rank = info["dp_rank"]
        self.world_size = info["dp_size"]
        self.dataset_indices = self._build_dataset_indices()
        self.rank_indices = [ix for i, ix in enumerate(self.dataset_indices) if i % self.world_size == self.rank]
        pin = device.is_cuda
        self.cpu_buffer = torch.empty(2 * self.B * self.T, dtype=torch.long, pin_memory=pin)
        self.gpu_buffer = torch.empty(2 * self.B * self.T, dtype=torch.long, device=device.device)
        self.cpu_inputs = self.cpu_buffer[: self.B * self.T].view(self.B, self.T)
        self.cpu_targets = self.cpu_buffer[self.B * self.T :].view(self.B, self.T)
        self.cpu_mask = torch.zeros(self.B, self.T, dtype=torch.long, pin_memory=pin)
        self.inputs = self.gpu_buffer[: self.B * self.T].view(self.B, self.T)
        self.targets = self.gpu_buffer[self.B * self.T :].view(self.B, self.T)
        self.mask = torch.zeros(self.B, self.T, dtype=torch.long, device=device.device)
        self.position = 0

    def _build_dataset_indices(self) -> list:
        idx = [(d, i) for d, ds in enumerate(self.datasets) for i in range(len(ds))]
        if self.shuffle:
            random.Random(42).shuffle(idx)
        return idx

    def _partition_for_rank(self) -> list:
        return self.rank_indices

    def _row(self, conversation: dict) -> tuple[list[int], list[int]]:
        ids, mask = self.tokenizer.render_conversation(conversation, self.max_tokens)
        if len(ids) <= self.T:
            pad = self.T + 1 - len(ids)
            ids = ids + [self.tokenizer.pad_token] * pad
            mask = mask + [0] * pad
        else:
            ids, mask = ids[: self.T + 1], mask[: self.T + 1]
        return ids, mask

    def batch_loader(self, split: str = "train", resume_state: dict | None = None) -> Iterator:  # noqa: ARG002
        total = len(self.rank_indices)
        if total == 0:
            return
        nb = self.device.is_cuda
        while True:
            for b in range(self.B):
                d, i = self.rank_indices[self.position % total]
                self.position += 1
                ids, mask = self._row(self.datasets[d][i])
                self.cpu_inputs[b] = torch.tensor(ids[:-1], dtype=torch.long)
                self.cpu_targets[b] = torch.tensor(ids[1:], dtype=torch.long)
                self.cpu_mask[b] = torch.tensor(mask[1:], dtype=torch.long)
            self.gpu_buffer.copy_(self.cpu_buffer, non_blocking=nb)
            self.mask.copy_(self.cpu_mask, non_blocking=nb)
            yield self.inputs, self.targets, self.mask, None

    def get_state(self) -> dict:
        return {"position": self.position}

    def set_state(self, state: dict) -> None:
        self.position = state.get("position", 0)

    def sample(self, num_samples: int = 1) -> list[dict]:
        out = []
        for _ in range(num_samples):
            ds = random.choice(self.datasets)  # noqa: S311
            conv = ds[random.randint(0, len(ds) - 1)]  # noqa: S311
            ids, _ = self.tokenizer.render_conversation(conv, self.max_tokens)
            ids = ids[: self.T]
            inp = torch.tensor(ids[:-1] if len(ids) > 1 else ids, dtype=torch.long)
            tgt = torch.tensor(ids[1:] if len(ids) > 1 else ids, dtype=torch.long)
            out.append({"input_tokens": inp, "target_tokens": tgt,
                        "input_str": self.tokenizer.decode(inp.unsqueeze(0))[0],
                        "target_str": self.tokenizer.decode(tgt.unsqueeze(0))[0]})
        return out
