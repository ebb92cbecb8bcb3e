"""DPO dataloader (mint/data/dist/dpo.py:14-190): JSONL ``{prompt, chosen, rejected}`` rows
(pydantic-validated), dp-strided, rendered as conversations; labels are -100 outside assistant
tokens; chosen and rejected are right-padded to a common length."""

from __future__ import annotations

import random
from collections.abc import Iterator
from pathlib import Path
from typing import Any, Literal

import torch
from pydantic import BaseModel, ConfigDict

from mint_b200.data.dataloader import DataloaderConfig, DistributedDataloader


class ContentPart(BaseModel):
    type: Literal["text", "python", "python_output"]
    text: str


class Message(BaseModel):
    role: Literal["system", "user", "assistant"]
    content: str | list[ContentPart]


class Row(BaseModel):
    prompt: list[Message]
    chosen: list[Message]
    rejected: list[Message]


class Batch(BaseModel):
    model_config = ConfigDict(arbitrary_types_allowed=True)
    chosen_input_ids: torch.Tensor
    chosen_attn_mask: torch.Tensor
    chosen_labels: torch.Tensor
    rejected_input_ids: torch.Tensor
    rejected_attn_mask: torch.Tensor
    rejected_labels: torch.Tensor


class DistributedDPODataloader(DistributedDataloader):
    def __init__(self, device: Any, config: DataloaderConfig, tokenizer: Any, filename: str,  # noqa: ANN401
                 *args: Any, **kwargs: Any) -> None:  # noqa: ANN401
        super().__init__(device, config.data_dir, config.batch_size, config.seq_length, tokenizer, *args, **kwargs)
        self.filepath = Path(config.data_dir) / Path(filename)
        info = device.process_info()
        self.rank = info["dp_rank"]
        self.world_size = info["dp_size"]
        if not self.filepath.exists():
            raise FileNotFoundError(f"DPO data not found: {self.filepath}")

    def _iter_rows(self) -> Iterator[Row]:
        with self.filepath.open("r", encoding="utf-8") as fh:
            for i, line in enumerate(fh):
                if i % self.world_size != self.rank or not line.strip():
                    continue
                yield Row.model_validate_json(line.strip())

    def _render(self, msgs: list[Message]) -> tuple[list[int], list[int]]:
        return self.tokenizer.render_conversation({"messages": [m.model_dump() for m in msgs]}, max_tokens=self.T)

    def _collate_batch(self, rows: list[Row]) -> Batch:
        seqs: dict[str, list[torch.Tensor]] = {k: [] for k in ("ci", "ca", "cl", "ri", "ra", "rl")}
        for row in rows:
            for tag, msgs in (("c", row.prompt + row.chosen), ("r", row.prompt + row.rejected)):
                ids, mask = self._render(msgs)
                labels = [t if m == 1 else -100 for t, m in zip(ids, mask, strict=False)]
                seqs[tag + "i"].append(torch.tensor(ids, dtype=torch.long))
                seqs[tag + "a"].append(torch.ones(len(ids), dtype=torch.bool))
                seqs[tag + "l"].append(torch.tensor(labels, dtype=torch.long))
        width = max(s.numel() for s in seqs["ci"] + seqs["ri"])
        dev = self.device.device

        def pad(items: list[torch.Tensor], value: int) -> torch.Tensor:
            out = torch.full((len(items), width), value, dtype=items[0].dtype)
            for i, s in enumerate(items):
                out[i, : s.numel()] = s
            return out.to(dev)

        pad_id = self.tokenizer.pad_token
        return Batch(
            chosen_input_ids=pad(seqs["ci"], pad_id), chosen_attn_mask=pad(seqs["ca"], 0),
            chosen_labels=pad(seqs["cl"], -100), rejected_input_ids=pad(seqs["ri"], pad_id),
            rejected_attn_mask=pad(seqs["ra"], 0), rejected_labels=pad(seqs["rl"], -100),
        )

    def batch_loader(self, split: str = "train", resume_state: dict | None = None) -> Iterator[Batch]:  # noqa: ARG002
        rows: list[Row] = []
        for row in self._iter_rows():
            rows.append(row)
            if len(rows) == self.B:
                yield self._collate_batch(rows)
                rows = []

    def get_state(self) -> dict:
        return {}

    def set_state(self, state: dict) -> None:
        pass

    def sample(self, num_samples: int = 1) -> list[dict]:
        rows = list(self._iter_rows())
        out: list[dict] = []
        for _ in range(num_samples if rows else 0):
            row = random.choice(rows)  # noqa: S311
            c_ids, c_mask = self._render(row.prompt + row.chosen)
            r_ids, r_mask = self._render(row.prompt + row.rejected)
            ct, rt = torch.tensor(c_ids[: self.T]), torch.tensor(r_ids[: self.T])
            out.append({"chosen_tokens": ct, "rejected_tokens": rt,
                        "chosen_str": self.tokenizer.decode(ct.unsqueeze(0))[0],
                        "rejected_str": self.tokenizer.decode(rt.unsqueeze(0))[0],
                        "chosen_mask": c_mask[: self.T], "rejected_mask": r_mask[: self.T]})
        return out
