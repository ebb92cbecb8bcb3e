"""Conversations from a local JSONL file, one message list per line (mint/data/datasets/customjsonl.py:8-25)."""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any

from mint_b200.data.datasets.base import SFTTrainDataset


class CustomJSON(SFTTrainDataset):
    def __init__(self, filepath: str) -> None:
        super().__init__()
        self.filepath = filepath
        self.conversations: list[Any] = []
        if Path(filepath).exists():
            with Path(filepath).open(encoding="utf-8") as fh:
                self.conversations = [json.loads(line) for line in fh if line.strip()]

    def __len__(self) -> int:
        return len(self.conversations)

    def __getitem__(self, index: int) -> dict[str, Any]:
        return {"messages": self.conversations[index]}
