"""SmolTalk chat SFT dataset (mint/data/datasets/smoltalk.py:8-17)."""

from __future__ import annotations

from typing import Any, Literal

from mint_b200.data.datasets.base import SFTTrainDataset, hf_load


class SmolTalk(SFTTrainDataset):
    def __init__(self, split: Literal["train", "test"] = "train", ds: Any = None) -> None:  # noqa: ANN401
        super().__init__()
        self.ds = ds if ds is not None else hf_load("HuggingFaceTB/smol-smoltalk", split=split)

    def __len__(self) -> int:
        return len(self.ds)

    def __getitem__(self, index: int) -> dict[str, Any]:
        return {"messages": self.ds[index]["messages"]}
