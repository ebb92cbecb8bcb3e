"""AI2 ARC multiple-choice SFT/eval dataset (mint/data/datasets/arc.py:8-38)."""

from __future__ import annotations

from typing import Any, Literal

from mint_b200.data.datasets.base import SFTEvalDataset, SFTTrainDataset, build_mc_prompt, hf_load


class ARC(SFTTrainDataset, SFTEvalDataset):
    def __init__(self, subset: Literal["ARC-Easy", "ARC-Challenge"] = "ARC-Challenge",
                 split: Literal["train", "validation", "test"] = "train", ds: Any = None) -> None:  # noqa: ANN401
        super().__init__()
        self.ds = ds if ds is not None else hf_load("allenai/ai2_arc", subset, split=split)

    @property
    def eval_type(self) -> Literal["categorical", "generative"]:
        return "categorical"

    def __len__(self) -> int:
        return len(self.ds)

    def __getitem__(self, index: int) -> dict[str, Any]:
        row = self.ds[index]
        letters = tuple(row["choices"]["label"])
        return {
            "messages": [
                {"role": "user", "content": build_mc_prompt(row["question"], letters, row["choices"]["text"])},
                {"role": "assistant", "content": row["answerKey"]},
            ],
            "letters": letters,
        }

    def evaluate(self, conversation: dict[str, Any], completion: str) -> bool:
        return completion == conversation["messages"][-1]["content"]
