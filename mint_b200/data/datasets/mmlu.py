"""MMLU multiple-choice SFT/eval dataset (mint/data/datasets/mmlu.py:8-40)."""

from __future__ import annotations

from typing import Any, Literal

from mint_b200.data.datasets.base import SFTEvalDataset, SFTTrainDataset, build_mc_prompt, hf_load


class MMLU(SFTTrainDataset, SFTEvalDataset):
    LETTERS = ("A", "B", "C", "D")

    def __init__(self, subset: Literal["all"] = "all",
                 split: Literal["auxiliary_train", "validation", "dev", "test"] = "test", ds: Any = None) -> None:  # noqa: ANN401
        super().__init__()
        self.ds = ds if ds is not None else hf_load("cais/mmlu", subset, split=split)

    @property
    def eval_type(self) -> Literal["categorical", "generative"]:
        return "categorical"

    def __len__(self) -> int:
        return len(self.ds)

    def __getitem__(self, index: int) -> dict[str, Any]:
        row = self.ds[index]
        return {
            "messages": [
                {"role": "user", "content": build_mc_prompt(row["question"], self.LETTERS, row["choices"])},
                {"role": "assistant", "content": self.LETTERS[row["answer"]]},
            ],
            "subject": row["subject"],
            "letters": self.LETTERS,
        }

    def evaluate(self, conversation: dict[str, Any], completion: str) -> bool:
        return completion == conversation["messages"][-1]["content"]
