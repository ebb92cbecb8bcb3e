"""GSM8K with calculator annotations turned into python / python_output parts (mint/data/datasets/gsm8k.py:9-61)."""

from __future__ import annotations

import re
from typing import Any, Literal

from mint_b200.data.datasets.base import SFTEvalDataset, SFTTrainDataset, hf_load

ANSWER_RE = re.compile(r"#### (\-?[0-9\.\,]+)")


def extract_answer(text: str) -> str | None:
    m = ANSWER_RE.search(text)
    return m.group(1).strip().replace(",", "") if m else None


def answer_parts(answer: str) -> list[dict[str, str]]:
    parts: list[dict[str, str]] = []
    for seg in re.split(r"(<<[^>]+>>)", answer):
        if seg.startswith("<<") and seg.endswith(">>"):
            inner = seg[2:-2]
            expr, result = inner.rsplit("=", 1) if "=" in inner else (inner, "")
            parts.append({"type": "python", "text": expr})
            parts.append({"type": "python_output", "text": result})
        else:
            parts.append({"type": "text", "text": seg})
    return parts


class GSM8K(SFTTrainDataset, SFTEvalDataset):
    ANSWER_RE = ANSWER_RE

    def __init__(self, subset: Literal["main", "socratic"] = "main",
                 split: Literal["train", "test"] = "train", ds: Any = None) -> None:  # noqa: ANN401
        super().__init__()
        self.ds = ds if ds is not None else hf_load("openai/gsm8k", subset, split=split)

    @property
    def eval_type(self) -> Literal["categorical", "generative"]:
        return "generative"

    def __len__(self) -> int:
        return len(self.ds)

    def __getitem__(self, index: int) -> dict[str, Any]:
        row = self.ds[index]
        return {"messages": [{"role": "user", "content": row["question"]},
                             {"role": "assistant", "content": answer_parts(row["answer"])}]}

    def evaluate(self, conversation: dict[str, Any], completion: str) -> bool:
        truth = conversation["messages"][-1]["content"][-1]["text"]
        return extract_answer(completion) == extract_answer(truth)

    def _extract_answer(self, text: str) -> str | None:
        return extract_answer(text)
