"""SFT dataset ABCs and the multiple-choice prompt builder (mint/data/datasets/base.py:5-45)."""

from __future__ import annotations

from abc import abstractmethod
from typing import Any, Literal


class SFTDataset:
    def __init__(self) -> None:
        super().__init__()
        self.index = 0

    @abstractmethod
    def __len__(self) -> int: ...

    @abstractmethod
    def __getitem__(self, index: int) -> dict[str, Any]: ...


class SFTTrainDataset(SFTDataset):
    def next(self) -> dict[str, Any]:
        example = self[self.index]
        self.index = (self.index + 1) % len(self)
        return example

    def reset(self) -> None:
        self.index = 0


class SFTEvalDataset(SFTDataset):
    @property
    @abstractmethod
    def eval_type(self) -> Literal["categorical", "generative"]: ...

    @abstractmethod
    def evaluate(self, conversation: dict[str, Any], completion: str) -> bool: ...


def build_mc_prompt(question: str, letters: tuple[str, ...], choices: list[str]) -> str:
    lines = [f"Multiple Choice question: {question}\n"]
    lines += [f"- {choice}={letter}\n" for letter, choice in zip(letters, choices, strict=True)]
    lines.append("\nRespond only with the letter of the correct answer.")
    return "".join(lines)


def hf_load(path: str, *args: Any, **kwargs: Any):  # noqa: ANN201, ANN401
    """``datasets.load_dataset(...).shuffle(seed=42)`` (the reference's loading convention)."""
    from datasets import load_dataset  # noqa: PLC0415

    return load_dataset(path, *args, **kwargs).shuffle(seed=42)
