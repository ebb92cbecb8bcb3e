"""Synthetic letter-counting / spelling tasks (mint/data/datasets/spellingbee.py:25-145)."""

from __future__ import annotations

import random
import re
import urllib.request
from pathlib import Path
from typing import Any, Literal

from mint_b200.data.datasets.base import SFTEvalDataset, SFTTrainDataset

LETTERS = "abcdefghijklmnopqrstuvwxyz"
WORD_LIST_URL = "https://raw.githubusercontent.com/dwyl/english-words/refs/heads/master/words_alpha.txt"
TEST_SEED_OFFSET = 10_000_000
USER_TEMPLATES = [
    "How many {letter} are in the word {word}",
    "How many {letter} are in {word}",
    "Count the number of {letter} in {word}",
    "How many times does {letter} appear in {word}",
    "What's the count of {letter} in {word}",
]
_CACHE = "/tmp/words_alpha.txt"  # noqa: S108


def load_words() -> list[str]:
    if not Path(_CACHE).exists():
        urllib.request.urlretrieve(WORD_LIST_URL, _CACHE)  # noqa: S310
    with Path(_CACHE).open() as fh:
        return [line.strip() for line in fh]


class SpellingBee(SFTTrainDataset, SFTEvalDataset):
    ANSWER_RE = re.compile(r"#### (\-?[0-9\.\,]+)")

    def __init__(self, size: int = 1000, split: Literal["train", "test"] = "train", words: list[str] | None = None) -> None:
        super().__init__()
        self.size = size
        self.split = split
        self.words = words if words is not None else load_words()

    @property
    def eval_type(self) -> Literal["categorical", "generative"]:
        return "generative"

    def __len__(self) -> int:
        return self.size

    def __getitem__(self, index: int) -> dict[str, Any]:
        rng = random.Random(index if self.split == "train" else TEST_SEED_OFFSET + index)  # noqa: S311
        word = rng.choice(self.words)
        letter = rng.choice(word) if rng.random() < 0.9 else rng.choice(LETTERS)
        count = word.count(letter)
        return {"messages": [{"role": "user", "content": self._create_user_message(rng, word, letter)},
                             {"role": "assistant", "content": self._create_assistant_parts(word, letter, count)}]}

    def evaluate(self, conversation: dict[str, Any], completion: str) -> bool:
        truth = conversation["messages"][-1]["content"][-1]["text"]
        return self._extract_answer(completion) == self._extract_answer(truth)

    @staticmethod
    def _create_user_message(rng: random.Random, word: str, letter: str) -> str:
        template = rng.choice(USER_TEMPLATES)
        if rng.random() < 0.3:
            template = template.lower()
        quote = rng.choice(["", "'", '"'])
        msg = template.format(letter=f"{quote}{letter}{quote}", word=f"{quote}{word}{quote}")
        return msg + "?" if rng.random() < 0.5 else msg

    @staticmethod
    def _create_assistant_parts(word: str, letter: str, count: int) -> list[dict[str, str]]:
        text = f"Let me spell '{word}': {','.join(word)}\n\nCounting '{letter}':\n"
        running = 0
        for i, ch in enumerate(word, 1):
            if ch == letter:
                running += 1
                text += f"{i}:{ch} hit! count={running}\n"
            else:
                text += f"{i}:{ch}\n"
        text += f"\nManual count: {running}"
        return [
            {"type": "text", "text": text},
            {"type": "text", "text": "\n\nVerifying with Python:\n\n"},
            {"type": "python", "text": f"'{word}'.count('{letter}')"},
            {"type": "python_output", "text": str(count)},
            {"type": "text", "text": f"\n\nFinal answer:\n\n#### {count}"},
        ]

    def _extract_answer(self, text: str) -> str | None:
        m = self.ANSWER_RE.search(text)
        return m.group(1).strip().replace(",", "") if m else None


class SimpleSpelling(SFTTrainDataset):
    def __init__(self, size: int = 1000, split: Literal["train", "test"] = "train", words: list[str] | None = None) -> None:
        super().__init__()
        self.size = size
        self.split = split
        ws = list(words) if words is not None else load_words()
        random.Random(42).shuffle(ws)  # noqa: S311
        self.words = ws

    def __len__(self) -> int:
        return self.size

    def __getitem__(self, index: int) -> dict[str, Any]:
        rng = random.Random(index if self.split == "train" else TEST_SEED_OFFSET + index)  # noqa: S311
        word = rng.choice(self.words)
        return {"messages": [{"role": "user", "content": f"Spell the word: {word}"},
                             {"role": "assistant", "content": f"{word}:{','.join(word)}"}]}
