"""SFT / eval conversation datasets as table entries of one generic adapter.

The reference has one hand-written class per dataset (mint/data/datasets/{arc,mmlu,gsm8k,humaneval,
smoltalk,spellingbee,customjsonl}.py). Here a dataset is a :class:`Spec` -- where rows come from,
how a row becomes a conversation, how a completion is graded -- and :class:`TableDataset` turns
any spec into the ``SFTTrainDataset`` / ``SFTEvalDataset`` interface. The conversations (message
texts, roles, the multiple-choice prompt wording, the calculator and letter-counting traces) are the
training / eval formats the reference's tokenizer and graders expect, so they are kept as is:

* multiple choice (ARC, MMLU): user = ``build_mc_prompt``, assistant = the answer letter, graded by
  exact match;
* GSM8K: ``<<expr=result>>`` calculator annotations become python / python_output parts, graded by
  the ``#### <number>`` answer;
* HumanEval: graded by running the completion's code against the task's tests in a separate
  process (``mint_b200.utils.exec``);
* SmolTalk / CustomJSON: message lists from the hub or a local JSONL file (train only);
* SpellingBee / SimpleSpelling: generated per index from a word list with a seeded RNG (test split
  seeds offset by 10,000,000).
"""

from __future__ import annotations

import json
import random
import re
import urllib.request
from collections.abc import Callable
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Literal

from mint_b200.data.datasets.base import SFTEvalDataset, SFTTrainDataset, build_mc_prompt, hf_load
from mint_b200.utils.exec import execute_code

Conversation = dict[str, Any]
Row = dict[str, Any]

ANSWER_RE = re.compile(r"#### (\-?[0-9\.\,]+)")
WORD_LIST_URL = "https://raw.githubusercontent.com/dwyl/english-words/refs/heads/master/words_alpha.txt"
WORD_CACHE = Path("/tmp/words_alpha.txt")  # noqa: S108
TEST_SEED_OFFSET = 10_000_000
ALPHABET = "abcdefghijklmnopqrstuvwxyz"


# ---------------------------------------------------------------------------------------------- graders
def final_number(text: str) -> str | None:
    """The ``#### <number>`` answer of a GSM8K-style solution, commas removed."""
    m = ANSWER_RE.search(text)
    return m.group(1).strip().replace(",", "") if m else None


def _reference_text(conv: Conversation) -> str:
    content = conv["messages"][-1]["content"]
    return content if isinstance(content, str) else content[-1]["text"]


def grade_exact(conv: Conversation, completion: str) -> bool:
    return completion == _reference_text(conv)


def grade_final_number(conv: Conversation, completion: str) -> bool:
    return final_number(completion) == final_number(_reference_text(conv))


def _leading_imports(prompt: str) -> str:
    """Import lines at the top of a HumanEval prompt (before the first code line)."""
    keep = []
    for line in prompt.splitlines():
        s = line.strip()
        if not s or s.startswith("#"):
            continue
        if not s.startswith(("import ", "from ")):
            break
        keep.append(s)
    return "\n".join(keep)


def _code_block(completion: str) -> str:
    blocks = re.findall(r"```(?:python)?\s*\n(.*?)\n```", completion, re.DOTALL)
    return (blocks[0] if blocks else completion).strip()


def grade_by_tests(conv: Conversation, completion: str) -> bool:
    program = "\n\n".join([_leading_imports(conv["messages"][0]["content"]), _code_block(completion),
                           f"{conv['test']}\ncheck({conv['entry_point']})"])
    return execute_code(program).success


# ---------------------------------------------------------------------------------------------- renderers
def _turns(user: Any, assistant: Any) -> list[dict[str, Any]]:  # noqa: ANN401
    return [{"role": "user", "content": user}, {"role": "assistant", "content": assistant}]


def multiple_choice(question: Callable[[Row], str], choices: Callable[[Row], list[str]],
                    letters: Callable[[Row], tuple[str, ...]], answer: Callable[[Row], str],
                    extra: tuple[str, ...] = ()) -> Callable[[Row], Conversation]:
    def render(row: Row) -> Conversation:
        ls = letters(row)
        conv = {"messages": _turns(build_mc_prompt(question(row), ls, choices(row)), answer(row)), "letters": ls}
        conv.update({k: row[k] for k in extra})
        return conv

    return render


def calculator_parts(solution: str) -> list[dict[str, str]]:
    """Split ``<<expr=result>>`` annotations of a solution into python / python_output parts."""
    parts = []
    for piece in re.split(r"(<<[^>]+>>)", solution):
        if piece.startswith("<<") and piece.endswith(">>"):
            inner = piece[2:-2]
            expr, _, result = inner.rpartition("=") if "=" in inner else (inner, "", "")
            parts += [{"type": "python", "text": expr}, {"type": "python_output", "text": result}]
        else:
            parts.append({"type": "text", "text": piece})
    return parts


def gsm8k_render(row: Row) -> Conversation:
    return {"messages": _turns(row["question"], calculator_parts(row["answer"]))}


def humaneval_render(row: Row) -> Conversation:
    return {"messages": _turns(row["prompt"], f"{row['prompt']}\n{row['canonical_solution']}"),
            "entry_point": row["entry_point"], "test": row["test"]}


def messages_render(row: Row) -> Conversation:
    return {"messages": row["messages"] if isinstance(row, dict) else row}


# ---------------------------------------------------------------------------------------------- synthetic
COUNT_QUESTIONS = (
    "How many {letter} are in the word {word}",
    "How many {letter} are in {word}",
    "Count the number of {letter} in {word}",
    "How many times does {letter} appear in {word}",
    "What's the count of {letter} in {word}",
)


def load_words() -> list[str]:
    if not WORD_CACHE.exists():
        urllib.request.urlretrieve(WORD_LIST_URL, WORD_CACHE)  # noqa: S310
    return [w.strip() for w in WORD_CACHE.read_text().splitlines()]


def _example_rng(index: int, split: str) -> random.Random:
    return random.Random(index if split == "train" else TEST_SEED_OFFSET + index)  # noqa: S311


def counting_trace(word: str, letter: str) -> list[dict[str, str]]:
    """Spell-and-count reasoning, a python check and the ``####`` answer for one (word, letter)."""
    hits = 0
    steps = []
    for pos, ch in enumerate(word, 1):
        hits += ch == letter
        steps.append(f"{pos}:{ch} hit! count={hits}" if ch == letter else f"{pos}:{ch}")
    manual = (f"Let me spell '{word}': {','.join(word)}\n\nCounting '{letter}':\n" + "\n".join(steps) + "\n"
              + f"\nManual count: {hits}")
    return [{"type": "text", "text": manual},
            {"type": "text", "text": "\n\nVerifying with Python:\n\n"},
            {"type": "python", "text": f"'{word}'.count('{letter}')"},
            {"type": "python_output", "text": str(word.count(letter))},
            {"type": "text", "text": f"\n\nFinal answer:\n\n#### {word.count(letter)}"}]


def counting_question(rng: random.Random, word: str, letter: str) -> str:
    template = rng.choice(COUNT_QUESTIONS)
    if rng.random() < 0.3:
        template = template.lower()
    quote = rng.choice(["", "'", '"'])
    text = template.format(letter=f"{quote}{letter}{quote}", word=f"{quote}{word}{quote}")
    return text + "?" if rng.random() < 0.5 else text


def spelling_bee_example(words: list[str], index: int, split: str) -> Conversation:
    rng = _example_rng(index, split)
    word = rng.choice(words)
    letter = rng.choice(word) if rng.random() < 0.9 else rng.choice(ALPHABET)
    return {"messages": _turns(counting_question(rng, word, letter), counting_trace(word, letter))}


def simple_spelling_example(words: list[str], index: int, split: str) -> Conversation:
    word = _example_rng(index, split).choice(words)
    return {"messages": _turns(f"Spell the word: {word}", f"{word}:{','.join(word)}")}


# ---------------------------------------------------------------------------------------------- the table
@dataclass(frozen=True)
class Spec:
    """How a dataset is read (``hub`` = (path, default subset) for ``hf_load``), rendered and graded."""

    render: Callable[[Row], Conversation]
    hub: tuple[str, str | None] | None = None
    default_split: str = "train"
    eval_type: Literal["categorical", "generative"] | None = None  # None: a training-only dataset
    grade: Callable[[Conversation, str], bool] | None = None
    notes: str = field(default="", compare=False)


SPECS: dict[str, Spec] = {
    "ARC": Spec(multiple_choice(lambda r: r["question"], lambda r: r["choices"]["text"],
                                lambda r: tuple(r["choices"]["label"]), lambda r: r["answerKey"]),
                hub=("allenai/ai2_arc", "ARC-Challenge"), default_split="train", eval_type="categorical",
                grade=grade_exact),
    "MMLU": Spec(multiple_choice(lambda r: r["question"], lambda r: r["choices"], lambda _r: ("A", "B", "C", "D"),
                                 lambda r: "ABCD"[r["answer"]], extra=("subject",)),
                 hub=("cais/mmlu", "all"), default_split="test", eval_type="categorical", grade=grade_exact),
    "GSM8K": Spec(gsm8k_render, hub=("openai/gsm8k", "main"), default_split="train", eval_type="generative",
                  grade=grade_final_number),
    "HumanEval": Spec(humaneval_render, hub=("openai/openai_humaneval", None), default_split="test",
                      eval_type="generative", grade=grade_by_tests),
    "SmolTalk": Spec(messages_render, hub=("HuggingFaceTB/smol-smoltalk", None), default_split="train"),
}


class TableDataset(SFTTrainDataset, SFTEvalDataset):
    """A dataset defined by ``SPECS[name]`` over ``rows`` (a hub dataset, a list, any indexable)."""

    name: str = ""

    def __init__(self, subset: str | None = None, split: str | None = None, ds: Any = None) -> None:  # noqa: ANN401
        super().__init__()
        self.spec = SPECS[self.name]
        if ds is None:
            path, default_subset = self.spec.hub
            args = [subset or default_subset] if (subset or default_subset) else []
            ds = hf_load(path, *args, split=split or self.spec.default_split)
        self.ds = ds

    @property
    def eval_type(self) -> Literal["categorical", "generative"]:
        if self.spec.eval_type is None:
            raise TypeError(f"{self.name} is a training-only dataset")
        return self.spec.eval_type

    def __len__(self) -> int:
        return len(self.ds)

    def __getitem__(self, index: int) -> Conversation:
        return self.spec.render(self.ds[index])

    def evaluate(self, conversation: Conversation, completion: str) -> bool:
        if self.spec.grade is None:
            raise TypeError(f"{self.name} has no grader")
        return self.spec.grade(conversation, completion)


class ARC(TableDataset):
    name = "ARC"


class MMLU(TableDataset):
    name = "MMLU"
    LETTERS = ("A", "B", "C", "D")


class GSM8K(TableDataset):
    name = "GSM8K"

    def _extract_answer(self, text: str) -> str | None:
        return final_number(text)


class HumanEval(TableDataset):
    name = "HumanEval"

    def __init__(self, ds: Any = None) -> None:  # noqa: ANN401
        super().__init__(ds=ds)


class SmolTalk(TableDataset):
    name = "SmolTalk"

    def __init__(self, split: str = "train", ds: Any = None) -> None:  # noqa: ANN401
        super().__init__(split=split, ds=ds)


class CustomJSON(SFTTrainDataset):
    """Conversations from a local JSONL file, one message list per line (missing file: empty)."""

    def __init__(self, filepath: str) -> None:
        super().__init__()
        self.filepath = filepath
        path = Path(filepath)
        lines = path.read_text(encoding="utf-8").splitlines() if path.exists() else []
        self.conversations = [json.loads(line) for line in lines if line.strip()]

    def __len__(self) -> int:
        return len(self.conversations)

    def __getitem__(self, index: int) -> Conversation:
        return messages_render(self.conversations[index])


class _Generated(SFTTrainDataset, SFTEvalDataset):
    """``size`` examples generated from a word list, reproducible per (index, split)."""

    make: Callable[[list[str], int, str], Conversation]

    def __init__(self, size: int = 1000, split: str = "train", words: list[str] | None = None) -> None:
        super().__init__()
        self.size, self.split = size, split
        self.words = list(words) if words is not None else load_words()

    def __len__(self) -> int:
        return self.size

    def __getitem__(self, index: int) -> Conversation:
        return type(self).make(self.words, index, self.split)

    @property
    def eval_type(self) -> Literal["categorical", "generative"]:
        return "generative"

    def evaluate(self, conversation: Conversation, completion: str) -> bool:
        return grade_final_number(conversation, completion)


class SpellingBee(_Generated):
    ANSWER_RE = ANSWER_RE
    make = staticmethod(spelling_bee_example)

    def _extract_answer(self, text: str) -> str | None:
        return final_number(text)


class SimpleSpelling(_Generated):
    make = staticmethod(simple_spelling_example)

    def __init__(self, size: int = 1000, split: str = "train", words: list[str] | None = None) -> None:
        super().__init__(size, split, words)
        random.Random(42).shuffle(self.words)  # noqa: S311  (a fixed word order, as the reference's)


REGISTRY: dict[str, type] = {cls.__name__: cls for cls in
                             (ARC, MMLU, GSM8K, HumanEval, SmolTalk, CustomJSON, SpellingBee, SimpleSpelling)}
