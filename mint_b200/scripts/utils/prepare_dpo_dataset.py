"""``mint prepare-dpo``: convert anthropic/hh-rlhf into ``{prompt, chosen, rejected}`` JSONL rows
(scripts/utils/prepare_dpo_dataset.py)."""

from __future__ import annotations

import argparse
import re
from pathlib import Path

from mint_b200.data.dist.dpo import Message, Row


def parse_anthropic_chat(text: str) -> list[Message]:
    parts = re.split(r"\n\n(Human|Assistant):\s*", text)
    msgs = []
    for i in range(1, len(parts), 2):
        role = "user" if parts[i] == "Human" else "assistant"
        msgs.append(Message(role=role, content=parts[i + 1].strip() if i + 1 < len(parts) else ""))
    return msgs


def to_row(item: dict) -> Row:
    chosen = parse_anthropic_chat(item["chosen"])
    rejected = parse_anthropic_chat(item["rejected"])
    return Row(prompt=chosen[:-1], chosen=[chosen[-1]], rejected=[rejected[-1]])


def main() -> None:
    p = argparse.ArgumentParser(description="Prepare the hh-rlhf DPO dataset")
    p.add_argument("--output", type=str, default="data/dpo/hh_rlhf_formatted.jsonl")
    p.add_argument("--split", type=str, default="train[:1000]")
    args = p.parse_args()
    from datasets import load_dataset  # noqa: PLC0415

    ds = load_dataset("anthropic/hh-rlhf", split=args.split)
    out = Path(args.output)
    out.parent.mkdir(parents=True, exist_ok=True)
    with out.open("w", encoding="utf-8") as fh:
        for item in ds:
            fh.write(to_row(item).model_dump_json() + "\n")


if __name__ == "__main__":
    main()
