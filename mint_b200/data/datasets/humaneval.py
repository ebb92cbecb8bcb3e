"""HumanEval, graded by executing the completion against the tests (mint/data/datasets/humaneval.py:10-58)."""

from __future__ import annotations

import re
from typing import Any, Literal

from mint_b200.data.datasets.base import SFTEvalDataset, SFTTrainDataset, hf_load
from mint_b200.utils.exec import execute_code


class HumanEval(SFTTrainDataset, SFTEvalDataset):
    def __init__(self, ds: Any = None) -> None:  # noqa: ANN401
        super().__init__()
        self.ds = ds if ds is not None else hf_load("openai/openai_humaneval", split="test")

    @property
    def eval_type(self) -> Literal["categorical", "generative"]:
        return "generative"

    def __len__(self) -> int:
        return len(self.ds)

    def __getitem__(self, index: int) -> dict[str, Any]:
        row = self.ds[index]
        return {
            "messages": [{"role": "user", "content": row["prompt"]},
                         {"role": "assistant", "content": f"{row['prompt']}\n{row['canonical_solution']}"}],
            "entry_point": row["entry_point"],
            "test": row["test"],
        }

    def evaluate(self, conversation: dict[str, Any], completion: str) -> bool:
        imports = self._extract_imports(conversation["messages"][0]["content"])
        code = self._extract_code(completion)
        program = f"{imports}\n\n{code}\n\n{conversation['test']}\ncheck({conversation['entry_point']})"
        return execute_code(program).success

    @staticmethod
    def _extract_imports(prompt: str) -> str:
        out = []
        for line in prompt.split("\n"):
            s = line.strip()
            if s.startswith(("import ", "from ")):
                out.append(s)
            elif s and not s.startswith("#"):
                break
        return "\n".join(out)

    @staticmethod
    def _extract_code(completion: str) -> str:
        found = re.findall(r"```(?:python)?\s*\n(.*?)\n```", completion, re.DOTALL)
        return found[0].strip() if found else completion.strip()
