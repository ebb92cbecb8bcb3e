"""ChatCORE: generative accuracy of a chat model on SFT eval datasets.

Same contract as the reference evaluator (mint/eval/dist/chatcore.py:16-102): each example's last
(assistant) message is dropped, the rest is rendered with the chat template, the model continues
greedily after ``<|assistant_start|>`` until ``<|assistant_end|>`` or ``max_new_tokens``, and the
dataset's ``evaluate(conversation, completion)`` grades the text; examples are dealt to the data-
parallel ranks round-robin and the result is ``{"tasks": {name: {"accuracy", "num_examples"}},
"accuracy": mean over tasks, "eval_time_sec"}``.

Organisation: every rank fills one ``[tasks, 2]`` tally (correct, graded) and the tallies of all
tasks are summed across the dp group in a single all-reduce at the end; prompts are built by
``prompt_ids`` and decoded by ``complete``, so a caller can grade one example without a dataset.
"""

from __future__ import annotations

import time
from typing import Any

import torch
import torch.distributed as dist
from torch import nn

from mint_b200.eval.base import EvalConfig, Evaluator
from mint_b200.nn.base import LogitsWrapper


class ChatCoreEvaluator(Evaluator):
    def __init__(self, model: nn.Module, config: EvalConfig, tokenizer: Any, device: Any, datasets: list) -> None:  # noqa: ANN401
        super().__init__(LogitsWrapper(model), config, device)
        self.tokenizer = tokenizer
        self.datasets = datasets

    # ------------------------------------------------------------------ one example
    def prompt_ids(self, conversation: dict[str, Any]) -> list[int]:
        """Chat-rendered history without the reference answer, ending in ``<|assistant_start|>``."""
        history = {**conversation, "messages": list(conversation["messages"][:-1])}
        ids, _mask = self.tokenizer.render_conversation(history, self.config.seq_length - 1)
        return [*ids, self.tokenizer.encode_special("<|assistant_start|>")]

    @torch.no_grad()
    def complete(self, conversation: dict[str, Any]) -> str:
        ids = self.prompt_ids(conversation)
        prompt = torch.tensor([ids], dtype=torch.long, device=self.device.device)
        stop = self.tokenizer.encode_special("<|assistant_end|>")
        with self.device.autocast():
            out = self.model.generate(prompt, attention_mask=torch.ones_like(prompt),
                                      pad_token_id=self.tokenizer.pad_token, max_new_tokens=self.config.max_new_tokens,
                                      eos_token_id=stop, do_sample=False, use_cache=True)
        return self.tokenizer.decode(out[0, len(ids):].cpu())[0]

    # ------------------------------------------------------------------ datasets
    def _share(self, dataset: Any, limit: int | None) -> range:  # noqa: ANN401
        total = len(dataset) if limit is None else min(limit, len(dataset))
        return range(self.process_info["dp_rank"], total, self.process_info["dp_size"])

    def evaluate(self, num_examples: int | None = None) -> dict[str, Any]:
        self.model.eval()
        t0 = time.perf_counter()
        names = [type(ds).__name__ for ds in self.datasets]
        tally = torch.zeros(len(self.datasets), 2, dtype=torch.float64)
        with torch.no_grad():
            for k, ds in enumerate(self.datasets):
                for idx in self._share(ds, num_examples):
                    conv = ds[idx]
                    tally[k, 0] += float(bool(ds.evaluate(conv, self.complete(conv))))
                    tally[k, 1] += 1.0
        tally = self._sum_over_dp(tally)
        self.device.synchronize()
        tasks = {name: {"accuracy": float(c / n) if n > 0 else 0.0, "num_examples": int(n)}
                 for name, (c, n) in zip(names, tally.tolist(), strict=True)}
        mean = sum(t["accuracy"] for t in tasks.values()) / len(tasks) if tasks else 0.0
        return {"tasks": tasks, "accuracy": mean, "eval_time_sec": time.perf_counter() - t0}

    def _sum_over_dp(self, tally: torch.Tensor) -> torch.Tensor:
        if self.process_info["dp_size"] <= 1 or tally.numel() == 0:
            return tally
        t = tally.to(self.device.device, torch.float32)
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.device.parallel.dp_group)
        return t.double().cpu()
