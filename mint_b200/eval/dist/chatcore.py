"""ChatCORE: generate a completion per example and grade it with the dataset's ``evaluate``
(mint/eval/dist/chatcore.py:16-102). ``Gemma.generate`` accepts the HF-style kwargs used here."""

from __future__ import annotations

import copy
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

    def evaluate(self, num_examples: int | None = None) -> dict[str, Any]:
        self.model.eval()
        t0 = time.perf_counter()
        results = {}
        with torch.no_grad():
            for ds in self.datasets:
                results[ds.__class__.__name__] = self._evaluate_dataset(ds, num_examples)
        self.device.synchronize()
        dt = time.perf_counter() - t0
        if not results:
            return {"tasks": {}, "accuracy": 0.0, "eval_time_sec": dt}
        return {"tasks": results, "accuracy": sum(r["accuracy"] for r in results.values()) / len(results),
                "eval_time_sec": dt}

    def _evaluate_dataset(self, dataset: Any, num_examples: int | None = None) -> dict[str, Any]:  # noqa: ANN401
        total = len(dataset) if num_examples is None else min(num_examples, len(dataset))
        rank, world = self.process_info["dp_rank"], self.process_info["dp_size"]
        correct = count = 0
        for i in range(rank, total, world):
            conv = dataset[i]
            if dataset.evaluate(conv, self._generate_completion(conv)):
                correct += 1
            count += 1
        if world > 1:
            t = torch.tensor([correct, count], dtype=torch.float32, device=self.device.device)
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.device.parallel.dp_group)
            correct, count = t[0].item(), t[1].item()
        return {"accuracy": correct / count if count else 0.0, "num_examples": int(count)}

    def _generate_completion(self, conversation: dict) -> str:
        conversation = copy.deepcopy(conversation)
        conversation["messages"].pop()
        ids, _ = self.tokenizer.render_conversation(conversation, self.config.seq_length - 1)
        ids.append(self.tokenizer.encode_special("<|assistant_start|>"))
        inp = torch.tensor([ids], dtype=torch.long, device=self.device.device)
        with self.device.autocast():
            out = self.model.generate(inp, attention_mask=torch.ones_like(inp), pad_token_id=self.tokenizer.pad_token,
                                      max_new_tokens=self.config.max_new_tokens,
                                      eos_token_id=self.tokenizer.encode_special("<|assistant_end|>"),
                                      do_sample=False, use_cache=True)
        return self.tokenizer.decode(out[0, inp.shape[1] :].cpu())[0]
