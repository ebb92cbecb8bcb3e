"""CORE in-context-learning evaluation (mint/eval/dist/core.py:16-295).

Eval-bundle tasks (``core.yaml``): multiple choice and schema tasks pick the option with the
lowest mean continuation loss; language-modeling tasks require an exact greedy match. Few-shot
examples are sampled with ``random.Random(seed + idx)``; examples are strided over dp ranks and
the per-example correctness vector is SUM all-reduced.
"""

from __future__ import annotations

import json
import random
import time
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist
import yaml
from torch import nn

from mint_b200.eval.base import EvalConfig, Evaluator, Task


class CoreEvaluator(Evaluator):
    def __init__(self, model: nn.Module, config: EvalConfig, tokenizer: Any, device: Any,  # noqa: ANN401
                 bundle_dir: str = "data/eval_bundle", config_path: str | None = None, seed: int = 42) -> None:
        super().__init__(model, config, device)
        self.tokenizer = tokenizer
        self.bundle_dir = Path(bundle_dir)
        self.config_path = Path(config_path) if config_path else self.bundle_dir / "core.yaml"
        self.seed = seed
        self.pad_token_id = getattr(tokenizer, "pad_token", None)
        if self.pad_token_id is None:
            raise ValueError("tokenizer.pad_token is required")
        if not self.config_path.exists():
            raise FileNotFoundError(self.config_path)
        with self.config_path.open() as fh:
            self.tasks = (yaml.safe_load(fh) or {}).get("icl_tasks", [])

    def evaluate(self, task_labels: list[str] | None = None, limit: int | None = None) -> dict[str, Any]:
        self.model.eval()
        t0 = time.perf_counter()
        tasks = self.tasks if task_labels is None else [t for t in self.tasks if t["label"] in set(task_labels)]
        results = {}
        with torch.no_grad():
            for task in tasks:
                results[task["label"]] = self.evaluate_task(task, limit=limit)
        self.device.synchronize()
        dt = time.perf_counter() - t0
        if not results:
            return {"tasks": {}, "core": 0.0, "eval_time_sec": dt, "tokens_per_second": 0.0}
        n = sum(r["num_examples"] for r in results.values())
        return {"tasks": results, "core": sum(r["accuracy"] for r in results.values()) / len(results),
                "eval_time_sec": dt, "tokens_per_second": n * self.process_info["dp_size"] / dt if dt > 0 else 0.0}

    def evaluate_task(self, task_meta: dict, limit: int | None = None) -> dict[str, Any]:
        data = self._load_dataset(task_meta["dataset_uri"])
        if limit is not None:
            data = data[:limit]
        rank, world = self.process_info["dp_rank"], self.process_info["dp_size"]
        correct = torch.zeros(len(data), dtype=torch.float32, device=self.device.device)
        for i in range(rank, len(data), world):
            correct[i] = float(self.evaluate_example(i, data, task_meta))
        if world > 1:
            dist.all_reduce(correct, op=dist.ReduceOp.SUM, group=self.device.parallel.dp_group)
        return {"accuracy": correct.mean().item() if len(data) else 0.0, "num_examples": len(data)}

    def evaluate_example(self, idx: int, data: list[dict], task_meta: dict) -> bool:
        item = data[idx]
        shots = self._sample_fewshot(idx, data, task_meta)
        kind = Task(task_meta["icl_task_type"])
        delim = task_meta.get("continuation_delimiter", " ")
        if kind in (Task.MC, Task.SCHEMA):
            if kind == Task.MC:
                fulls, prefixes = self._render_multiple_choice(item, shots, delim), \
                    self._render_multiple_choice_prefixes(item, shots, delim)
            else:
                fulls, prefixes = self._render_schema(item, shots, delim), self._render_schema_prefixes(item, shots, delim)
            full_t = self._encode_prompts(fulls)
            pre_t = self._encode_prompts(prefixes)
            losses = [self._continuation_mean_loss(f, len(p)) for f, p in zip(full_t, pre_t, strict=False)]
            return min(range(len(losses)), key=lambda i: losses[i]) == item["gold"]
        prompt, full = self._render_language_modeling(item, shots, delim)
        return self._language_model_exact_match(self._encode_single(full), len(self._encode_single(prompt)))

    def _load_dataset(self, uri: str) -> list[dict]:
        with (self.bundle_dir / "eval_data" / uri).open() as fh:
            return [json.loads(line) for line in fh if line.strip()]

    def _sample_fewshot(self, idx: int, data: list[dict], task_meta: dict) -> list[dict]:
        vals = task_meta.get("num_fewshot", [0])
        k = vals[0] if vals else 0
        if k <= 0:
            return []
        if task_meta.get("has_categories") and "category" in data[idx]:
            cat = data[idx]["category"]
            cand = [i for i, r in enumerate(data) if i != idx and r.get("category") == cat]
        else:
            cand = [i for i in range(len(data)) if i != idx]
        if not cand:
            return []
        rng = random.Random(self.seed + idx)  # noqa: S311
        return [data[i] for i in rng.sample(cand, min(k, len(cand)))]

    def _mc_prefix(self, item: dict, shots: list[dict], delim: str) -> str:
        parts = [f"{e['query']}{delim}{e['choices'][e['gold']]}" for e in shots]
        parts.append(f"{item['query']}{delim}")
        return "\n\n".join(parts)

    def _render_multiple_choice(self, item: dict, shots: list[dict], delim: str) -> list[str]:
        pre = self._mc_prefix(item, shots, delim)
        return [pre + c for c in item["choices"]]

    def _render_multiple_choice_prefixes(self, item: dict, shots: list[dict], delim: str) -> list[str]:
        return [self._mc_prefix(item, shots, delim) for _ in item["choices"]]

    def _schema_shots(self, shots: list[dict], delim: str) -> str:
        return "\n\n".join(f"{e['context_options'][e['gold']]}{delim}{e['continuation']}" for e in shots)

    def _render_schema(self, item: dict, shots: list[dict], delim: str) -> list[str]:
        pre = self._schema_shots(shots, delim)
        suffix = f"{delim}{item['continuation']}"
        return [f"{pre}\n\n{o}{suffix}" if pre else f"{o}{suffix}" for o in item["context_options"]]

    def _render_schema_prefixes(self, item: dict, shots: list[dict], delim: str) -> list[str]:
        pre = self._schema_shots(shots, delim)
        return [f"{pre}\n\n{o}{delim}" if pre else f"{o}{delim}" for o in item["context_options"]]

    def _render_language_modeling(self, item: dict, shots: list[dict], delim: str) -> tuple[str, str]:
        parts = [f"{e['context'].rstrip()}{delim}{e['continuation']}" for e in shots]
        prefix = f"{item['context'].rstrip()}{delim}"
        prompt = "\n\n".join([*parts, prefix]) if parts else prefix
        return prompt, prompt + item["continuation"]

    def _encode_prompts(self, prompts: list[str]) -> list[list[int]]:
        return self.tokenizer.encode_to_list(prompts, add_bos=True, add_eos=False, padding=False)

    def _encode_single(self, text: str) -> list[int]:
        return self.tokenizer.encode_to_list([text], add_bos=True, add_eos=False, padding=False)[0]

    def _forward(self, tokens: list[int]) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        tokens = tokens[-int(self.config.seq_length):]
        ids = torch.tensor([tokens], dtype=torch.long, device=self.device.device)
        with self.device.autocast():
            logits = self.model(ids)
        sl, st = logits[:, :-1].float(), ids[:, 1:]
        losses = torch.nn.functional.cross_entropy(sl.reshape(-1, sl.size(-1)), st.reshape(-1), reduction="none")
        return ids, losses, sl.argmax(dim=-1)[0]

    def _crop(self, full: list[int], plen: int) -> tuple[list[int], int]:
        mx = int(self.config.seq_length)
        if len(full) > mx:
            crop = len(full) - mx
            return full[crop:], max(0, plen - crop)
        return full, plen

    def _continuation_mean_loss(self, full: list[int], plen: int) -> float:
        full, plen = self._crop(full, plen)
        if plen >= len(full):
            return float("inf")
        _, losses, _ = self._forward(full)
        span = losses[max(plen - 1, 0) : len(full) - 1]
        return span.mean().item() if span.numel() else float("inf")

    def _language_model_exact_match(self, full: list[int], plen: int) -> bool:
        full, plen = self._crop(full, plen)
        if plen >= len(full):
            return False
        ids, _, pred = self._forward(full)
        s, e = max(plen - 1, 0), len(full) - 1
        p = pred[s:e]
        return bool(p.numel()) and bool(torch.equal(p, ids[0, s + 1 : e + 1]))
