"""Validation loss / bits-per-byte (mint/eval/bpb.py:13-79): masked CE over ``num_steps`` val batches,
dp all-reduce AVG, ``bpb = loss / ln 2`` (no bytes-per-token correction, as in the reference)."""

from __future__ import annotations

import math
import time
from typing import Any

import torch
import torch.distributed as dist
from torch import nn

from mint_b200.eval.base import EvalConfig, Evaluator
from mint_b200.ops.cross_entropy import masked_cross_entropy


class BPBEvaluator(Evaluator):
    def __init__(self, model: nn.Module, config: EvalConfig, device: Any, dataloader: Any) -> None:  # noqa: ANN401
        super().__init__(model, config, device)
        self.dataloader = dataloader

    def evaluate(self, num_steps: int = 10, _step: int | None = None) -> dict[str, Any]:
        self.model.eval()
        total_loss = torch.zeros((), dtype=torch.float32, device=self.device.device)
        total_tokens = torch.zeros((), dtype=torch.float32, device=self.device.device)
        t0 = time.perf_counter()
        done = 0
        vocab = getattr(getattr(self.model, "config", None), "vocab_size", None)
        with torch.no_grad():
            for i, (x, y, m, _d) in enumerate(self.dataloader.batch_loader(split="val")):
                if i >= num_steps:
                    break
                with self.device.autocast():
                    logits = self.model(x)
                    total_loss += masked_cross_entropy(logits, y, m, vocab if logits.size(-1) > (vocab or 0) else None)
                total_tokens += m.sum()
                done += 1
        self.device.synchronize()
        dt = time.perf_counter() - t0
        avg = (total_loss / max(done, 1))
        if self.process_info["dp_size"] > 1:
            dist.all_reduce(avg, op=dist.ReduceOp.SUM, group=self.device.parallel.dp_group)
            avg = avg / self.process_info["dp_size"]
        loss = float(avg)
        toks = float(total_tokens)
        return {"loss": loss, "bpb": loss / math.log(2), "eval_time_sec": dt,
                "tokens_per_second": toks * self.process_info["dp_size"] / dt if dt > 0 else 0.0}
