"""Pretraining task on the shared loop (reference behaviour: mint/trainer/pretrain.py:27-266).

Resume restores model, optimizer, step and this rank's dataloader cursor from the checkpoint's
``{"per_rank": {rank: state}}`` table (gathered to rank 0 when saving); evaluations are the
bits-per-byte validation loss (which also drives the best checkpoint) and the CORE benchmark; the
profiler records windows of optimizer steps.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import torch
import torch.distributed as dist
from torch import nn
from torch.optim import Optimizer

from mint_b200.eval.bpb import BPBEvaluator
from mint_b200.eval.dist.core import CoreEvaluator
from mint_b200.trainer.base import BasetrainConfig, BaseTrainer, Evaluation
from mint_b200.utils.device import Device
from mint_b200.utils.logger import logger
from mint_b200.utils.profiler import ProfilerConfig, StepProfiler


@dataclass
class PretrainConfig(BasetrainConfig):
    profiler: ProfilerConfig = field(default_factory=ProfilerConfig)


def flatten_metrics(prefix: str, value: Any, out: dict[str, Any] | None = None) -> dict[str, Any]:  # noqa: ANN401
    """``{"a": {"b": 1}}`` under ``prefix`` -> ``{"prefix/a/b": 1}``."""
    out = {} if out is None else out
    if isinstance(value, dict):
        for k, v in value.items():
            flatten_metrics(f"{prefix}/{k}", v, out)
    else:
        out[prefix] = value
    return out


class PreTrainer(BaseTrainer):
    def __init__(self, model: nn.Module, optimizer: Optimizer, dataloader: Any, device: Device,  # noqa: ANN401
                 config: PretrainConfig, tokenizer: Any = None, core_bundle_dir: str | None = None) -> None:  # noqa: ANN401
        super().__init__(model, optimizer, dataloader, device, config, tokenizer)
        self.bpb_evaluator = BPBEvaluator(model=model, config=config.eval, device=device, dataloader=dataloader)
        self.core_evaluator = self._make_core(core_bundle_dir)
        self.profiler = StepProfiler(config.profiler)
        self.resume_state: dict = {}
        if config.ckpt.resume_from_checkpoint:
            self.resume()

    def _make_core(self, bundle_dir: str | None) -> CoreEvaluator | None:
        if self.tokenizer is None:
            return None
        kw = {"bundle_dir": bundle_dir} if bundle_dir else {}
        try:
            return CoreEvaluator(model=self.model, config=self.config.eval, tokenizer=self.tokenizer,
                                 device=self.device, **kw)
        except FileNotFoundError:
            logger.warning("CORE eval bundle not found; CORE evaluation disabled")
            return None

    # ------------------------------------------------------------------ resume / dataloader state
    def resume(self) -> None:
        src = self.config.ckpt.resume_from_checkpoint
        info = self.checkpointer.load_checkpoint(model=self.model, optimizer=self.optimizer,
                                                 checkpoint_path=src if isinstance(src, str) else None,
                                                 load_best=self.config.ckpt.load_best_checkpoint)
        self.start_step = info["step"]
        self.resume_state = self.rank_state(info.get("dataloader_state", {}))
        if self.resume_state and hasattr(self.dataloader, "set_state"):
            self.dataloader.set_state(self.resume_state)
        logger.info(f"Resuming training from step {self.start_step}")

    def rank_state(self, saved: dict) -> dict:
        """This rank's dataloader state from a checkpoint (a single-process state is used as is)."""
        if not saved:
            return {}
        table = saved.get("per_rank")
        if table is None:
            return saved
        rank = self.process_info["rank"] if self.process_info["distributed"] else 0
        return table.get(rank, table.get(str(rank), {}))

    def dataloader_state(self) -> dict:
        """Collective under distribution: every rank's cursor, gathered to rank 0."""
        local = self.dataloader.get_state() if hasattr(self.dataloader, "get_state") else {}
        if not self.process_info["distributed"]:
            return local
        gathered: list[dict] | None = [{} for _ in range(self.process_info["world_size"])] if self.is_main_process else None
        dist.gather_object(local, gathered, dst=0)
        return {"per_rank": dict(enumerate(gathered))} if gathered is not None else {}

    # ------------------------------------------------------------------ task
    def micro_batches(self) -> Any:  # noqa: ANN401
        return self.dataloader.batch_loader(split="train", resume_state=self.resume_state or None)

    def evaluations(self) -> list[Evaluation]:
        evs = [Evaluation("val", self.config.eval_every_n_steps, self._validate)]
        if self.core_evaluator is not None:
            evs.append(Evaluation("core", self.config.core_eval_every_n_step, self._core))
        return evs

    def _evaluate(self, evaluator: Any, prefix: str, step: int, **kw: Any) -> dict[str, Any]:  # noqa: ANN401
        self.model.eval()
        with torch.no_grad():
            results = evaluator.evaluate(**kw)
        self.model.train()
        metrics = flatten_metrics(prefix, results)
        if self.is_main_process:
            logger.info(f"Eval step={step} | " + " | ".join(f"{k}={v:.4f}" for k, v in metrics.items()
                                                            if isinstance(v, (int, float))))
        self.sink.log(metrics, step=step)
        return results

    def _validate(self, step: int) -> None:
        results = self._evaluate(self.bpb_evaluator, "val", step, num_steps=self.config.eval_num_steps)
        val_loss = results.get("loss")
        if val_loss is not None:
            best = self.checkpointer.should_checkpoint_on_eval(val_loss)
            self.save(step, val_loss=val_loss, is_best=best)
        if hasattr(self.dataloader, "sample"):
            self.log_sample_predictions(self.dataloader.sample(num_samples=3))

    def _core(self, step: int) -> None:
        self._evaluate(self.core_evaluator, "core", step, task_labels=["hellaswag_zeroshot"], limit=1)

    # ------------------------------------------------------------------ profiler around the loop
    def after_step(self, step: int, metrics: dict) -> None:  # noqa: ARG002
        self.profiler.step()

    def train(self) -> None:
        with self.profiler:
            super().train()
