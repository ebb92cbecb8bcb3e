"""Pretraining loop (mint/trainer/pretrain.py:27-266): resume (step + per-rank dataloader state),
gradient accumulation, BPB eval + best checkpoint, CORE eval, profiler stepping, device-timed tok/s."""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Any

import torch
import torch.distributed as dist
from torch import nn
from torch.optim import Optimizer

from mint_b200.eval.bpb import BPBEvaluator
from mint_b200.eval.dist.core import CoreEvaluator
from mint_b200.trainer.base import BasetrainConfig, BaseTrainer
from mint_b200.trainer.scheduler import Scheduler
from mint_b200.utils.checkpointer import Checkpointer
from mint_b200.utils.device import Device
from mint_b200.utils.logger import logger
from mint_b200.utils.profiler import ProfilerConfig, TorchProfiler


@dataclass
class PretrainConfig(BasetrainConfig):
    profiler: ProfilerConfig = field(default_factory=ProfilerConfig)


class PreTrainer(BaseTrainer):
    def __init__(self, model: nn.Module, optimizer: Optimizer, dataloader: Any, device: Device,  # noqa: ANN401
                 config: PretrainConfig, tokenizer: Any = None, core_bundle_dir: str | None = None) -> None:  # noqa: ANN401
        super().__init__(model=model, optimizer=optimizer, dataloader=dataloader, device=device, config=config,
                         tokenizer=tokenizer)
        self.checkpointer = Checkpointer(config=config.ckpt, is_main_process=self.is_main_process)
        self.scheduler = Scheduler(num_iterations=config.train_num_steps, config=config.sched)
        self.core_evaluator = None
        if tokenizer is not None:
            try:
                self.core_evaluator = CoreEvaluator(model=model, config=config.eval, tokenizer=tokenizer,
                                                    device=device, **({"bundle_dir": core_bundle_dir} if core_bundle_dir else {}))
            except FileNotFoundError:
                logger.warning("CORE eval bundle not found; CORE evaluation disabled")
        self.bpb_evaluator = BPBEvaluator(model=model, config=config.eval, device=device, dataloader=dataloader)
        self.start_step = 0
        self.dataloader_state: dict = {}
        if config.ckpt.resume_from_checkpoint:
            self._load_pretrained_checkpoint()
        self.profiler = TorchProfiler(config.profiler)
        self.last_metrics: dict = {}

    def _load_pretrained_checkpoint(self) -> None:
        path = self.config.ckpt.resume_from_checkpoint
        info = self.checkpointer.load_checkpoint(model=self.model, optimizer=self.optimizer,
                                                 checkpoint_path=path if isinstance(path, str) else None,
                                                 load_best=self.config.ckpt.load_best_checkpoint)
        self.start_step = info["step"]
        self.dataloader_state = self._extract_rank_dataloader_state(info.get("dataloader_state", {}))
        if self.dataloader_state and hasattr(self.dataloader, "set_state"):
            self.dataloader.set_state(self.dataloader_state)
        logger.info(f"Resuming training from step {self.start_step}")

    def _local_dataloader_state(self) -> dict:
        return self.dataloader.get_state() if hasattr(self.dataloader, "get_state") else {}

    def _get_dataloader_state(self) -> dict:
        local = self._local_dataloader_state()
        if not self.process_info["distributed"]:
            return local
        if self.is_main_process:
            gathered: list[dict] = [{} for _ in range(self.process_info["world_size"])]
            dist.gather_object(local, gathered, dst=0)
            return {"per_rank": dict(enumerate(gathered))}
        dist.gather_object(local, None, dst=0)
        return {}

    def _extract_rank_dataloader_state(self, state: dict) -> dict:
        if not state:
            return {}
        if not self.process_info["distributed"]:
            return state.get("per_rank", {}).get(0, state) if "per_rank" in state else state
        per = state.get("per_rank", {})
        return per.get(self.process_info["rank"], per.get(str(self.process_info["rank"]), {}))

    def _run_evaluation(self, evaluator: Any, step: int, metric_prefix: str, *, save_checkpoint: bool = False,  # noqa: ANN401
                        **eval_kwargs: Any) -> dict[str, Any]:  # noqa: ANN401
        self.model.eval()
        with torch.no_grad():
            results = evaluator.evaluate(**eval_kwargs)
        self.model.train()
        metrics: dict[str, Any] = {}

        def flatten(prefix: str, value: Any) -> None:  # noqa: ANN401
            if isinstance(value, dict):
                for k, v in value.items():
                    flatten(f"{prefix}/{k}", v)
            else:
                metrics[prefix] = value

        for k, v in results.items():
            flatten(f"{metric_prefix}/{k}", v)
        if self.is_main_process:
            logger.info(f"Eval step={step} | " + " | ".join(f"{k}={v:.4f}" for k, v in metrics.items()
                                                            if isinstance(v, (int, float))))
        self._log_wandb(metrics, step=step)
        val_loss = results.get("loss") if save_checkpoint else None
        if val_loss is not None:
            state = self._get_dataloader_state()
            is_best = self.checkpointer.should_checkpoint_on_eval(val_loss)
            self.checkpointer.save_checkpoint(step=step, model=self.model, optimizer=self.optimizer,
                                              dataloader_state=state, val_loss=val_loss, is_best=is_best)
        return results

    def train(self) -> None:
        self.model.train()
        t_train0 = time.perf_counter()
        accum = self.config.gradient_accumulation_steps
        micro_step = self.start_step * accum
        acc_loss: Any = 0.0
        batches = self.dataloader.batch_loader(split="train", resume_state=self.dataloader_state or None)
        with self.profiler:
            for inputs, targets, loss_mask, doc_ids in batches:
                step = micro_step // accum
                if micro_step % accum == 0:
                    if self._handle_interrupt(step, self.checkpointer) or step >= self.config.train_num_steps:
                        break
                    self.timer.start()
                    self.optimizer.zero_grad()
                last = (micro_step + 1) % accum == 0
                self.device.set_grad_sync(last)
                loss = self._compute_loss(inputs, targets, loss_mask, step, doc_ids)
                self.device.backward(loss)
                acc_loss = acc_loss + loss.detach()
                micro_step += 1
                if not last:
                    continue
                step = micro_step // accum
                sched = self.scheduler.step(self.optimizer, step)
                self._perform_optimization_step(micro_step, step, sched)
                dev_t, wall_t = self.timer.stop()
                acc_loss = float(acc_loss)
                tokens = targets.numel() * self.process_info["dp_size"] * accum
                metrics = self._calculate_step_metrics(acc_loss, wall_t, tokens, sched, t_train0, device_time=dev_t)
                self.last_metrics = metrics
                if step % self.config.eval_every_n_steps == 0 and step > 0:
                    self._run_evaluation(self.bpb_evaluator, step, "val", save_checkpoint=True,
                                         num_steps=self.config.eval_num_steps)
                    self._log_sample_predictions(step)
                if self.core_evaluator is not None and step % self.config.core_eval_every_n_step == 0 and step > 0:
                    self._run_evaluation(self.core_evaluator, step, "core", task_labels=["hellaswag_zeroshot"], limit=1)
                self._maybe_save_checkpoint(step, self.checkpointer)
                self._log_training_progress(step, metrics)
                self.profiler.step()
                acc_loss = 0.0
        self._finalize_training(micro_step // accum, self.checkpointer)
