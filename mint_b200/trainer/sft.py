"""SFT loop (mint/trainer/sft.py:23-242): NaN/Inf checks, tokens counted from the loss mask,
ChatCORE evaluation; ``HFSFTTrainer`` wraps HuggingFace causal LMs."""

from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Any

import torch
from torch import nn
from torch.optim import Optimizer

from mint_b200.eval.dist.chatcore import ChatCoreEvaluator
from mint_b200.nn.base import LogitsWrapper
from mint_b200.trainer.base import BasetrainConfig, BaseTrainer
from mint_b200.trainer.scheduler import Scheduler
from mint_b200.utils.checkpointer import Checkpointer
from mint_b200.utils.device import Device
from mint_b200.utils.logger import logger


@dataclass
class SFTConfig(BasetrainConfig): ...


class SFTTrainer(BaseTrainer):
    def __init__(self, model: nn.Module, optimizer: Optimizer, dataloader: Any, device: Device, config: SFTConfig,  # noqa: ANN401
                 tokenizer: Any = None, eval_datasets: list | None = None) -> None:  # noqa: ANN401
        super().__init__(model=model, optimizer=optimizer, dataloader=dataloader, device=device, config=config,
                         tokenizer=tokenizer)
        self.checkpointer = Checkpointer(config=config.ckpt, is_main_process=self.is_main_process)
        self.scheduler = Scheduler(num_iterations=config.train_num_steps, config=config.sched)
        self.evaluator = (ChatCoreEvaluator(model=model, config=config.eval, tokenizer=tokenizer, device=device,
                                            datasets=eval_datasets) if eval_datasets else None)
        if config.ckpt.resume_from_checkpoint:
            self._load_pretrained_checkpoint()

    def _load_pretrained_checkpoint(self) -> None:
        path = self.config.ckpt.resume_from_checkpoint
        self.checkpointer.load_checkpoint(model=self.model, optimizer=self.optimizer,
                                          checkpoint_path=path if isinstance(path, str) else None,
                                          load_best=self.config.ckpt.load_best_checkpoint)
        bad = [n for n, p in self.model.named_parameters() if p.numel() and not torch.isfinite(p).all()]
        if bad:
            logger.error(f"non-finite parameters after loading checkpoint: {bad}")

    def _validate_batch(self, inputs: torch.Tensor, targets: torch.Tensor, step: int) -> None:  # noqa: ARG002
        if inputs.is_floating_point() and not torch.isfinite(inputs).all():
            logger.error(f"non-finite inputs at step {step}")

    def _forward_pass(self, inputs: torch.Tensor, doc_ids: torch.Tensor | None = None) -> torch.Tensor:  # noqa: ARG002
        logits = self.model(inputs)
        if torch.isnan(logits).any():
            logger.warning("NaN detected in logits")
        return logits

    def _run_evaluation(self, step: int, num_examples: int | None = None) -> None:
        if self.evaluator is None:
            return
        self.model.eval()
        with torch.no_grad():
            results = self.evaluator.evaluate(num_examples=num_examples)
        self.model.train()
        metrics = {}
        for k, v in results.items():
            if isinstance(v, dict):
                for sk, sv in v.items():
                    metrics[f"eval/{k}/{sk}"] = sv
            else:
                metrics[f"eval/{k}"] = v
        if self.is_main_process:
            logger.info(f"Eval step={step} | " + " | ".join(f"{k}={v}" for k, v in metrics.items()))
        self._log_wandb(metrics, step=step)

    def train(self) -> None:
        self.model.train()
        t0 = time.perf_counter()
        accum = self.config.gradient_accumulation_steps
        micro_step = 0
        acc_loss = 0.0
        for inputs, targets, loss_mask, _ in self.dataloader.batch_loader(split="train"):
            step = micro_step // accum
            if micro_step % accum == 0:
                if self._handle_interrupt(step, self.checkpointer) or step >= self.config.train_num_steps:
                    break
                self.timer.start()
                self.optimizer.zero_grad()
            last = (micro_step + 1) % accum == 0
            self.device.set_grad_sync(last)
            loss = self._compute_loss(inputs, targets, loss_mask, step)
            self.device.backward(loss)
            acc_loss += loss.item()
            micro_step += 1
            if not last:
                continue
            step = micro_step // accum
            sched = self.scheduler.step(self.optimizer, step)
            self._perform_optimization_step(micro_step, step, sched)
            dev_t, wall_t = self.timer.stop()
            tokens = int(loss_mask.sum().item()) * self.process_info["dp_size"] * accum
            metrics = self._calculate_step_metrics(acc_loss, wall_t, tokens, sched, t0, device_time=dev_t)
            if step % self.config.eval_every_n_steps == 0 and step > 0:
                self._run_evaluation(step=step, num_examples=self.config.eval_num_steps)
            self._maybe_save_checkpoint(step, self.checkpointer)
            self._log_training_progress(step, metrics)
            acc_loss = 0.0
        self._finalize_training(micro_step // accum, self.checkpointer)


class HFSFTTrainer(SFTTrainer):
    def __init__(self, model: nn.Module, optimizer: Optimizer, dataloader: Any, device: Device, config: SFTConfig,  # noqa: ANN401
                 tokenizer: Any = None, eval_datasets: list | None = None) -> None:  # noqa: ANN401
        super().__init__(model=LogitsWrapper(model), optimizer=optimizer, dataloader=dataloader, device=device,
                         config=config, tokenizer=tokenizer, eval_datasets=eval_datasets)

    def _forward_pass(self, inputs: torch.Tensor, doc_ids: torch.Tensor | None = None) -> torch.Tensor:  # noqa: ARG002
        return self.model(input_ids=inputs)

    def train(self) -> None:
        for g in self.optimizer.param_groups:
            g.setdefault("initial_lr", g["lr"])
        super().train()
