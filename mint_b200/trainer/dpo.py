"""DPO loop (mint/trainer/dpo.py:25-288): chosen and rejected concatenated on the batch dim,
policy forward with grad, frozen reference forward without, sigmoid DPO loss."""

from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Any

import torch
from torch import nn
from torch.optim import Optimizer

from mint_b200.eval.dist.chatcore import ChatCoreEvaluator
from mint_b200.loss.dpo import DPOLoss, compute_logps
from mint_b200.nn.base import LogitsWrapper
from mint_b200.trainer.base import BasetrainConfig, BaseTrainer
from mint_b200.trainer.scheduler import Scheduler
from mint_b200.utils.checkpointer import Checkpointer
from mint_b200.utils.device import Device
from mint_b200.utils.logger import logger


@dataclass
class DPOConfig(BasetrainConfig):
    beta: float = 0.1


class DPOTrainer(BaseTrainer):
    def __init__(self, policy_model: nn.Module, optimizer: Optimizer, dataloader: Any, device: Device,  # noqa: ANN401
                 config: DPOConfig, reference_model: nn.Module, tokenizer: Any = None,  # noqa: ANN401
                 eval_datasets: list | None = None) -> None:
        super().__init__(model=policy_model, optimizer=optimizer, dataloader=dataloader, device=device, config=config,
                         tokenizer=tokenizer)
        self.policy_model = LogitsWrapper(policy_model)
        self.reference_model = LogitsWrapper(reference_model)
        self.checkpointer = Checkpointer(config=config.ckpt, is_main_process=self.is_main_process)
        self.scheduler = None
        if getattr(config, "sched", None) is not None:
            self.scheduler = Scheduler(num_iterations=config.train_num_steps, config=config.sched)
            for g in optimizer.param_groups:
                g["initial_lr"] = g["lr"]
        self.criterion = DPOLoss(beta=getattr(config, "beta", 0.1))
        self.evaluator = (ChatCoreEvaluator(model=policy_model, config=config.eval, tokenizer=tokenizer, device=device,
                                            datasets=eval_datasets) if eval_datasets else None)
        if config.ckpt.resume_from_checkpoint:
            path = config.ckpt.resume_from_checkpoint
            self.checkpointer.load_checkpoint(model=self.model, optimizer=self.optimizer,
                                              checkpoint_path=path if isinstance(path, str) else None,
                                              load_best=config.ckpt.load_best_checkpoint)
        self.last_metrics: dict = {}

    def _forward_pass(self, inputs: torch.Tensor, doc_ids: torch.Tensor | None = None) -> torch.Tensor:  # noqa: ARG002
        return self.model(inputs)

    def _compute_dpo_loss(self, concat_ids: torch.Tensor, concat_mask: torch.Tensor,  # noqa: ARG002
                          c_labels: torch.Tensor, r_labels: torch.Tensor) -> tuple[torch.Tensor, dict]:
        with self.device.autocast():
            pol = self.policy_model(concat_ids)
            pc, pr = pol.chunk(2, dim=0)
            p_c, p_r = compute_logps(pc, c_labels), compute_logps(pr, r_labels)
            with torch.no_grad():
                ref = self.reference_model(concat_ids)
                rc, rr = ref.chunk(2, dim=0)
                r_c, r_r = compute_logps(rc, c_labels), compute_logps(rr, r_labels)
            loss, metrics = self.criterion(p_c, p_r, r_c, r_r)
        return loss / self.config.gradient_accumulation_steps, metrics

    def train(self) -> None:
        self.policy_model.train()
        self.reference_model.eval()
        t0 = time.perf_counter()
        accum = self.config.gradient_accumulation_steps
        micro_step = 0
        acc_loss = 0.0
        for batch in self.dataloader.batch_loader(split="train"):
            step = micro_step // accum
            if micro_step % accum == 0:
                if self._handle_interrupt(step, self.checkpointer) or step >= self.config.train_num_steps:
                    break
                self.timer.start()
                self.optimizer.zero_grad()
            concat_ids = torch.cat([batch.chosen_input_ids, batch.rejected_input_ids], dim=0)
            concat_mask = torch.cat([batch.chosen_attn_mask, batch.rejected_attn_mask], dim=0)
            last = (micro_step + 1) % accum == 0
            self.device.set_grad_sync(last)
            loss, _m = self._compute_dpo_loss(concat_ids, concat_mask, batch.chosen_labels, batch.rejected_labels)
            self.device.backward(loss)
            acc_loss += loss.item()
            micro_step += 1
            if not last:
                continue
            step = micro_step // accum
            sched = self.scheduler.step(self.optimizer, step) if self.scheduler is not None else {}
            self._perform_optimization_step(micro_step, step, sched)
            dev_t, wall_t = self.timer.stop()
            tokens = concat_ids.numel() * self.process_info["dp_size"] * accum
            metrics = self._calculate_step_metrics(acc_loss, wall_t, tokens, sched, t0, device_time=dev_t)
            self.last_metrics = metrics
            if self.evaluator is not None and step % self.config.eval_every_n_steps == 0 and step > 0:
                self.model.eval()
                with torch.no_grad():
                    res = self.evaluator.evaluate(num_examples=100)
                self.model.train()
                if self.is_main_process:
                    logger.info(f"eval step={step}: {res}")
            self._maybe_save_checkpoint(step, self.checkpointer)
            self._log_training_progress(step, metrics)
            acc_loss = 0.0
        self._finalize_training(micro_step // accum, self.checkpointer)
