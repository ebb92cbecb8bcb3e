"""Direct Preference Optimization on the shared loop (reference behaviour: mint/trainer/dpo.py:25-288).

Each micro-batch's chosen and rejected sequences run through the policy as ONE batch (concatenated
on the batch dimension) with gradients, and through the frozen reference model without; summed
response log-probabilities feed the sigmoid DPO loss (``beta``, default 0.1).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch
from torch import nn
from torch.optim import Optimizer

from mint_b200.eval.dist.chatcore import ChatCoreEvaluator
from mint_b200.loss.dpo import DPOLoss, sequence_logps
from mint_b200.nn.base import LogitsWrapper
from mint_b200.trainer.base import BasetrainConfig, BaseTrainer, Evaluation
from mint_b200.utils.device import Device
from mint_b200.utils.logger import logger


@dataclass
class DPOConfig(BasetrainConfig):
    beta: float = 0.1


class DPOTrainer(BaseTrainer):
    def __init__(self, policy_model: nn.Module, optimizer: Optimizer, dataloader: Any, device: Device,  # noqa: ANN401
                 config: DPOConfig, reference_model: nn.Module, tokenizer: Any = None,  # noqa: ANN401
                 eval_datasets: list | None = None) -> None:
        super().__init__(policy_model, optimizer, dataloader, device, config, tokenizer)
        self.policy_model = LogitsWrapper(policy_model)
        self.reference_model = LogitsWrapper(reference_model)
        self.reference_model.eval()
        self.criterion = DPOLoss(beta=config.beta)
        self.evaluator = (ChatCoreEvaluator(model=policy_model, config=config.eval, tokenizer=tokenizer, device=device,
                                            datasets=eval_datasets) if eval_datasets else None)
        if config.ckpt.resume_from_checkpoint:
            src = config.ckpt.resume_from_checkpoint
            info = self.checkpointer.load_checkpoint(model=self.model, optimizer=self.optimizer,
                                                     checkpoint_path=src if isinstance(src, str) else None,
                                                     load_best=config.ckpt.load_best_checkpoint)
            self.start_step = info["step"]

    def pair_logps(self, model: nn.Module, ids: torch.Tensor, chosen: torch.Tensor,
                   rejected: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        logps = sequence_logps(model, ids, torch.cat([chosen, rejected], dim=0))
        return logps.chunk(2, dim=0)

    def micro_loss(self, batch: Any, step: int) -> tuple[torch.Tensor, int]:  # noqa: ANN401, ARG002
        ids = torch.cat([batch.chosen_input_ids, batch.rejected_input_ids], dim=0)
        with self.device.autocast():
            pol_c, pol_r = self.pair_logps(self.policy_model, ids, batch.chosen_labels, batch.rejected_labels)
            with torch.no_grad():
                ref_c, ref_r = self.pair_logps(self.reference_model, ids, batch.chosen_labels, batch.rejected_labels)
            loss, self.last_dpo_metrics = self.criterion(pol_c, pol_r, ref_c, ref_r)
        return loss / self.config.gradient_accumulation_steps, ids.numel()

    def evaluations(self) -> list[Evaluation]:
        return [Evaluation("chatcore", self.config.eval_every_n_steps, self._chatcore)] if self.evaluator else []

    def _chatcore(self, step: int) -> None:
        self.model.eval()
        with torch.no_grad():
            res = self.evaluator.evaluate(num_examples=100)
        self.model.train()
        if self.is_main_process:
            logger.info(f"eval step={step}: {res}")

    def train(self) -> None:
        self.reference_model.eval()
        super().train()
