"""Supervised fine-tuning tasks on the shared loop (reference behaviour: mint/trainer/sft.py:23-242).

``SFTTrainer``: chat-rendered conversations with an assistant-token loss mask; tokens per step are
counted from the mask; ChatCORE evaluation on the given eval datasets; non-finite inputs, logits and
loaded parameters are reported. ``HFSFTTrainer``: the same task for a HuggingFace causal LM (its
``.logits`` are unwrapped and it is called with ``input_ids=``).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch
from torch import nn
from torch.optim import Optimizer

from mint_b200.eval.dist.chatcore import ChatCoreEvaluator
from mint_b200.nn.base import LogitsWrapper
from mint_b200.ops.cross_entropy import masked_cross_entropy
from mint_b200.trainer.base import BasetrainConfig, BaseTrainer, Evaluation
from mint_b200.utils.device import Device
from mint_b200.utils.logger import logger


@dataclass
class SFTConfig(BasetrainConfig): ...


class SFTTrainer(BaseTrainer):
    def __init__(self, model: nn.Module, optimizer: Optimizer, dataloader: Any, device: Device, config: SFTConfig,  # noqa: ANN401
                 tokenizer: Any = None, eval_datasets: list | None = None) -> None:  # noqa: ANN401
        super().__init__(model, optimizer, dataloader, device, config, tokenizer)
        self.evaluator = (ChatCoreEvaluator(model=model, config=config.eval, tokenizer=tokenizer, device=device,
                                            datasets=eval_datasets) if eval_datasets else None)
        if config.ckpt.resume_from_checkpoint:
            src = config.ckpt.resume_from_checkpoint
            self.checkpointer.load_checkpoint(model=self.model, optimizer=self.optimizer,
                                              checkpoint_path=src if isinstance(src, str) else None,
                                              load_best=config.ckpt.load_best_checkpoint)
            bad = [n for n, p in self.model.named_parameters() if p.numel() and not torch.isfinite(p).all()]
            if bad:
                logger.error(f"non-finite parameters after loading checkpoint: {bad}")

    def logits(self, inputs: torch.Tensor) -> torch.Tensor:
        out = self.model(inputs)
        if torch.isnan(out).any():
            logger.warning("NaN detected in logits")
        return out

    def micro_loss(self, batch: Any, step: int) -> tuple[torch.Tensor, torch.Tensor]:  # noqa: ANN401
        inputs, targets, loss_mask, _doc = batch
        if inputs.is_floating_point() and not torch.isfinite(inputs).all():
            logger.error(f"non-finite inputs at step {step}")
        if type(self).logits is SFTTrainer.logits:
            loss = self.lm_loss(inputs, targets, loss_mask)  # the model's fused LM head + CE
        else:
            with self.device.autocast():
                loss = masked_cross_entropy(self.logits(inputs), targets, loss_mask, self._loss_vocab)
        return loss / self.config.gradient_accumulation_steps, loss_mask.sum()

    def evaluations(self) -> list[Evaluation]:
        return [Evaluation("chatcore", self.config.eval_every_n_steps, self._chatcore)] if self.evaluator else []

    def _chatcore(self, step: int) -> None:
        self.model.eval()
        with torch.no_grad():
            results = self.evaluator.evaluate(num_examples=self.config.eval_num_steps)
        self.model.train()
        metrics: dict[str, Any] = {}
        for k, v in results.items():
            if isinstance(v, dict):
                metrics.update({f"eval/{k}/{sk}": sv for sk, sv in v.items()})
            else:
                metrics[f"eval/{k}"] = v
        if self.is_main_process:
            logger.info(f"Eval step={step} | " + " | ".join(f"{k}={v}" for k, v in metrics.items()))
        self.sink.log(metrics, step=step)


class HFSFTTrainer(SFTTrainer):
    def __init__(self, model: nn.Module, optimizer: Optimizer, dataloader: Any, device: Device, config: SFTConfig,  # noqa: ANN401
                 tokenizer: Any = None, eval_datasets: list | None = None) -> None:  # noqa: ANN401
        super().__init__(LogitsWrapper(model), optimizer, dataloader, device, config, tokenizer, eval_datasets)

    def logits(self, inputs: torch.Tensor) -> torch.Tensor:
        return self.model(input_ids=inputs)
