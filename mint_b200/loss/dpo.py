"""DPO loss (mint/loss/dpo.py:6-52): sequence log-probs over labelled tokens (-100 ignored) and the
sigmoid DPO objective ``-log sigmoid(beta * ((pi_c - pi_r) - (ref_c - ref_r)))`` with reward metrics."""

from __future__ import annotations

import torch
import torch.nn.functional as F  # noqa: N812
from torch import nn


def compute_logps(logits: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
    """Sum of next-token log-probs of ``labels`` (shifted) where ``labels != -100``."""
    labels = labels[:, 1:]
    logits = logits[:, :-1, :]
    mask = labels != -100
    safe = labels.masked_fill(~mask, 0)
    logp = torch.log_softmax(logits.float(), dim=-1).gather(-1, safe.unsqueeze(-1)).squeeze(-1)
    return (logp * mask).sum(dim=-1)


def sequence_logps(model: nn.Module, input_ids: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
    """``compute_logps(model(input_ids), labels)`` without the [B, T, V] fp32 log-softmax: models
    with ``token_logps`` (Gemma) give the per-position log-prob of the next label directly."""
    if not hasattr(model, "token_logps"):
        return compute_logps(model(input_ids), labels)
    nxt = torch.full_like(labels, -100)
    nxt[:, :-1] = labels[:, 1:]
    mask = nxt != -100
    logp = model.token_logps(input_ids, nxt.masked_fill(~mask, 0))
    return (logp * mask).sum(dim=-1)


class DPOLoss(nn.Module):
    def __init__(self, beta: float = 0.1) -> None:
        super().__init__()
        self.beta = beta

    def forward(self, policy_chosen_logps: torch.Tensor, policy_rejected_logps: torch.Tensor,
                reference_chosen_logps: torch.Tensor, reference_rejected_logps: torch.Tensor):  # noqa: ANN201
        pi = policy_chosen_logps - policy_rejected_logps
        ref = reference_chosen_logps - reference_rejected_logps
        losses = -F.logsigmoid(self.beta * (pi - ref))
        with torch.no_grad():
            cr = self.beta * (policy_chosen_logps - reference_chosen_logps)
            rr = self.beta * (policy_rejected_logps - reference_rejected_logps)
            stats = torch.stack([losses.mean(), cr.mean(), rr.mean(), (cr - rr).mean(), (pi > ref).float().mean()])
            vals = stats.tolist()
        return losses.mean(), {"loss": vals[0], "chosen_rewards": vals[1], "rejected_rewards": vals[2],
                               "reward_margins": vals[3], "accuracy": vals[4]}
