"""Single-process MuonAdamW (mint/optim/muon_adamw.py:11-269) and its config tables."""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass

import torch
from torch.optim import Optimizer

from mint_b200.config.base import Config
from mint_b200.optim.functional import POLAR_EXPRESS_COEFFS, adamw_update, normuon_update


@dataclass
class AdamConfig(Config):
    adamw_beta1: float = 0.8
    adamw_beta2_lm_head: float = 0.96
    adamw_beta2_embedding: float = 0.995
    adamw_beta2_scalar: float = 0.95
    adamw_eps: float = 1e-10


@dataclass
class MuonConfig(Config):
    muon_momentum: float = 0.95
    muon_beta2: float = 0.9
    muon_ns_steps: int = 5


@dataclass
class MuonAdamWConfig(AdamConfig, MuonConfig):
    # "adamw": every group AdamW (reference behaviour); "muon": 2-D block matrices use NorMuon
    matrix_optimizer: str = "adamw"


class MuonAdamW(Optimizer):
    """Per-parameter AdamW / NorMuon for non-distributed use. Groups carry ``kind``."""

    def __init__(self, param_groups: list[dict]) -> None:
        super().__init__(param_groups, defaults={})

    def _step_adamw(self, group: dict) -> None:
        beta1, beta2 = group["betas"]
        for p in group["params"]:
            if p.grad is None:
                continue
            st = self.state[p]
            if not st:
                st["step"] = 0
                st["exp_avg"] = torch.zeros_like(p)
                st["exp_avg_sq"] = torch.zeros_like(p)
            st["step"] += 1
            adamw_update(p.data, p.grad, st["exp_avg"], st["exp_avg_sq"], st["step"], group["lr"], beta1, beta2,
                         group["eps"], group["weight_decay"])

    def _step_muon(self, group: dict) -> None:
        for p in group["params"]:
            if p.grad is None:
                continue
            st = self.state[p]
            if "momentum_buffer" not in st:
                st["momentum_buffer"] = torch.zeros_like(p, dtype=torch.float32)
                rows, cols = p.shape
                shape = (rows, 1) if rows >= cols else (1, cols)
                st["second_momentum_buffer"] = torch.zeros(shape, dtype=torch.float32, device=p.device)
            normuon_update(
                p.data, p.grad.float(), st["momentum_buffer"], st["second_momentum_buffer"],
                lr=group["lr"], momentum=group["momentum"],
                beta2=group["beta2"] if group.get("beta2") is not None else 0.0,
                wd=group["weight_decay"], ns_steps=group.get("ns_steps", 5),
            )

    @torch.no_grad()
    def step(self, closure: Callable[[], float] | None = None) -> float | None:  # type: ignore[override]
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            if group["kind"] == "adamw":
                self._step_adamw(group)
            elif group["kind"] == "muon":
                self._step_muon(group)
            else:
                raise ValueError(f"Unknown optimizer kind: {group['kind']}")
        return loss


__all__ = ["POLAR_EXPRESS_COEFFS", "AdamConfig", "MuonAdamW", "MuonAdamWConfig", "MuonConfig"]
