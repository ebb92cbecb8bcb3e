"""Checkpointing in the reference layout (mint/utils/checkpointer.py:15-195), consolidated.

Files: ``checkpoint_latest.pt``, ``checkpoint_step_{N}.pt`` (rotated to
``keep_last_n_checkpoints``), ``checkpoint_best.pt``, ``metadata.json``; payload
``{step, model_state_dict, optimizer_state_dict, dataloader_state, val_loss, best_val_loss}``.

The reference saves rank 0's ``state_dict()``, which under ZeRO-3 holds empty tensors and under
TP holds only TP-rank-0 shards. Here every rank takes part in consolidation (dp shards are
all-gathered by the gradient engine, TP shards are all-gathered over the TP group and
concatenated along their split dimension) and rank 0 writes full tensors, so a checkpoint
loads into any (dp, tp, ddp_level) layout and into the reference's ``Gemma``.
"""

from __future__ import annotations

import json
import signal
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist
from torch import nn
from torch.optim import Optimizer

from mint_b200.config.base import Config
from mint_b200.parallel.zero import get_engine
from mint_b200.utils.logger import logger


@dataclass
class CheckpointerConfig(Config):
    checkpoint_dir: str = "checkpoints"
    save_checkpoint_every_n_steps: int | None = 200
    keep_last_n_checkpoints: int = 1
    resume_from_checkpoint: str | bool | None = ""
    load_best_checkpoint: bool = True


def _strip_compile_prefix(sd: dict[str, Any]) -> dict[str, Any]:
    return {k.removeprefix("_orig_mod."): v for k, v in sd.items()}


def _tp_group_of(model: nn.Module):  # noqa: ANN202
    tp = getattr(model, "tp", None)
    if tp is None or tp.size <= 1:
        return None, 1, 0
    return tp.group, tp.size, tp.rank


@torch.no_grad()
def consolidated_state_dict(model: nn.Module) -> dict[str, torch.Tensor]:
    """Full-tensor CPU state dict (collective over dp and tp when the model is sharded)."""
    model = getattr(model, "_orig_mod", model)
    eng = get_engine(model)
    group, tsize, _ = _tp_group_of(model)
    out: dict[str, torch.Tensor] = {}
    params = dict(model.named_parameters(remove_duplicate=False))
    for key, value in model.state_dict(keep_vars=True).items():
        p = params.get(key)
        t = value
        if p is not None and eng is not None and id(p) in eng.by_param:
            t = eng.full_param(p)
        t = t.detach()
        if p is not None and getattr(p, "_tp_sharded", False) and tsize > 1:
            parts = [torch.empty_like(t) for _ in range(tsize)]
            dist.all_gather(parts, t.contiguous(), group=group)
            t = torch.cat(parts, dim=getattr(p, "_tp_dim", 0))
        out[key] = t.cpu().clone()
    return out


@torch.no_grad()
def load_consolidated_state_dict(model: nn.Module, state: dict[str, torch.Tensor], strict: bool = True) -> None:
    model = getattr(model, "_orig_mod", model)
    state = _strip_compile_prefix(state)
    eng = get_engine(model)
    _, tsize, trank = _tp_group_of(model)
    params = dict(model.named_parameters(remove_duplicate=False))
    own = model.state_dict(keep_vars=True)
    missing = [k for k in own if k not in state]
    unexpected = [k for k in state if k not in own]
    if strict and (missing or unexpected):
        raise RuntimeError(f"state dict mismatch: missing={missing} unexpected={unexpected}")
    for key, value in state.items():
        if key not in own:
            continue
        p = params.get(key)
        v = value
        if p is not None and getattr(p, "_tp_sharded", False) and tsize > 1:
            v = v.chunk(tsize, dim=getattr(p, "_tp_dim", 0))[trank]
        if p is not None and eng is not None and id(p) in eng.by_param:
            eng.load_full_param(p, v.to(eng.slot(p)[0].shard_data.device))
        else:
            own[key].data.copy_(v.to(own[key].device, own[key].dtype))


def _barrier() -> None:
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()


def _check_kernel_status(model: nn.Module) -> None:
    """Synchronous read of the device status word before parameters are consolidated and written."""
    dev = next((p.device for p in model.parameters() if p.device.type == "cuda"), None)
    if dev is None:
        return
    from mint_b200.ops import _ext  # noqa: PLC0415

    if _ext.available() and _ext.kernels_enabled():
        _ext.status_watch(dev.index or 0).flush()


class Checkpointer:
    def __init__(self, config: CheckpointerConfig, *, is_main_process: bool) -> None:
        self.checkpoint_dir = Path(config.checkpoint_dir)
        self.save_every_n_steps = config.save_checkpoint_every_n_steps
        self.keep_last_n = config.keep_last_n_checkpoints
        self.is_main_process = is_main_process
        if is_main_process:
            self.checkpoint_dir.mkdir(parents=True, exist_ok=True)
        self.best_val_loss = float("inf")
        self.interrupt_requested = False
        try:
            signal.signal(signal.SIGINT, self._signal_handler)
        except ValueError:  # not the main thread
            pass

    def _signal_handler(self, signum, frame) -> None:  # noqa: ANN001, ARG002
        logger.warning("Keyboard interrupt received: a checkpoint will be saved at the next step boundary")
        self.interrupt_requested = True

    def save_checkpoint(
        self,
        step: int,
        model: nn.Module,
        optimizer: Optimizer,
        dataloader_state: dict[str, Any],
        val_loss: float | None = None,
        *,
        is_best: bool = False,
        force: bool = False,
    ) -> Path | None:
        """Collective when the model is sharded: every rank calls it; rank 0 writes."""
        should = force or is_best
        if not should and self.save_every_n_steps is not None:
            should = step % self.save_every_n_steps == 0
        if not should:
            return None
        _check_kernel_status(model)  # never write parameters that a failed kernel may have touched
        model_sd = consolidated_state_dict(model)
        optim_sd = optimizer.state_dict()
        try:
            if self.is_main_process:
                return self._write(step, model_sd, optim_sd, dataloader_state, val_loss, is_best)
            return None
        finally:
            # rank 0 writes for seconds while the others would otherwise start the next step and
            # wait in their fused collectives for it: every rank leaves the save together
            _barrier()

    def _write(self, step: int, model_sd: dict, optim_sd: dict, dataloader_state: dict[str, Any],
               val_loss: float | None, is_best: bool) -> Path:
        ckpt = {
            "step": step,
            "model_state_dict": model_sd,
            "optimizer_state_dict": optim_sd,
            "dataloader_state": dataloader_state,
            "val_loss": val_loss,
            "best_val_loss": self.best_val_loss,
        }
        latest = self.checkpoint_dir / "checkpoint_latest.pt"
        torch.save(ckpt, latest)
        step_path = self.checkpoint_dir / f"checkpoint_step_{step}.pt"
        torch.save(ckpt, step_path)
        logger.info(f"Saved checkpoint at step {step} to {step_path}")
        if is_best:
            torch.save(ckpt, self.checkpoint_dir / "checkpoint_best.pt")
            logger.info(f"Saved best checkpoint (val_loss={val_loss:.4f})")
        self._cleanup_old_checkpoints()
        self._save_metadata(step, val_loss)
        return step_path

    def _cleanup_old_checkpoints(self) -> None:
        steps = sorted(self.checkpoint_dir.glob("checkpoint_step_*.pt"), key=lambda p: int(p.stem.split("_")[-1]))
        if len(steps) > self.keep_last_n:
            for old in steps[: -self.keep_last_n]:
                old.unlink()

    def _save_metadata(self, step: int, val_loss: float | None) -> None:
        meta = {"last_step": step, "last_val_loss": val_loss, "best_val_loss": self.best_val_loss}
        with (self.checkpoint_dir / "metadata.json").open("w") as fh:
            json.dump(meta, fh, indent=2)

    @classmethod
    def load_model(cls, model: nn.Module, checkpoint_path: str | None = None) -> dict[str, Any]:
        if checkpoint_path is None:
            raise ValueError("invalid checkpoint path")
        path = Path(checkpoint_path)
        if not path.exists():
            logger.warning(f"Checkpoint not found: {path}")
            return {"step": 0, "dataloader_state": {}}
        ckpt = torch.load(path, map_location="cpu", weights_only=False)
        load_consolidated_state_dict(model, ckpt["model_state_dict"])
        logger.info(f"Loaded model from {path} (step {ckpt['step']})")
        return {"step": ckpt["step"], "dataloader_state": ckpt.get("dataloader_state", {}), "val_loss": ckpt.get("val_loss")}

    def load_checkpoint(
        self,
        model: nn.Module,
        optimizer: Optimizer,
        checkpoint_path: str | None = None,
        *,
        load_best: bool = False,
    ) -> dict[str, Any]:
        if checkpoint_path:
            path = Path(checkpoint_path)
        elif load_best:
            path = self.checkpoint_dir / "checkpoint_best.pt"
        else:
            path = self.checkpoint_dir / "checkpoint_latest.pt"
        if not path.exists():
            logger.warning(f"Checkpoint not found: {path}")
            return {"step": 0, "dataloader_state": {}}
        ckpt = torch.load(path, map_location="cpu", weights_only=False)
        load_consolidated_state_dict(model, ckpt["model_state_dict"])
        optimizer.load_state_dict(ckpt["optimizer_state_dict"])
        self.best_val_loss = ckpt.get("best_val_loss", float("inf"))
        logger.info(f"Loaded checkpoint {path} (step {ckpt['step']})")
        return {"step": ckpt["step"], "dataloader_state": ckpt.get("dataloader_state", {}), "val_loss": ckpt.get("val_loss")}

    def should_checkpoint_on_eval(self, val_loss: float) -> bool:
        if val_loss < self.best_val_loss:
            self.best_val_loss = val_loss
            return True
        return False

    def get_resume_info(self) -> dict[str, Any]:
        path = self.checkpoint_dir / "metadata.json"
        if path.exists():
            with path.open() as fh:
                return json.load(fh)
        return {}
