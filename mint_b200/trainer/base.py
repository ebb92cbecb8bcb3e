"""Shared training loop pieces (mint/trainer/base.py:25-300).

W&B init with offline fallback, masked next-token loss under autocast, optimizer step through
``Device`` (gradient engine, clipping over dp x tp), step metrics, SIGINT checkpoint and
periodic / final checkpoints. Step time is measured on the device with CUDA events in addition
to the host wall clock (``train/step_time_device_sec``).
"""

from __future__ import annotations

import importlib.util
import netrc
import os
import time
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any
from urllib.parse import urlsplit

import torch
from torch import nn
from torch.optim import Optimizer

from mint_b200.config.base import Config
from mint_b200.eval.base import EvalConfig
from mint_b200.ops.cross_entropy import masked_cross_entropy
from mint_b200.trainer.scheduler import SchedulerConfig
from mint_b200.utils.checkpointer import Checkpointer, CheckpointerConfig
from mint_b200.utils.device import Device
from mint_b200.utils.logger import LoggerConfig, logger
from mint_b200.utils.profiler import ProfilerConfig


@dataclass
class BasetrainConfig(Config):
    mixed_precision: bool = True
    gradient_checkpointing: bool = False
    use_meta_device: bool = True
    compile_model: bool = True
    train_num_steps: int = 1000
    grad_clip: float = 1.0
    log_every_n_steps: int = 10
    eval_every_n_steps: int = 100
    eval_num_steps: int = 10
    core_eval_every_n_step: int = 500
    gradient_accumulation_steps: int = 1
    ckpt: CheckpointerConfig = field(default_factory=CheckpointerConfig)
    sched: SchedulerConfig = field(default_factory=SchedulerConfig)
    lg: LoggerConfig = field(default_factory=LoggerConfig)
    eval: EvalConfig = field(default_factory=EvalConfig)
    profiler: ProfilerConfig = field(default_factory=ProfilerConfig)


def _wandb_has_credentials() -> bool:
    if os.environ.get("WANDB_API_KEY") or os.environ.get("WANDB_IDENTITY_TOKEN_FILE"):
        return True
    path = Path(os.environ["NETRC"]).expanduser() if os.environ.get("NETRC") else Path("~/.netrc").expanduser()
    host = urlsplit(os.environ.get("WANDB_BASE_URL", "https://api.wandb.ai")).netloc
    try:
        creds = netrc.netrc(path).authenticators(host)
    except (OSError, netrc.NetrcParseError):
        return False
    return bool(creds and creds[2])


_masked_cross_entropy = masked_cross_entropy


class StepTimer:
    """CUDA-event step timer (host wall clock on CPU)."""

    def __init__(self, cuda: bool) -> None:
        self.cuda = cuda
        self._start: Any = None
        self._end: Any = None
        self._t0 = 0.0

    def start(self) -> None:
        self._t0 = time.perf_counter()
        if self.cuda:
            self._start = torch.cuda.Event(enable_timing=True)
            self._end = torch.cuda.Event(enable_timing=True)
            self._start.record()

    def stop(self) -> tuple[float, float]:
        """Returns (device seconds, wall seconds); synchronizes the end event."""
        if self.cuda:
            self._end.record()
            self._end.synchronize()
            dev = self._start.elapsed_time(self._end) / 1e3
        else:
            dev = time.perf_counter() - self._t0
        return dev, time.perf_counter() - self._t0


class BaseTrainer:
    def __init__(self, model: nn.Module, optimizer: Optimizer, dataloader: Any, device: Device,  # noqa: ANN401
                 config: BasetrainConfig, tokenizer: Any = None) -> None:  # noqa: ANN401
        self.model = model
        self.optimizer = optimizer
        self.dataloader = dataloader
        self.device = device
        self.config = config
        self.tokenizer = tokenizer
        cfg = getattr(model, "config", None)
        self._pads_vocab = getattr(cfg, "pad_vocab_multiple", 1) > 1
        self._loss_vocab_size = cfg.vocab_size if (self._pads_vocab and cfg is not None) else None
        self.scheduler: Any = None
        self.process_info = device.process_info()
        self.is_main_process = self.process_info["is_main"]
        self.timer = StepTimer(device.is_cuda)
        self.wandb_run = self._init_wandb()

    def _init_wandb(self) -> Any | None:  # noqa: ANN401
        if not self.config.lg.wandb_enabled or not self.is_main_process:
            return None
        if importlib.util.find_spec("wandb") is None:
            raise ImportError("wandb is enabled in config but the package is not installed.")
        import wandb  # noqa: PLC0415

        if not os.environ.get("WANDB_MODE") and not _wandb_has_credentials():
            logger.warning("No W&B credentials found; logging offline.")
            os.environ["WANDB_MODE"] = "offline"
        run = wandb.init(project=self.config.lg.wandb_project, name=self.config.lg.wandb_run_name,
                         entity=self.config.lg.wandb_entity or None,
                         config={k: str(v) if isinstance(v, torch.dtype) else v for k, v in self.config.__dict__.items()})
        return run

    def _log_wandb(self, metrics: dict, step: int) -> None:
        if self.wandb_run is not None:
            self.wandb_run.log(metrics, step=step)

    def _get_dataloader_state(self) -> dict:
        return {}

    def _validate_batch(self, inputs: torch.Tensor, targets: torch.Tensor, step: int) -> None:
        pass

    def _forward_pass(self, inputs: torch.Tensor, doc_ids: torch.Tensor | None = None) -> torch.Tensor:
        extra = {"unpad_logits": False} if self._pads_vocab else {}
        if doc_ids is not None:
            return self.model(inputs, doc_ids=doc_ids, **extra)
        return self.model(inputs, **extra)

    def _compute_loss(self, inputs: torch.Tensor, targets: torch.Tensor, loss_mask: torch.Tensor, step: int,
                      doc_ids: torch.Tensor | None = None) -> torch.Tensor:
        self._validate_batch(inputs, targets, step)
        with self.device.autocast():
            fused = getattr(self.model, "loss", None)
            if callable(fused) and type(self)._forward_pass is BaseTrainer._forward_pass:
                loss = fused(inputs, targets, loss_mask, doc_ids=doc_ids)
            else:
                logits = self._forward_pass(inputs, doc_ids)
                loss = masked_cross_entropy(logits, targets, loss_mask, self._loss_vocab_size)
            return loss / self.config.gradient_accumulation_steps

    def _perform_optimization_step(self, _micro_step: int, step: int, scheduler_metrics: dict | None = None) -> dict:
        if scheduler_metrics is None:
            if self.scheduler is None:
                raise AttributeError("Scheduler not initialized")
            scheduler_metrics = self.scheduler.step(self.optimizer, step)
        self.device.optimizer_step(self.optimizer, grad_clip=self.config.grad_clip, params=self.model.parameters())
        return scheduler_metrics or {}

    def _calculate_step_metrics(self, accumulated_loss: float, step_time: float, tokens_count: int,
                                scheduler_metrics: dict, train_start_time: float, device_time: float | None = None) -> dict:
        out = {
            "train/loss": accumulated_loss,
            "train/step_time_sec": step_time,
            "train/tokens_per_step": tokens_count,
            "train/tokens_per_second": tokens_count / step_time if step_time > 0 else 0.0,
            "train/elapsed_time_sec": time.perf_counter() - train_start_time,
            "scheduler/lr_multiplier": scheduler_metrics.get("lr_multiplier", 1.0),
            "scheduler/muon_momentum": scheduler_metrics.get("muon_momentum", 0.0),
            "scheduler/muon_weight_decay": scheduler_metrics.get("muon_weight_decay", 0.0),
        }
        if device_time is not None:
            out["train/step_time_device_sec"] = device_time
            out["train/tokens_per_second_device"] = tokens_count / device_time if device_time > 0 else 0.0
        return out

    def _handle_interrupt(self, step: int, checkpointer: Checkpointer) -> bool:
        flag = torch.tensor([1.0 if checkpointer.interrupt_requested else 0.0])
        if self.process_info["distributed"]:
            import torch.distributed as dist  # noqa: PLC0415

            flag = flag.to(self.device.device)
            dist.all_reduce(flag, op=dist.ReduceOp.MAX)
        if flag.item() > 0:
            # every rank observed the interrupt (MAX-reduced), so the collective save is safe
            checkpointer.interrupt_requested = True
            state = self._get_dataloader_state()
            checkpointer.save_checkpoint(step=step, model=self.model, optimizer=self.optimizer,
                                         dataloader_state=state, force=True)
            return True
        return False

    def _log_training_progress(self, step: int, metrics: dict) -> None:
        if step % self.config.log_every_n_steps == 0 and self.is_main_process:
            logger.info(
                f"Step {step:4d} | Loss: {metrics['train/loss']:.4f} | Step Time: {metrics['train/step_time_sec']:.4f}s"
                f" | Tokens/s: {metrics['train/tokens_per_second']:.2f} | Memory: {self.device.memory()}"
            )
            self._log_wandb({**metrics, "train/memory": self.device.memory()}, step=step)

    def _maybe_save_checkpoint(self, step: int, checkpointer: Checkpointer, *, force: bool = False) -> None:
        every = self.config.ckpt.save_checkpoint_every_n_steps
        if force or (every is not None and step % every == 0 and step > 0):
            state = self._get_dataloader_state()
            checkpointer.save_checkpoint(step=step, model=self.model, optimizer=self.optimizer,
                                         dataloader_state=state, force=force)

    def _finalize_training(self, step: int, checkpointer: Checkpointer) -> None:
        state = self._get_dataloader_state()
        checkpointer.save_checkpoint(step=step, model=self.model, optimizer=self.optimizer,
                                     dataloader_state=state, force=True)
        if self.wandb_run is not None:
            self.wandb_run.finish()

    def _log_sample_predictions(self, step: int, num_samples: int = 3) -> None:  # noqa: ARG002
        if not self.is_main_process or not self.tokenizer or not hasattr(self.dataloader, "sample"):
            return
        for i, s in enumerate(self.dataloader.sample(num_samples=num_samples), 1):
            with torch.no_grad():
                logits = self.model(s["input_tokens"].unsqueeze(0).to(self.device.device))
                pred = self.tokenizer.decode(logits.argmax(dim=-1))[0]
            logger.debug(f"Sample {i}: input ...{s['input_str'][-100:]} | pred ...{pred[-100:]}")
