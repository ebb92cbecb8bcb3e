"""The training loop shared by pretraining, SFT and DPO.

Public surface kept from the reference (mint/trainer/base.py:25-300): ``BasetrainConfig`` (the
``[train]`` TOML table and its sub-tables), ``BaseTrainer`` with ``train()``, the step metric names
(``train/loss``, ``train/step_time_sec``, ``train/tokens_per_step``, ``train/tokens_per_second``,
``train/elapsed_time_sec``, ``scheduler/*``, ``train/memory``), SIGINT-triggered checkpoints,
periodic and final checkpoints, W&B logging with an offline fallback.

Structure (this framework's own): a trainer describes its *task* through four hooks --
``micro_batches()`` (an iterator of micro-batches), ``micro_loss(batch, step)`` (the loss scaled for
accumulation and the number of tokens it covers), ``evaluations()`` (named, periodic evaluation
callbacks) and ``dataloader_state()`` -- and ``BaseTrainer.train`` owns everything else: grouping
micro-batches into optimizer steps, gradient-sync control, device-timed steps, the collective
interrupt check, the optimizer step through ``Device`` (clipping over dp x tp), logging, evaluation
and checkpoint cadence. A forward that is collective under tensor parallelism (sample predictions)
runs on every rank.
"""

from __future__ import annotations

import importlib.util
import itertools
import netrc
import os
import time
from collections.abc import Callable, Iterable, Iterator
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any
from urllib.parse import urlsplit

import torch
import torch.distributed as dist
from torch import nn
from torch.optim import Optimizer

from mint_b200.config.base import Config
from mint_b200.eval.base import EvalConfig
from mint_b200.ops.cross_entropy import masked_cross_entropy
from mint_b200.trainer.scheduler import Scheduler, SchedulerConfig
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


# the reference's name for the loss helper its trainers use
_masked_cross_entropy = masked_cross_entropy


# ---------------------------------------------------------------------------------------------- logging sink
def wandb_credentials_available() -> bool:
    """An API key in the environment, an identity-token file, or a netrc entry for the W&B host."""
    if os.environ.get("WANDB_API_KEY") or os.environ.get("WANDB_IDENTITY_TOKEN_FILE"):
        return True
    host = urlsplit(os.environ.get("WANDB_BASE_URL", "https://api.wandb.ai")).netloc
    for path in filter(None, [os.environ.get("NETRC"), "~/.netrc", "~/_netrc"]):
        try:
            entry = netrc.netrc(Path(path).expanduser()).authenticators(host)
        except (OSError, netrc.NetrcParseError):
            continue
        if entry and entry[2]:
            return True
    return False


class MetricSink:
    """W&B on the main process (offline when no credentials are found), nothing elsewhere."""

    def __init__(self, config: BasetrainConfig, enabled: bool) -> None:
        self.run = None
        if not (enabled and config.lg.wandb_enabled):
            return
        if importlib.util.find_spec("wandb") is None:
            raise ImportError("wandb is enabled in config but the package is not installed.")
        import wandb  # noqa: PLC0415

        if "WANDB_MODE" not in os.environ and not wandb_credentials_available():
            logger.warning("No W&B credentials found; logging offline.")
            os.environ["WANDB_MODE"] = "offline"
        flat = {k: (str(v) if isinstance(v, torch.dtype) else v) for k, v in vars(config).items()}
        self.run = wandb.init(project=config.lg.wandb_project, name=config.lg.wandb_run_name,
                              entity=config.lg.wandb_entity or None, config=flat)

    def log(self, metrics: dict[str, Any], step: int) -> None:
        if self.run is not None:
            self.run.log(metrics, step=step)

    def close(self) -> None:
        if self.run is not None:
            self.run.finish()
            self.run = None


# ---------------------------------------------------------------------------------------------- timing
class StepTimer:
    """Device time (CUDA events on the current stream) and host wall time of one optimizer step."""

    def __init__(self, cuda: bool) -> None:
        self.cuda = cuda
        self._events: tuple[Any, Any] | None = None
        self._t0 = 0.0

    def start(self) -> None:
        self._t0 = time.perf_counter()
        if self.cuda:
            self._events = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            self._events[0].record()

    def stop(self) -> tuple[float, float]:
        """(device seconds, wall seconds); waits for the step's last kernel."""
        if self.cuda and self._events is not None:
            self._events[1].record()
            self._events[1].synchronize()
            dev = self._events[0].elapsed_time(self._events[1]) / 1e3
        else:
            dev = time.perf_counter() - self._t0
        return dev, time.perf_counter() - self._t0


@dataclass
class Evaluation:
    """``run(step)`` every ``every`` optimizer steps (never at step 0)."""

    name: str
    every: int
    run: Callable[[int], Any]

    def due(self, step: int) -> bool:
        return self.every > 0 and step > 0 and step % self.every == 0


# ---------------------------------------------------------------------------------------------- the loop
class BaseTrainer:
    def __init__(self, model: nn.Module, optimizer: Optimizer, dataloader: Any, device: Device,  # noqa: ANN401
                 config: BasetrainConfig, tokenizer: Any = None) -> None:  # noqa: ANN401
        self.model = model
        self.optimizer = optimizer
        self.dataloader = dataloader
        self.device = device
        self.config = config
        self.tokenizer = tokenizer
        self.process_info = device.process_info()
        self.is_main_process = self.process_info["is_main"]
        self.timer = StepTimer(device.is_cuda)
        self.sink = MetricSink(config, self.is_main_process)
        self.checkpointer = Checkpointer(config=config.ckpt, is_main_process=self.is_main_process)
        sched = getattr(config, "sched", None)
        self.scheduler = Scheduler(num_iterations=config.train_num_steps, config=sched) if sched is not None else None
        for g in optimizer.param_groups:
            g.setdefault("initial_lr", g["lr"])
        cfg = getattr(model, "config", None)
        self._loss_vocab = cfg.vocab_size if cfg is not None and getattr(cfg, "pad_vocab_multiple", 1) > 1 else None
        self.start_step = 0
        self.last_metrics: dict[str, Any] = {}

    # ------------------------------------------------------------------ the task (overridden)
    def micro_batches(self) -> Iterable[Any]:
        return self.dataloader.batch_loader(split="train")

    def micro_loss(self, batch: Any, step: int) -> tuple[torch.Tensor, int | torch.Tensor]:  # noqa: ANN401
        """Loss of one micro-batch scaled by 1 / accumulation, and the tokens it covers."""
        inputs, targets, loss_mask, doc_ids = batch
        loss = self.lm_loss(inputs, targets, loss_mask, doc_ids)
        return loss / self.config.gradient_accumulation_steps, targets.numel()

    def evaluations(self) -> list[Evaluation]:
        return []

    def dataloader_state(self) -> dict:
        return {}

    # ------------------------------------------------------------------ shared pieces
    def lm_loss(self, inputs: torch.Tensor, targets: torch.Tensor, loss_mask: torch.Tensor,
                doc_ids: torch.Tensor | None = None) -> torch.Tensor:
        """Masked next-token loss under autocast: the model's fused LM-head + CE when it has one."""
        with self.device.autocast():
            fused = getattr(self.model, "loss", None)
            if callable(fused):
                return fused(inputs, targets, loss_mask, doc_ids=doc_ids)
            logits = self.model(inputs, doc_ids=doc_ids) if doc_ids is not None else self.model(inputs)
            return masked_cross_entropy(logits, targets, loss_mask, self._loss_vocab)

    def _interrupted(self) -> bool:
        """SIGINT on any rank stops every rank at the same step boundary (MAX-reduced flag)."""
        flag = torch.tensor([1.0 if self.checkpointer.interrupt_requested else 0.0])
        if self.process_info["distributed"]:
            flag = flag.to(self.device.device)
            dist.all_reduce(flag, op=dist.ReduceOp.MAX)
        hit = bool(flag.item() > 0)
        if hit:
            self.checkpointer.interrupt_requested = True
        return hit

    def save(self, step: int, *, force: bool = False, val_loss: float | None = None, is_best: bool = False) -> None:
        """Collective: every rank takes part in consolidating the model and optimizer state."""
        self.checkpointer.save_checkpoint(step=step, model=self.model, optimizer=self.optimizer,
                                          dataloader_state=self.dataloader_state(), val_loss=val_loss,
                                          is_best=is_best, force=force)

    def memory(self) -> str:
        return self.device.memory()

    def _metrics(self, loss: float, dev_t: float, wall_t: float, tokens: int, sched: dict, t_train: float) -> dict:
        return {
            "train/loss": loss,
            "train/step_time_sec": wall_t,
            "train/tokens_per_step": tokens,
            "train/tokens_per_second": tokens / wall_t if wall_t > 0 else 0.0,
            "train/elapsed_time_sec": time.perf_counter() - t_train,
            "train/step_time_device_sec": dev_t,
            "train/tokens_per_second_device": tokens / dev_t if dev_t > 0 else 0.0,
            "scheduler/lr_multiplier": sched.get("lr_multiplier", 1.0),
            "scheduler/muon_momentum": sched.get("muon_momentum", 0.0),
            "scheduler/muon_weight_decay": sched.get("muon_weight_decay", 0.0),
        }

    def _report(self, step: int, metrics: dict) -> None:
        if step % self.config.log_every_n_steps or not self.is_main_process:
            return
        logger.info(f"Step {step:4d} | Loss: {metrics['train/loss']:.4f} | Step Time: "
                    f"{metrics['train/step_time_sec']:.4f}s | Tokens/s: {metrics['train/tokens_per_second']:.2f} | "
                    f"Memory: {self.memory()}")
        self.sink.log({**metrics, "train/memory": self.memory()}, step=step)

    def log_sample_predictions(self, samples: list[dict[str, Any]]) -> None:
        """Greedy next-token predictions on a few samples. Under tensor parallelism the forward is
        collective, so every rank runs it (same samples) and only the main process logs."""
        tp = getattr(self.model, "tp", None)
        collective = tp is not None and getattr(tp, "size", 1) > 1
        if not self.tokenizer or not (self.is_main_process or collective):
            return
        with torch.no_grad():
            for i, s in enumerate(samples, 1):
                logits = self.model(s["input_tokens"].unsqueeze(0).to(self.device.device))
                if self.is_main_process:
                    pred = self.tokenizer.decode(logits.argmax(dim=-1))[0]
                    logger.debug(f"Sample {i}: input ...{s['input_str'][-100:]} | pred ...{pred[-100:]}")

    # ------------------------------------------------------------------ train
    def _steps(self) -> Iterator[list[Any]]:
        """Micro-batches grouped into optimizer steps (a trailing partial group is dropped)."""
        it = iter(self.micro_batches())
        accum = self.config.gradient_accumulation_steps
        while True:
            group = list(itertools.islice(it, accum))
            if len(group) < accum:
                return
            yield group

    def before_step(self, step: int) -> None:  # noqa: ARG002
        """Called after the previous step's optimizer update, before this step's first forward."""

    def after_step(self, step: int, metrics: dict) -> None:  # noqa: ARG002
        """Called once a step is fully done (metrics computed, before evaluations / checkpoints)."""

    def train(self) -> None:
        self.model.train()
        t_train = time.perf_counter()
        evaluations = self.evaluations()
        step = self.start_step
        steps = self._steps()
        while step < self.config.train_num_steps:
            # decide before drawing the next micro-batches, so a checkpoint's dataloader cursor
            # points exactly at the first batch of the step a resumed run starts with
            if self._interrupted():
                self.save(step, force=True)
                return self._close()
            group = next(steps, None)
            if group is None:
                break
            self.before_step(step)
            self.timer.start()
            self.optimizer.zero_grad()
            loss_sum: torch.Tensor | float = 0.0
            tokens = 0
            for i, batch in enumerate(group):
                self.device.set_grad_sync(i == len(group) - 1)  # one gradient collective per step
                loss, n = self.micro_loss(batch, step)
                self.device.backward(loss)
                loss_sum = loss_sum + loss.detach()
                tokens += int(n)
            step += 1
            sched = self.scheduler.step(self.optimizer, step) if self.scheduler is not None else {}
            self.device.optimizer_step(self.optimizer, grad_clip=self.config.grad_clip, params=self.model.parameters())
            dev_t, wall_t = self.timer.stop()
            tokens *= self.process_info["dp_size"]
            metrics = self._metrics(float(loss_sum), dev_t, wall_t, tokens, sched, t_train)
            self.last_metrics = metrics
            self.after_step(step, metrics)
            for ev in evaluations:
                if ev.due(step):
                    ev.run(step)
            every = self.config.ckpt.save_checkpoint_every_n_steps
            if every and step % every == 0:
                self.save(step)
            self._report(step, metrics)
        self.save(step, force=True)
        self._close()

    def _close(self) -> None:
        self.device.check_kernel_status()
        self.sink.close()
