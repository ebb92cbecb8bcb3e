"""Device / distributed / mixed-precision runtime (mint/utils/device.py:33-299).

torchrun env -> ``init_process_group`` (NCCL on CUDA, gloo on CPU) with a bounded timeout,
device detection, bf16 autocast (fp16 + GradScaler only on pre-sm80 parts), meta-device
materialization, ``setup_parallel`` and the sharded optimizer step with global-norm clipping
over the dp x tp mesh (the reference only reduces the norm over dp, device.py:199-200).
``compile_model`` is accepted for config compatibility but never wraps the model in
``torch.compile``: the hot path is the framework's own kernels.
"""

from __future__ import annotations

import datetime
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist
from torch import nn
from torch.amp.autocast_mode import autocast
from torch.amp.grad_scaler import GradScaler

from mint_b200.config.base import Config
from mint_b200.parallel.context import ParallelContext
from mint_b200.parallel.zero import get_engine
from mint_b200.parallel.api import setup_parallel
from mint_b200.utils.logger import logger


@dataclass
class DeviceConfig(Config):
    mixed_precision: bool = True
    tp_size: int = 1
    ddp_level: int = 0
    sp: bool = False
    # extension: gradient bucket cap (MiB of fp32 grads per bucket)
    bucket_cap_mb: float = 256.0


class Device:
    def __init__(self, config: DeviceConfig) -> None:
        self.config = config
        self._init_distributed()
        self.device = self._detect()
        self.type = self.device.type
        self.parallel = ParallelContext.build(
            tp_size=config.tp_size, ddp_level=config.ddp_level, sp=config.sp, device_type=self.type
        )
        self.is_cuda = self.type == "cuda"
        self.is_mps = self.type == "mps"
        self.is_cpu = self.type == "cpu"
        self.use_amp = self.is_cuda and config.mixed_precision
        self.amp_dtype = self._get_amp_dtype()
        self.scaler = GradScaler(enabled=self.use_amp and self.amp_dtype == torch.float16)
        self._model: nn.Module | None = None
        logger.info(
            f"Device {self.device} | AMP={self.use_amp} {self.amp_dtype} | rank={self.parallel.rank} "
            f"world={self.parallel.world_size} dp={self.parallel.dp_size} tp={self.parallel.tp_size} "
            f"ddp_level={self.parallel.ddp_level} sp={self.parallel.sp}"
        )

    @staticmethod
    def _init_distributed() -> None:
        world = int(os.getenv("WORLD_SIZE", "1"))
        if world <= 1 or dist.is_initialized():
            return
        timeout = datetime.timedelta(seconds=float(os.getenv("MINT_PG_TIMEOUT_S", "600")))
        if torch.cuda.is_available():
            torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
            dist.init_process_group(backend="nccl", timeout=timeout,
                                    device_id=torch.device("cuda", int(os.environ["LOCAL_RANK"])))
        else:
            dist.init_process_group(backend="gloo", timeout=timeout)

    def _detect(self) -> torch.device:
        if torch.cuda.is_available():
            return torch.device("cuda", torch.cuda.current_device())
        if torch.backends.mps.is_available():
            return torch.device("mps")
        return torch.device("cpu")

    def _get_amp_dtype(self) -> torch.dtype | None:
        if not self.use_amp:
            return None
        if self.is_cuda and torch.cuda.get_device_capability()[0] >= 8:
            return torch.bfloat16
        return torch.float16

    def compile_model(self, model: nn.Module, *, enabled: bool = True) -> nn.Module:  # noqa: ARG002
        if enabled:
            logger.info("compile_model: kernels are hand-written; the model is not wrapped in torch.compile")
        return model

    def move_to_device(self, model: nn.Module, *, from_meta: bool = False) -> nn.Module:
        if from_meta:
            model = model.to_empty(device=self.device)

            def _reset(m: nn.Module) -> None:
                fn = getattr(m, "reset_parameters", None)
                if callable(fn):
                    fn()

            model.apply(_reset)
            return model
        return model.to(self.device)

    def setup_parallel(self, model: nn.Module, tp_plan: dict[str, str] | None = None) -> nn.Module:
        model = setup_parallel(model, self.parallel, tp_plan=tp_plan, bucket_cap_mb=self.config.bucket_cap_mb)
        self._model = model
        return model

    def autocast(self) -> torch.autocast:
        return autocast(device_type="cuda" if self.is_cuda else "cpu", dtype=self.amp_dtype, enabled=self.use_amp)

    def to_device(self, *tensors: torch.Tensor, non_blocking: bool = True) -> list[torch.Tensor]:
        return [t.to(self.device, non_blocking=non_blocking and self.is_cuda) for t in tensors]

    def backward(self, loss: torch.Tensor) -> None:
        if self.scaler.is_enabled():
            self.scaler.scale(loss).backward()
        else:
            loss.backward()

    def set_grad_sync(self, enabled: bool) -> None:
        """Gradient accumulation: only the last micro-step of a step needs a gradient collective."""
        eng = get_engine(self._model) if self._model is not None else None
        if eng is not None:
            eng.sync_grads = enabled

    def _poll_kernel_status(self) -> None:
        """Raise if a kernel of the previous step recorded an error (a timed-out peer wait in a
        fused collective, a bad argument). The snapshot is asynchronous, so the host never stalls
        on the current step; the update kernels skip their updates on the device meanwhile."""
        if not self.is_cuda:
            return
        from mint_b200.ops import _ext  # noqa: PLC0415

        if _ext.available() and _ext.kernels_enabled():
            _ext.status_watch(self.device.index or 0).poll()

    def check_kernel_status(self) -> None:
        """Synchronous form of the per-step check (checkpointing, end of training)."""
        if not self.is_cuda:
            return
        from mint_b200.ops import _ext  # noqa: PLC0415

        if _ext.available() and _ext.kernels_enabled():
            _ext.status_watch(self.device.index or 0).flush()

    def optimizer_step(self, optimizer: torch.optim.Optimizer, grad_clip: float = 0.0, params=None) -> None:  # noqa: ANN001
        eng = getattr(optimizer, "engine", None)
        if eng is not None:
            eng.finish_grad_sync()
            eng.sync_tp_partial_grads()
            eng._synced = True
            if self.scaler.is_enabled():
                raise NotImplementedError("fp16 GradScaler with the gradient engine is not supported (use bf16)")
            if grad_clip > 0:
                eng.clip_grad_norm(grad_clip)
            optimizer.step()
            self._poll_kernel_status()
            return
        self._optimizer_step_plain(optimizer, grad_clip, params)
        self._poll_kernel_status()

    def _optimizer_step_plain(self, optimizer: torch.optim.Optimizer, grad_clip: float, params) -> None:  # noqa: ANN001
        if grad_clip > 0 and params is None:
            raise ValueError("params required for grad clipping")
        if self.scaler.is_enabled():
            if grad_clip > 0:
                self.scaler.unscale_(optimizer)
                torch.nn.utils.clip_grad_norm_(list(params), grad_clip)
            self.scaler.step(optimizer)
            self.scaler.update()
            return
        if grad_clip > 0:
            torch.nn.utils.clip_grad_norm_(list(params), grad_clip)
        optimizer.step()

    def synchronize(self) -> None:
        if self.is_cuda:
            torch.cuda.synchronize()

    def empty_cache(self) -> None:
        if self.is_cuda:
            torch.cuda.empty_cache()

    def memory(self) -> str:
        if self.is_cuda:
            return f"{torch.cuda.memory_allocated() / 2**30:.2f}GB / {torch.cuda.memory_reserved() / 2**30:.2f}GB"
        return ""

    def process_info(self) -> dict:
        on = dist.is_available() and dist.is_initialized()
        rank = dist.get_rank() if on else int(os.getenv("RANK", "0"))
        world = dist.get_world_size() if on else int(os.getenv("WORLD_SIZE", "1"))
        local = int(os.getenv("LOCAL_RANK", rank))
        name = f"{self.type}:{local}" if local != rank else str(self.device)
        return {
            "rank": rank, "local_rank": local, "world_size": world,
            "dp_rank": self.parallel.dp_rank, "dp_size": self.parallel.dp_size,
            "tp_rank": self.parallel.tp_rank, "tp_size": self.parallel.tp_size,
            "name": name, "is_main": rank == 0, "distributed": on,
        }

    def __str__(self) -> str:
        return str(self.device)
