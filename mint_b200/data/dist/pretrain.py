"""Pretraining dataloaders.

``DistributedBOSBestfitPretrainDataloader`` follows the reference
(mint/data/dist/pretrain.py:16-375): parquet shards under ``data_dir/{train,val}``, row groups
strided by dp rank, tokenization with BOS, best-fit packing into rows of ``T + 1`` tokens,
``doc_ids`` and ``loss_mask = doc[t] == doc[t+1]``, a background producer thread with depth-2
prefetch into pinned memory, dynamic shard discovery and resumable ``(shard_idx, rg_idx,
batches_consumed)`` state.

``DistributedVarlenPretrainDataloader`` (a stub in the reference, pretrain.py:378) emits the
same packed rows plus per-row ``cu_seqlens`` for variable-length attention.

``SyntheticPretrainDataloader`` produces uniform-random token ids (benchmarks): host-generated
pinned batches, copied to the device every step like real data.
"""

from __future__ import annotations

import queue
import random
import threading
import time
from collections.abc import Generator, Iterator
from typing import Any

import torch

from mint_b200.data.dataloader import DataloaderConfig, DistributedDataloader
from mint_b200.data.packing import BestFitBuffer, pack_row
from mint_b200.utils.logger import logger


def prefetch(source: Iterator, depth: int) -> Generator:
    """Run ``source`` in a daemon thread; exceptions are re-raised in the consumer."""
    buf: queue.Queue = queue.Queue(maxsize=depth)
    stop = threading.Event()
    done = object()

    def put(item: object) -> bool:
        while not stop.is_set():
            try:
                buf.put(item, timeout=0.1)
            except queue.Full:
                continue
            return True
        return False

    def worker() -> None:
        try:
            for item in source:
                if not put(item):
                    return
            put(done)
        except BaseException as exc:  # noqa: BLE001
            put(exc)

    thread = threading.Thread(target=worker, daemon=True)
    thread.start()
    try:
        while True:
            item = buf.get()
            if item is done:
                return
            if isinstance(item, BaseException):
                raise item
            yield item
    finally:
        stop.set()


class DistributedBOSBestfitPretrainDataloader(DistributedDataloader):
    def __init__(
        self,
        device: Any,  # noqa: ANN401
        config: DataloaderConfig,
        tokenizer: Any,  # noqa: ANN401
        min_shards_required: int = 2,
        max_shards_to_wait: int = -1,
        shard_check_interval: float = 5.0,
        *args: Any,  # noqa: ANN401
        **kwargs: Any,  # noqa: ANN401
    ) -> None:
        super().__init__(device, config.data_dir, config.batch_size, config.seq_length, tokenizer, *args, **kwargs)
        self.buffer_size = config.buffer_size
        self.tokenizer_batch_size = config.tokenizer_batch_size
        info = device.process_info()
        self.rank = info["dp_rank"]
        self.world_size = info["dp_size"]
        self.is_main = info["is_main"]
        self.min_shards_required = min_shards_required
        self.max_shards_to_wait = max_shards_to_wait
        self.shard_check_interval = shard_check_interval
        self.train_shards: list = []
        self.val_shards: list = []
        self._refresh_shard_lists()
        self.row_capacity = self.T + 1
        self.prefetch_depth = 2
        dev = device.device
        self.inputs = torch.empty((self.B, self.T), dtype=torch.long, device=dev)
        self.targets = torch.empty((self.B, self.T), dtype=torch.long, device=dev)
        self.loss_mask = torch.empty((self.B, self.T), dtype=torch.float32, device=dev)
        self.doc_ids = torch.empty((self.B, self.T), dtype=torch.long, device=dev)
        self.current_shard_idx = 0
        self.current_rg_idx = self.rank
        self.batches_consumed = 0
        self.last_shard_refresh = time.time()

    def _refresh_shard_lists(self) -> None:
        self.train_shards = sorted((self.data_dir / "train").glob("*.parquet"))
        self.val_shards = sorted((self.data_dir / "val").glob("*.parquet"))

    def _shards(self, split: str) -> list:
        return self.train_shards if split == "train" else self.val_shards

    def _wait_for_shards(self, split: str, required: int) -> None:
        shards = self._shards(split)
        while len(shards) < required:
            if self.max_shards_to_wait > 0 and len(shards) >= self.max_shards_to_wait:
                return
            if self.is_main:
                logger.info(f"Waiting for shards... ({len(shards)}/{required} available)")
            time.sleep(self.shard_check_interval)
            self._refresh_shard_lists()
            shards = self._shards(split)

    def _should_refresh(self) -> bool:
        now = time.time()
        if now - self.last_shard_refresh > self.shard_check_interval:
            self.last_shard_refresh = now
            return True
        return False

    def _document_batches(self, split: str, start_shard_idx: int = 0, start_rg_idx: int = -1) -> Iterator[list]:
        import pyarrow.parquet as pq  # noqa: PLC0415

        self._wait_for_shards(split, self.min_shards_required)
        shards = self._shards(split)
        first = start_shard_idx % len(shards) if shards else 0
        while True:
            if self._should_refresh():
                old = len(shards)
                self._refresh_shard_lists()
                shards = self._shards(split)
                if len(shards) > old and self.is_main:
                    logger.info(f"Discovered {len(shards) - old} new shard(s)")
            if not shards:
                if self.max_shards_to_wait > 0:
                    return
                time.sleep(self.shard_check_interval)
                self._refresh_shard_lists()
                shards = self._shards(split)
                continue
            for k in range(len(shards)):
                idx = (first + k) % len(shards)
                path = shards[idx]
                if not path.exists():
                    continue
                pf = pq.ParquetFile(path)
                rg = start_rg_idx if k == 0 and start_rg_idx >= 0 else self.rank
                while rg < pf.num_row_groups:
                    texts = pf.read_row_group(rg).column("text").to_pylist()
                    for i in range(0, len(texts), self.tokenizer_batch_size):
                        yield texts[i : i + self.tokenizer_batch_size]
                        self.batches_consumed += 1
                    rg += self.world_size
                    self.current_rg_idx = rg
                self.current_shard_idx = (idx + 1) % len(shards)
            start_rg_idx = -1

    def _cpu_batches(self, split: str, resume_state: dict | None) -> Generator:
        use_cuda = self.device.is_cuda
        if resume_state and split == "train":
            shard0 = resume_state.get("shard_idx", 0)
            rg0 = resume_state.get("rg_idx", self.rank)
            skip = resume_state.get("batches_consumed", 0)
        else:
            shard0, rg0, skip = 0, self.rank, 0
        # Resume restarts at the saved (shard, row group) cursor. The reference additionally
        # re-skips ``batches_consumed`` batches from that cursor (pretrain.py:200-216), which
        # double-skips data; here the counter only continues.
        self.batches_consumed = skip
        docs = self._document_batches(split, shard0, rg0)
        buf = BestFitBuffer()

        def refill() -> None:
            while len(buf) < self.buffer_size:
                batch = next(docs)
                for toks in self.tokenizer.encode_to_list(batch, add_bos=True, add_eos=False, padding=False):
                    buf.add(toks)

        while True:
            rows = torch.empty((self.B, self.row_capacity), dtype=torch.long)
            row_docs = torch.empty((self.B, self.row_capacity), dtype=torch.long)
            for r in range(self.B):
                toks, dids = pack_row(buf, self.row_capacity, refill)
                rows[r] = torch.tensor(toks, dtype=torch.long)
                row_docs[r] = torch.tensor(dids, dtype=torch.long)
            yield self._to_pinned(rows, row_docs, use_cuda)

    def _to_pinned(self, rows: torch.Tensor, row_docs: torch.Tensor, pin: bool) -> tuple:
        x = torch.empty((self.B, self.T), dtype=torch.long, pin_memory=pin)
        y = torch.empty((self.B, self.T), dtype=torch.long, pin_memory=pin)
        m = torch.empty((self.B, self.T), dtype=torch.float32, pin_memory=pin)
        d = torch.empty((self.B, self.T), dtype=torch.long, pin_memory=pin)
        x.copy_(rows[:, :-1])
        y.copy_(rows[:, 1:])
        m.copy_(row_docs[:, :-1] == row_docs[:, 1:])
        d.copy_(row_docs[:, :-1])
        return x, y, m, d

    def batch_loader(self, split: str = "train", resume_state: dict | None = None) -> Generator:
        nb = self.device.is_cuda
        for x, y, m, d in prefetch(self._cpu_batches(split, resume_state), self.prefetch_depth):
            self.inputs.copy_(x, non_blocking=nb)
            self.targets.copy_(y, non_blocking=nb)
            self.doc_ids.copy_(d, non_blocking=nb)
            self.loss_mask.copy_(m, non_blocking=nb)
            yield self.inputs, self.targets, self.loss_mask, self.doc_ids

    def get_state(self) -> dict:
        return {"shard_idx": self.current_shard_idx, "rg_idx": self.current_rg_idx,
                "batches_consumed": self.batches_consumed}

    def set_state(self, state: dict) -> None:
        self.current_shard_idx = state.get("shard_idx", 0)
        self.current_rg_idx = state.get("rg_idx", self.rank)
        self.batches_consumed = state.get("batches_consumed", 0)

    def sample(self, num_samples: int = 1) -> list[dict]:
        import pyarrow.parquet as pq  # noqa: PLC0415

        shards = self.train_shards or self.val_shards
        out: list[dict] = []
        for _ in range(num_samples if shards else 0):
            pf = pq.ParquetFile(random.choice(shards))  # noqa: S311
            texts = pf.read_row_group(random.randint(0, pf.num_row_groups - 1)).column("text").to_pylist()  # noqa: S311
            toks = self.tokenizer.encode([random.choice(texts)], add_bos=True, add_eos=False, padding=False)[0]  # noqa: S311
            toks = toks[: self.T]
            inp = toks[:-1] if len(toks) > 1 else toks
            tgt = toks[1:] if len(toks) > 1 else toks
            out.append({"input_tokens": inp, "target_tokens": tgt,
                        "input_str": self.tokenizer.decode(inp.unsqueeze(0))[0],
                        "target_str": self.tokenizer.decode(tgt.unsqueeze(0))[0]})
        return out


class DistributedVarlenPretrainDataloader(DistributedBOSBestfitPretrainDataloader):
    """Best-fit rows plus ``cu_seqlens`` (document boundaries over the flattened batch)."""

    def batch_loader(self, split: str = "train", resume_state: dict | None = None) -> Generator:
        for x, y, m, d in super().batch_loader(split, resume_state):
            flat = (d + torch.arange(d.shape[0], device=d.device)[:, None] * (self.T + 1)).reshape(-1)
            change = torch.ones_like(flat, dtype=torch.bool)
            change[1:] = flat[1:] != flat[:-1]
            starts = torch.nonzero(change).flatten().to(torch.int32)
            cu = torch.cat([starts, torch.tensor([flat.numel()], dtype=torch.int32, device=d.device)])
            yield x, y, m, d, cu


class SyntheticPretrainDataloader(DistributedDataloader):
    """Uniform-random token ids in ``[0, vocab)``; no documents (``doc_ids`` is None)."""

    def __init__(self, device: Any, config: DataloaderConfig, vocab_size: int, *args: Any,  # noqa: ANN401
                 tokenizer: Any = None, seed: int | None = None, **kwargs: Any) -> None:  # noqa: ANN401
        super().__init__(device, config.data_dir, config.batch_size, config.seq_length, tokenizer, *args, **kwargs)
        info = device.process_info()
        self.rank = info["dp_rank"]
        self.vocab_size = vocab_size
        self.seed = (config.seed if seed is None else seed) + self.rank  # TP ranks share the batch
        self.step = 0
        dev = device.device
        self.inputs = torch.empty((self.B, self.T), dtype=torch.long, device=dev)
        self.targets = torch.empty((self.B, self.T), dtype=torch.long, device=dev)
        self.loss_mask = torch.ones((self.B, self.T), dtype=torch.float32, device=dev)

    def _cpu_batches(self) -> Generator:
        pin = self.device.is_cuda
        gen = torch.Generator().manual_seed(self.seed)
        for _ in range(self.step):
            torch.randint(0, self.vocab_size, (self.B, self.T + 1), generator=gen)
        while True:
            row = torch.randint(0, self.vocab_size, (self.B, self.T + 1), generator=gen)
            x = torch.empty((self.B, self.T), dtype=torch.long, pin_memory=pin)
            y = torch.empty((self.B, self.T), dtype=torch.long, pin_memory=pin)
            x.copy_(row[:, :-1])
            y.copy_(row[:, 1:])
            yield x, y

    def batch_loader(self, split: str = "train", resume_state: dict | None = None) -> Generator:  # noqa: ARG002
        nb = self.device.is_cuda
        for x, y in prefetch(self._cpu_batches(), 2):
            self.inputs.copy_(x, non_blocking=nb)
            self.targets.copy_(y, non_blocking=nb)
            self.step += 1
            yield self.inputs, self.targets, self.loss_mask, None

    def get_state(self) -> dict:
        return {"step": self.step}

    def set_state(self, state: dict) -> None:
        self.step = state.get("step", 0)

    def sample(self, num_samples: int = 1) -> list[dict]:  # noqa: ARG002
        return []
