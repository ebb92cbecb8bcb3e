"""``mint download-climbmix``: concurrent download of ClimbMix parquet shards (the last one is the
validation shard) into ``data_dir/{train,val}`` (scripts/utils/async_download_climbmix.py)."""

from __future__ import annotations

import argparse
import asyncio
import multiprocessing as mp
from pathlib import Path

from mint_b200.utils.logger import logger

REPO = "karpathy/climbmix-400b-shuffle"
BASE_URL = f"https://huggingface.co/datasets/{REPO}/resolve/main"
PATTERN = "shard_{:05d}.parquet"


class DownloadCoordinator:
    """Counters shared between the download and training processes."""

    def __init__(self, min_shards: int) -> None:
        self.min_shards = min_shards
        self.downloaded_count = mp.Value("i", 0)
        self.total_shards = mp.Value("i", 0)
        self.download_complete = mp.Value("i", 0)
        self.lock = mp.Lock()

    def increment_downloaded(self) -> int:
        with self.lock:
            self.downloaded_count.value += 1
            return self.downloaded_count.value

    def set_total_shards(self, total: int) -> None:
        with self.lock:
            self.total_shards.value = total

    def mark_complete(self) -> None:
        with self.lock:
            self.download_complete.value = 1

    def is_ready_for_training(self) -> bool:
        with self.lock:
            return self.downloaded_count.value >= self.min_shards

    def is_complete(self) -> bool:
        with self.lock:
            return self.download_complete.value == 1

    def get_status(self) -> dict:
        with self.lock:
            return {"downloaded": self.downloaded_count.value, "total": self.total_shards.value,
                    "complete": self.download_complete.value == 1}


async def _fetch(session, url: str, dest: Path) -> bool:  # noqa: ANN001
    tmp = dest.with_suffix(dest.suffix + ".part")
    try:
        async with session.get(url) as resp:
            if resp.status != 200:
                logger.error(f"HTTP {resp.status} for {url}")
                return False
            with tmp.open("wb") as fh:
                async for chunk in resp.content.iter_chunked(1 << 20):
                    fh.write(chunk)
        tmp.rename(dest)
        return True
    except Exception as exc:  # noqa: BLE001
        logger.error(f"download failed for {url}: {exc}")
        tmp.unlink(missing_ok=True)
        return False


async def download_all_shards(output_dir: str, num_train_shards: int, coordinator: DownloadCoordinator,
                              max_concurrent: int = 3, base_url: str = BASE_URL, pattern: str = PATTERN) -> None:
    import aiohttp  # noqa: PLC0415

    out = Path(output_dir)
    (out / "train").mkdir(parents=True, exist_ok=True)
    (out / "val").mkdir(parents=True, exist_ok=True)
    total = num_train_shards + 1
    coordinator.set_total_shards(total)
    sem = asyncio.Semaphore(max_concurrent)
    async with aiohttp.ClientSession(connector=aiohttp.TCPConnector(limit=max_concurrent)) as session:

        async def one(i: int) -> None:
            name = pattern.format(i)
            dest = out / ("train" if i < total - 1 else "val") / name
            async with sem:
                ok = dest.exists() or await _fetch(session, f"{base_url}/{name}", dest)
            if ok and coordinator.increment_downloaded() == coordinator.min_shards:
                logger.info(f"{coordinator.min_shards} shards ready: training can start")

        await asyncio.gather(*(one(i) for i in range(total)))
    coordinator.mark_complete()


def download_process(output_dir: str, num_train_shards: int, coordinator: DownloadCoordinator,
                     max_concurrent: int) -> None:
    asyncio.run(download_all_shards(output_dir, num_train_shards, coordinator, max_concurrent))


def main() -> None:
    p = argparse.ArgumentParser(description="Download ClimbMix shards")
    p.add_argument("--data-dir", type=str, default="data/climbmix")
    p.add_argument("--num-train-shards", type=int, default=10)
    p.add_argument("--max-concurrent-downloads", type=int, default=3)
    args = p.parse_args()
    download_process(args.data_dir, args.num_train_shards, DownloadCoordinator(1), args.max_concurrent_downloads)


if __name__ == "__main__":
    main()
