"""``mint stream-train``: start training once ``--min-shards`` shards have arrived while the rest download
(scripts/utils/train_with_streaming_download.py)."""

from __future__ import annotations

import argparse
import multiprocessing as mp
import subprocess
import sys
import time

from mint_b200.scripts.utils.async_download_climbmix import DownloadCoordinator, download_process
from mint_b200.utils.logger import logger


def training_process(train_script: str, train_args: list[str], coordinator: DownloadCoordinator,
                     use_torchrun: bool, torchrun_args: list[str]) -> None:  # noqa: FBT001
    while not coordinator.is_ready_for_training():
        time.sleep(2.0)
    if use_torchrun:
        cmd = [sys.executable, "-m", "torch.distributed.run", *torchrun_args, train_script, *train_args]
    else:
        cmd = [sys.executable, train_script, *train_args]
    logger.info(f"launching: {' '.join(cmd)}")
    subprocess.run(cmd, check=True)  # noqa: S603


def main() -> None:
    p = argparse.ArgumentParser(description="Train with streaming dataset download",
                                formatter_class=argparse.ArgumentDefaultsHelpFormatter)
    p.add_argument("--data-dir", type=str, default="data/climbmix")
    p.add_argument("--num-train-shards", type=int, default=10)
    p.add_argument("--min-shards", type=int, default=3)
    p.add_argument("--max-concurrent-downloads", type=int, default=3)
    p.add_argument("--max-shards-to-wait", type=int, default=-1)
    p.add_argument("--train-script", type=str, required=True)
    p.add_argument("--use-torchrun", action="store_true")
    p.add_argument("--torchrun-args", type=str, default="")
    p.add_argument("--train-args", type=str, default="")
    p.add_argument("--skip-download", action="store_true")
    args = p.parse_args()
    train_args = (args.train_args.split() if args.train_args else []) + ["--min-shards", str(args.min_shards)]
    if args.max_shards_to_wait > 0:
        train_args += ["--max-shards-to-wait", str(args.max_shards_to_wait)]
    coord = DownloadCoordinator(args.min_shards)
    procs = []
    if not args.skip_download:
        procs.append(mp.Process(target=download_process, args=(args.data_dir, args.num_train_shards, coord,
                                                               args.max_concurrent_downloads)))
    else:
        coord.set_total_shards(args.num_train_shards + 1)
        for _ in range(args.min_shards):
            coord.increment_downloaded()
    procs.append(mp.Process(target=training_process, args=(args.train_script, train_args, coord, args.use_torchrun,
                                                           args.torchrun_args.split() if args.torchrun_args else [])))
    for pr in procs:
        pr.start()
    try:
        for pr in procs:
            pr.join()
    except KeyboardInterrupt:
        for pr in procs:
            if pr.is_alive():
                pr.terminate()
        sys.exit(1)


if __name__ == "__main__":
    mp.set_start_method("spawn", force=True)
    main()
