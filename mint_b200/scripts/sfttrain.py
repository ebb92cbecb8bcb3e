"""``mint sft`` (scripts/sfttrain.py:56-184 in the reference)."""

from __future__ import annotations

import argparse
from dataclasses import dataclass

import torch.distributed as dist

from mint_b200.config.base import Config
from mint_b200.data.dataloader import DataloaderConfig
from mint_b200.data.datasets.base import SFTEvalDataset
from mint_b200.data.datasets.catalog import ARC, GSM8K, MMLU, CustomJSON, HumanEval, SimpleSpelling, SmolTalk, SpellingBee
from mint_b200.data.dist.sft import DistributedSFTDataloader
from mint_b200.models.gemma import GemmaConfig, configure_optimizer
from mint_b200.optim.muon_adamw import MuonAdamWConfig
from mint_b200.scripts.common import build_model, check_vocab
from mint_b200.tokenizer import TikTokenizer
from mint_b200.trainer.sft import SFTConfig, SFTTrainer
from mint_b200.utils.device import Device, DeviceConfig
from mint_b200.utils.logger import logger


@dataclass
class MetaConfig(Config):
    train: SFTConfig
    model: GemmaConfig
    optim: MuonAdamWConfig
    device: DeviceConfig
    dl: DataloaderConfig


TRAIN_DATASETS = {
    "arc": lambda: ARC(subset="ARC-Challenge", split="train"),
    "mmlu": lambda: MMLU(subset="all", split="auxiliary_train"),
    "gsm8k": lambda: GSM8K(subset="main", split="train"),
    "humaneval": HumanEval,
    "smoltalk": lambda: SmolTalk(split="train"),
    "spellingbee": lambda: SpellingBee(size=1000, split="train"),
    "simplespelling": lambda: SimpleSpelling(size=1000, split="train"),
}
EVAL_DATASETS = {
    "arc": lambda: ARC(subset="ARC-Challenge", split="test"),
    "mmlu": lambda: MMLU(subset="all", split="test"),
    "gsm8k": lambda: GSM8K(subset="main", split="test"),
    "humaneval": HumanEval,
    "spellingbee": lambda: SpellingBee(size=100, split="test"),
    "simplespelling": lambda: SimpleSpelling(size=100, split="test"),
}


def parse_dataset_spec(spec: str, dataset_map: dict) -> list:
    count, name = (int(spec.split("*", 1)[0]), spec.split("*", 1)[1].strip()) if "*" in spec else (1, spec.strip())
    if name in dataset_map:
        return [dataset_map[name]() for _ in range(count)]
    try:
        return [CustomJSON(filepath=name) for _ in range(count)]
    except Exception as exc:  # noqa: BLE001
        logger.error(f"Failed to load dataset '{name}': {exc}")
        return []


def main() -> None:
    parser = argparse.ArgumentParser(description="SFT training for Gemma model")
    parser.add_argument("--config", type=str, default="configs/config_d12_sft.toml", help="Path to config TOML file")
    parser.add_argument("--datasets", type=str, nargs="+",
                        default=["gsm8k", "smoltalk", "arc", "mmlu", "humaneval", "spellingbee", "simplespelling"],
                        help="Datasets to train on (e.g. 'arc', '3*arc', or a path.jsonl)")
    parser.add_argument("--shuffle", action="store_true", default=True, help="Shuffle dataset mixture")
    args = parser.parse_args()
    tokenizer = TikTokenizer()
    config = MetaConfig.from_toml(args.config)
    check_vocab(config.model, tokenizer)
    device = Device(config.device)
    train_ds = [ds for spec in args.datasets for ds in parse_dataset_spec(spec, TRAIN_DATASETS)]
    names = {type(ds).__name__.lower() for ds in train_ds}
    eval_ds = [EVAL_DATASETS[n]() for n in names if n in EVAL_DATASETS]
    eval_ds = [d for d in eval_ds if isinstance(d, SFTEvalDataset)]
    model = build_model(config.model, config.train, device)
    optimizer = configure_optimizer(model, model_cfg=config.model, optim_cfg=config.optim,
                                    sched_cfg=config.train.sched, dp_group=device.parallel.dp_group)
    loader = DistributedSFTDataloader(device=device, config=config.dl, tokenizer=tokenizer, datasets=train_ds,
                                      shuffle=args.shuffle)
    SFTTrainer(model=model, optimizer=optimizer, dataloader=loader, device=device, config=config.train,
               tokenizer=tokenizer, eval_datasets=eval_ds).train()
    if dist.is_initialized():
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
