"""``mint pretrain`` (scripts/pretrain.py:28-118 in the reference)."""

from __future__ import annotations

import argparse
from dataclasses import dataclass

import torch.distributed as dist

from mint_b200.config.base import Config
from mint_b200.data.dataloader import DataloaderConfig
from mint_b200.data.dist.pretrain import DistributedBOSBestfitPretrainDataloader, SyntheticPretrainDataloader
from mint_b200.models.gemma import GemmaConfig, configure_optimizer
from mint_b200.optim.muon_adamw import MuonAdamWConfig
from mint_b200.scripts.common import build_model, check_vocab
from mint_b200.tokenizer import TikTokenizer
from mint_b200.trainer.pretrain import PretrainConfig, PreTrainer
from mint_b200.utils.device import Device, DeviceConfig


@dataclass
class MetaConfig(Config):
    train: PretrainConfig
    model: GemmaConfig
    optim: MuonAdamWConfig
    device: DeviceConfig
    dl: DataloaderConfig


def main() -> None:
    parser = argparse.ArgumentParser(description="Train Gemma model with distributed dataloader")
    parser.add_argument("--config", type=str, default="configs/d12_b200.toml", help="Path to config TOML file")
    parser.add_argument("--min-shards", type=int, default=2, help="Minimum shards required before starting training")
    parser.add_argument("--max-shards-to-wait", type=int, default=-1, help="Maximum shards to wait for (-1 = forever)")
    args = parser.parse_args()
    config = MetaConfig.from_toml(args.config)
    synthetic = config.dl.source == "synthetic"
    tokenizer = None if synthetic else TikTokenizer()
    check_vocab(config.model, tokenizer)
    device = Device(config.device)
    model = build_model(config.model, config.train, device)
    optimizer = configure_optimizer(model, model_cfg=config.model, optim_cfg=config.optim,
                                    sched_cfg=config.train.sched, dp_group=device.parallel.dp_group)
    if synthetic:
        dataloader = SyntheticPretrainDataloader(device, config.dl, vocab_size=config.dl.synthetic_vocab_size
                                                 or config.model.vocab_size)
    else:
        dataloader = DistributedBOSBestfitPretrainDataloader(device=device, config=config.dl, tokenizer=tokenizer,
                                                             min_shards_required=args.min_shards,
                                                             max_shards_to_wait=args.max_shards_to_wait)
    trainer = PreTrainer(model=model, optimizer=optimizer, dataloader=dataloader, device=device, config=config.train,
                         tokenizer=tokenizer)
    trainer.train()
    if dist.is_initialized():
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
