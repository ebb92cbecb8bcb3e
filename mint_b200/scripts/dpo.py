"""``mint dpo`` (scripts/dpo.py:28-111 in the reference)."""

from __future__ import annotations

import argparse
from dataclasses import dataclass

import torch
import torch.distributed as dist

from mint_b200.config.base import Config
from mint_b200.data.dataloader import DataloaderConfig
from mint_b200.data.dist.dpo import DistributedDPODataloader
from mint_b200.models.gemma import Gemma, GemmaConfig, configure_optimizer
from mint_b200.optim.muon_adamw import MuonAdamWConfig
from mint_b200.scripts.common import build_model, check_vocab
from mint_b200.tokenizer import TikTokenizer
from mint_b200.trainer.dpo import DPOConfig, DPOTrainer
from mint_b200.utils.checkpointer import Checkpointer
from mint_b200.utils.device import Device, DeviceConfig


@dataclass
class MetaConfig(Config):
    train: DPOConfig
    model: GemmaConfig
    optim: MuonAdamWConfig
    device: DeviceConfig
    dl: DataloaderConfig


def main() -> None:
    parser = argparse.ArgumentParser(description="DPO training for Gemma")
    parser.add_argument("--config", type=str, default="configs/config_d12_dpo.toml", help="Path to config TOML file")
    parser.add_argument("--ref-model", type=str, default=None, help="Path to ref model checkpoint")
    parser.add_argument("--data-file", type=str, default="hh_rlhf_formatted.jsonl", help="JSONL file under dl.data_dir")
    args = parser.parse_args()
    tokenizer = TikTokenizer()
    config = MetaConfig.from_toml(args.config)
    check_vocab(config.model, tokenizer)
    device = Device(config.device)
    policy = build_model(config.model, config.train, device)
    with torch.device("meta"):
        reference = Gemma(config.model, gradient_checkpointing=False)
    reference = device.move_to_device(reference, from_meta=True)
    reference.requires_grad_(False)
    if args.ref_model:
        Checkpointer.load_model(reference, checkpoint_path=args.ref_model)
    optimizer = configure_optimizer(policy, model_cfg=config.model, optim_cfg=config.optim,
                                    sched_cfg=config.train.sched, dp_group=device.parallel.dp_group)
    loader = DistributedDPODataloader(device=device, config=config.dl, tokenizer=tokenizer, filename=args.data_file)
    DPOTrainer(policy_model=policy, reference_model=reference, optimizer=optimizer, dataloader=loader, device=device,
               config=config.train, tokenizer=tokenizer).train()
    if dist.is_initialized():
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
