"""Worker processes for test_fault_tolerance.py (gloo ranks on CPU, one process per rank).

    python fault_worker.py <mode> <rank> <world> <port> <workdir>

modes:
  full     train 6 steps without interruption, save the final parameters
  sigint   train; rank 0 raises SIGINT in itself after step 3 -> every rank stops at the next step
           boundary and the collective forced checkpoint is written
  resume   resume from that checkpoint and train to step 6, save the final parameters
  die      rank 1 exits (no exception, no cleanup) between steps 2 and 3; rank 0 must fail its next
           collective instead of waiting forever
"""

from __future__ import annotations

import os
import signal
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[2]))


def main() -> None:
    mode, rank, world, port, work = sys.argv[1], int(sys.argv[2]), int(sys.argv[3]), sys.argv[4], Path(sys.argv[5])
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=port, MINT_PG_TIMEOUT_S="20")
    torch.manual_seed(0)
    from mint_b200.data.dataloader import DataloaderConfig
    from mint_b200.data.dist.pretrain import SyntheticPretrainDataloader
    from mint_b200.models.gemma import GemmaConfig, configure_optimizer
    from mint_b200.optim.muon_adamw import MuonAdamWConfig
    from mint_b200.scripts.common import build_model
    from mint_b200.trainer.pretrain import PretrainConfig, PreTrainer
    from mint_b200.utils.checkpointer import CheckpointerConfig, consolidated_state_dict
    from mint_b200.utils.device import Device, DeviceConfig

    device = Device(DeviceConfig(mixed_precision=False, tp_size=1, ddp_level=2))
    mcfg = GemmaConfig(embed_dim=32, hidden_dim=64, seq_length=16, vocab_size=64, n_layers=2, n_heads=2, n_kv_heads=2,
                       head_dim=16)
    tcfg = PretrainConfig(train_num_steps=6, use_meta_device=False, compile_model=False, log_every_n_steps=100,
                          eval_every_n_steps=0, core_eval_every_n_step=0, grad_clip=1.0,
                          ckpt=CheckpointerConfig(checkpoint_dir=str(work / "ckpt"), save_checkpoint_every_n_steps=None,
                                                  keep_last_n_checkpoints=2,
                                                  resume_from_checkpoint=(mode == "resume"), load_best_checkpoint=False))
    model = build_model(mcfg, tcfg, device, seed=3)
    opt = configure_optimizer(model, mcfg, tcfg.sched, MuonAdamWConfig(matrix_optimizer="muon"),
                              dp_group=device.parallel.dp_group)
    loader = SyntheticPretrainDataloader(device, DataloaderConfig(batch_size=2, seq_length=16, source="synthetic"),
                                         vocab_size=64)

    class Trainer(PreTrainer):
        def after_step(self, step: int, metrics: dict) -> None:
            super().after_step(step, metrics)
            if mode == "sigint" and rank == 0 and step == 3:
                os.kill(os.getpid(), signal.SIGINT)  # handled by the checkpointer: a flag, no exception
            if mode == "die" and rank == 1 and step == 2:
                os._exit(0)  # leaves between steps: none of its collectives is in flight

    trainer = Trainer(model=model, optimizer=opt, dataloader=loader, device=device, config=tcfg)
    if mode == "resume":
        print(f"[rank {rank}] resumed at step {trainer.start_step}", flush=True)
    trainer.train()
    sd = consolidated_state_dict(model)
    if rank == 0 and mode in ("full", "resume"):
        torch.save(sd, work / f"final_{mode}.pt")
    print(f"[rank {rank}] {mode} done", flush=True)
    import torch.distributed as dist

    dist.destroy_process_group()


if __name__ == "__main__":
    main()
