"""Multi-process (gloo, CPU) parity of DDP / ZeRO-1/2/3 / TP / SP / 2-D mesh against one process.

Each rank trains the same model on its dp shard of a global batch; after several optimizer steps
(with global-norm clipping) the consolidated parameters must equal a single-process run on the
whole batch. The reference's tests only check that these configurations run
(tests/integration/test_distributed.py:14-84); its TP gradients are wrong.
"""

import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
from torch.multiprocessing.spawn import spawn

from mint_b200.models.gemma import Gemma, GemmaConfig, configure_optimizer
from mint_b200.optim.muon_adamw import MuonAdamWConfig
from mint_b200.parallel.api import setup_parallel
from mint_b200.parallel.context import ParallelContext
from mint_b200.parallel.zero import get_engine
from mint_b200.trainer.scheduler import SchedulerConfig
from mint_b200.utils.checkpointer import consolidated_state_dict

CFG = dict(embed_dim=64, hidden_dim=128, seq_length=32, vocab_size=96, n_layers=2, n_heads=4, n_kv_heads=2,
           head_dim=16, pad_vocab_multiple=4)
STEPS = 3


def _free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return int(s.getsockname()[1])


def _batches(dp: int):
    g = torch.Generator().manual_seed(7)
    out = []
    for _ in range(STEPS):
        x = torch.randint(0, CFG["vocab_size"], (2 * dp, CFG["seq_length"]), generator=g)
        y = torch.randint(0, CFG["vocab_size"], (2 * dp, CFG["seq_length"]), generator=g)
        out.append((x, y))
    return out


def _train(model, opt, engine, batches, dp_rank, dp, clip):
    for x, y in batches:
        xs, ys = x.chunk(dp)[dp_rank], y.chunk(dp)[dp_rank]
        opt.zero_grad()
        loss = model.loss(xs, ys, torch.ones_like(xs, dtype=torch.float32))
        loss.backward()
        engine.finish_grad_sync()
        engine.sync_tp_partial_grads()
        engine._synced = True
        engine.clip_grad_norm(clip)
        opt.step()


def _tp_full_grads(model, tp_group, tp_size):
    out = {}
    for name, p in model.named_parameters():
        g = p.grad.detach().clone()
        if getattr(p, "_tp_sharded", False) and tp_size > 1:
            parts = [torch.empty_like(g) for _ in range(tp_size)]
            dist.all_gather(parts, g.contiguous(), group=tp_group)
            g = torch.cat(parts, dim=getattr(p, "_tp_dim", 0))
        out[name] = g
    return out


def _worker(rank, world, port, tp, level, sp, muon, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pctx = ParallelContext.build(tp_size=tp, ddp_level=level, sp=sp, device_type="cpu")
        torch.manual_seed(1337)
        model = Gemma(GemmaConfig(**CFG))
        model = setup_parallel(model, pctx, bucket_cap_mb=0.05)
        opt = configure_optimizer(model, GemmaConfig(**CFG), SchedulerConfig(),
                                  MuonAdamWConfig(matrix_optimizer="muon" if muon else "adamw"), dp_group=pctx.dp_group)
        grads = None
        if level == 0:
            x, y = _batches(pctx.dp_size)[0]
            xs, ys = x.chunk(pctx.dp_size)[pctx.dp_rank], y.chunk(pctx.dp_size)[pctx.dp_rank]
            eng = get_engine(model)
            opt.zero_grad()
            model.loss(xs, ys, torch.ones_like(xs, dtype=torch.float32)).backward()
            eng.finish_grad_sync()
            eng.sync_tp_partial_grads()
            grads = _tp_full_grads(model, pctx.tp_group, pctx.tp_size)
            opt.zero_grad()
        _train(model, opt, get_engine(model), _batches(pctx.dp_size), pctx.dp_rank, pctx.dp_size, 0.5)
        sd = consolidated_state_dict(model)
        osd = opt.state_dict()
        if rank == 0:
            torch.save({"model": sd, "optim": osd, "grads": grads}, out_path)
    finally:
        dist.destroy_process_group()


def _single_grads(dp: int):
    torch.manual_seed(1337)
    model = Gemma(GemmaConfig(**CFG))
    x, y = _batches(dp)[0]
    model.loss(x, y, torch.ones_like(x, dtype=torch.float32)).backward()
    return {n: p.grad for n, p in model.named_parameters()}


def _single(dp: int, muon: bool):
    torch.manual_seed(1337)
    model = setup_parallel(Gemma(GemmaConfig(**CFG)), ParallelContext())
    opt = configure_optimizer(model, GemmaConfig(**CFG), SchedulerConfig(),
                              MuonAdamWConfig(matrix_optimizer="muon" if muon else "adamw"))
    _train(model, opt, get_engine(model), _batches(dp), 0, 1, 0.5)
    return consolidated_state_dict(model), opt.state_dict()


def _run(world, tp, level, sp, muon):
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "out.pt")
        spawn(_worker, args=(world, _free_port(), tp, level, sp, muon, path), nprocs=world, join=True)
        got = torch.load(path, weights_only=False)
    want_sd, want_osd = _single(world // tp, muon)
    if got["grads"] is not None:
        # first-step gradients: exact up to summation order (the reference's TP grads are off by up to 2x)
        for k, v in _single_grads(world // tp).items():
            assert torch.allclose(got["grads"][k], v, atol=1e-6, rtol=1e-4), (k, (got["grads"][k] - v).abs().max())
    # after 3 Adam(W)/NorMuon steps: Adam's per-element normalization amplifies summation-order
    # differences of near-zero gradient entries by up to ~lr, so the bound scales with the group lr
    atol = 2e-5 if tp == 1 else 1e-3
    for k, v in want_sd.items():
        assert torch.allclose(got["model"][k], v, atol=atol, rtol=1e-4), (k, (got["model"][k] - v).abs().max())
    # optimizer state is layout independent (full tensors)
    for pid, st in want_osd["state"].items():
        for name, t in st.items():
            if torch.is_tensor(t):
                assert torch.allclose(got["optim"]["state"][pid][name], t, atol=atol, rtol=1e-3), (pid, name)


@pytest.mark.parametrize("level", [0, 1, 2, 3])
def test_dp2_zero_levels_match_single_process(level):
    _run(2, 1, level, False, muon=False)


@pytest.mark.parametrize("level", [1, 2, 3])
def test_dp2_normuon_owner_sharding_matches_single_process(level):
    _run(2, 1, level, False, muon=True)


@pytest.mark.parametrize("sp", [False, True])
def test_tp2_matches_single_process(sp):
    _run(2, 2, 0, sp, muon=False)


def test_2d_mesh_tp2_sp_zero3_matches_single_process():
    _run(4, 2, 3, True, muon=False)


def test_2d_mesh_tp2_sp_zero2_muon_matches_single_process():
    _run(4, 2, 2, True, muon=True)
