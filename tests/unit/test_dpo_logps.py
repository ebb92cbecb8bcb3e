"""Fused DPO sequence log-probs (``Gemma.token_logps`` through ``sequence_logps``) against the
reference formulation ``log_softmax(model(ids)).gather`` on CPU: values and parameter gradients,
one process and a vocab-parallel TP=2 group (gloo)."""

import os
import socket

import torch
import torch.distributed as dist
from torch.multiprocessing.spawn import spawn

from mint_b200.loss.dpo import compute_logps, sequence_logps
from mint_b200.models.gemma import Gemma, GemmaConfig
from mint_b200.nn.base import LogitsWrapper

CFG = dict(embed_dim=64, hidden_dim=128, seq_length=32, vocab_size=100, n_layers=2, n_heads=2, n_kv_heads=2,
           head_dim=32, rope_base_theta=10000)


def _batch():
    g = torch.Generator().manual_seed(3)
    ids = torch.randint(0, 100, (4, 32), generator=g)
    labels = ids.clone()
    labels[:, :7] = -100
    return ids, labels


def test_sequence_logps_matches_logits_path():
    torch.manual_seed(0)
    model = Gemma(GemmaConfig(**CFG))
    ids, labels = _batch()
    got = sequence_logps(LogitsWrapper(model), ids, labels)
    got.sum().backward()
    grads = {n: p.grad.clone() for n, p in model.named_parameters()}
    model.zero_grad()
    want = compute_logps(model(ids), labels)
    want.sum().backward()
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-4)
    for n, p in model.named_parameters():
        torch.testing.assert_close(grads[n], p.grad, rtol=1e-4, atol=1e-5, msg=n)


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return int(s.getsockname()[1])


def _tp_worker(rank, world, port, out):
    from mint_b200.parallel.api import setup_parallel
    from mint_b200.parallel.context import ParallelContext
    from mint_b200.parallel.zero import get_engine

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pctx = ParallelContext.build(tp_size=2, sp=False, device_type="cpu")
        torch.manual_seed(0)
        model = setup_parallel(Gemma(GemmaConfig(**CFG)), pctx)
        ids, labels = _batch()
        lp = sequence_logps(model, ids, labels)
        lp.sum().backward()
        eng = get_engine(model)
        eng.finish_grad_sync()
        eng.sync_tp_partial_grads()
        grads = {}
        for name, p in model.named_parameters():
            g = p.grad.detach().clone()
            if getattr(p, "_tp_sharded", False):
                parts = [torch.empty_like(g) for _ in range(2)]
                dist.all_gather(parts, g.contiguous(), group=pctx.tp_group)
                g = torch.cat(parts, dim=getattr(p, "_tp_dim", 0))
            grads[name] = g
        if rank == 0:
            torch.save({"lp": lp.detach(), "grads": grads}, out)
    finally:
        dist.destroy_process_group()


def test_sequence_logps_vocab_parallel_tp2(tmp_path):
    out = str(tmp_path / "tp.pt")
    spawn(_tp_worker, args=(2, _port(), out), nprocs=2, join=True)
    got = torch.load(out)
    torch.manual_seed(0)
    model = Gemma(GemmaConfig(**CFG))
    ids, labels = _batch()
    want = compute_logps(model(ids), labels)
    want.sum().backward()
    torch.testing.assert_close(got["lp"], want.detach(), rtol=1e-5, atol=1e-4)
    for n, p in model.named_parameters():
        gn = got["grads"][n][: p.shape[0]] if got["grads"][n].shape != p.shape else got["grads"][n]
        err = ((gn - p.grad).norm() / p.grad.norm().clamp_min(1e-12)).item()
        assert err < 1e-4, (n, err, gn.norm().item(), p.grad.norm().item())
