import pytest
"""Config / CLI / tokenizer / packing / scheduler / checkpoint behaviour on CPU."""

import json
import subprocess
import sys
from pathlib import Path

import torch

from mint_b200.data.packing import BestFitBuffer, pack_row
from mint_b200.tokenizer import TikTokenizer, byte_level_encoding
from mint_b200.trainer.scheduler import Scheduler, SchedulerConfig

ROOT = Path(__file__).resolve().parents[2]


def test_cli_lists_commands():
    out = subprocess.run([sys.executable, "-m", "mint_b200", "--help"], capture_output=True, text=True, cwd=ROOT)
    assert out.returncode == 0
    for cmd in ("pretrain", "sft", "dpo", "chat", "gen-config", "stream-train", "download-climbmix", "download-eval",
                "prepare-dpo"):
        assert cmd in out.stdout


def test_reference_configs_parse():
    from mint_b200.scripts.pretrain import MetaConfig

    for name in ("d12_b200.toml", "config_d12_pretrain.toml"):
        cfg = MetaConfig.from_toml(str(ROOT / "configs" / name))
        assert cfg.model.n_layers > 0 and cfg.device.ddp_level in (0, 1, 2, 3)


def test_tokenizer_ids_layout():
    tok = TikTokenizer(encoding=byte_level_encoding())
    mx = 255
    assert (tok.bos_token, tok.pad_token, tok.vocab_size) == (mx + 1, mx + 2, mx + 11)
    assert tok.encode_special("<|user_start|>") == mx + 3 and tok.encode_special("<|output_end|>") == mx + 10
    ids, mask = tok.render_conversation({"messages": [
        {"role": "system", "content": "sys"},
        {"role": "user", "content": "hi"},
        {"role": "assistant", "content": [{"type": "text", "text": "a"}, {"type": "python", "text": "1+1"},
                                          {"type": "python_output", "text": "2"}]},
    ]})
    assert ids[0] == tok.bos_token and mask[0] == 0
    assert len(ids) == len(mask)
    assert tok.decode(torch.tensor(ids)) == ["sys\n\nhia1+12"]


def test_tokenizer_matches_reference_rendering(reference_mint):
    import mint.tokenizer as rt

    class _RefTok(rt.TikTokenizer):
        def __init__(self, enc):  # the reference constructor downloads GPT-2 ranks; reuse its methods only
            self.encoding = enc
            mx = enc.max_token_value
            self._bos_token, self._eos_token, self._pad_token = mx + 1, mx, mx + 2
            self.special_tokens = {k: mx + 3 + i for i, k in enumerate([
                "<|user_start|>", "<|user_end|>", "<|assistant_start|>", "<|assistant_end|>",
                "<|python_start|>", "<|python_end|>", "<|output_start|>", "<|output_end|>"])}

    enc = byte_level_encoding()
    ours, ref = TikTokenizer(encoding=enc), _RefTok(enc)
    conv = {"messages": [{"role": "user", "content": "count r in strawberry"},
                         {"role": "assistant", "content": [{"type": "text", "text": "x"},
                                                           {"type": "python", "text": "'s'.count('r')"},
                                                           {"type": "python_output", "text": "3"}]}]}
    assert ours.render_conversation(conv, 64) == ref.render_conversation(conv, 64)
    assert ours.encode_to_list(["ab", "c"]) == ref.encode_to_list(["ab", "c"])


def _reference_pack(docs, B, cap, buffer_size):
    """The reference's O(buffer) best-fit scan (mint/data/dist/pretrain.py:218-257), as the oracle."""
    it = iter(docs)
    buf = []
    rows = []
    for _ in range(B):
        row, pos = [], 0
        while pos < cap:
            while len(buf) < buffer_size:
                buf.append(next(it))
            rem = cap - pos
            best, best_len = -1, 0
            for i, d in enumerate(buf):
                if best_len < len(d) <= rem:
                    best, best_len = i, len(d)
            if best >= 0:
                d = buf.pop(best)
            else:
                i = min(range(len(buf)), key=lambda k: len(buf[k]))
                d = buf.pop(i)[:rem]
            row += d
            pos += len(d)
        rows.append(row)
    return rows


def test_best_fit_packing_matches_reference_scan():
    import random

    rng = random.Random(0)
    docs = [[rng.randrange(100) for _ in range(rng.randint(1, 60))] for _ in range(4000)]
    want = _reference_pack(docs, 20, 129, 50)
    it = iter(docs)
    buf = BestFitBuffer()

    def refill():
        while len(buf) < 50:
            buf.add(next(it))

    got = [pack_row(buf, 129, refill)[0] for _ in range(20)]
    assert got == want


def test_scheduler_matches_reference(reference_mint):
    from mint.trainer.scheduler import Scheduler as RS
    from mint.trainer.scheduler import SchedulerConfig as RC

    kw = dict(warmup_steps=5, warmdown_ratio=0.4, muon_momentum_warmup_steps=10, weight_decay=0.1)
    ours, ref = Scheduler(50, SchedulerConfig(**kw)), RS(50, RC(**kw))
    for s in range(50):  # same curves; the evaluation order of the arithmetic may differ in the last ulp
        assert ours.get_lr_multiplier(s) == pytest.approx(ref.get_lr_multiplier(s), rel=1e-12, abs=1e-15)
        assert ours.get_muon_momentum(s) == pytest.approx(ref.get_muon_momentum(s), rel=1e-12, abs=1e-15)
        assert ours.get_weight_decay(s) == pytest.approx(ref.get_weight_decay(s), rel=1e-12, abs=1e-15)


def test_gen_config_emits_loadable_toml(tmp_path):
    out = tmp_path / "cfg.toml"
    r = subprocess.run([sys.executable, "-m", "mint_b200", "gen-config", "--depth-target", "4", "--output", str(out)],
                       capture_output=True, text=True, cwd=ROOT)
    assert r.returncode == 0, r.stderr
    from mint_b200.scripts.pretrain import MetaConfig

    cfg = MetaConfig.from_toml(str(out))
    assert cfg.model.n_layers == 4


def test_checkpoint_roundtrip_and_rotation(tmp_path):
    from mint_b200.models.gemma import Gemma, GemmaConfig, configure_optimizer
    from mint_b200.optim.muon_adamw import MuonAdamWConfig
    from mint_b200.parallel.api import setup_parallel
    from mint_b200.parallel.context import ParallelContext
    from mint_b200.utils.checkpointer import Checkpointer, CheckpointerConfig

    cfg = GemmaConfig(embed_dim=32, hidden_dim=64, seq_length=16, vocab_size=50, n_layers=2, n_heads=2, n_kv_heads=1,
                      head_dim=16)
    torch.manual_seed(0)
    model = setup_parallel(Gemma(cfg), ParallelContext())
    opt = configure_optimizer(model, cfg, SchedulerConfig(), MuonAdamWConfig(matrix_optimizer="muon"))
    x = torch.randint(0, 50, (2, 16))
    for _ in range(2):
        opt.zero_grad()
        model.loss(x, x, torch.ones(2, 16)).backward()
        opt.step()
    ck = Checkpointer(CheckpointerConfig(checkpoint_dir=str(tmp_path), keep_last_n_checkpoints=2), is_main_process=True)
    for s in (1, 2, 3):
        ck.save_checkpoint(s, model, opt, {"shard_idx": 0}, force=True)
    names = sorted(p.name for p in tmp_path.glob("checkpoint_step_*.pt"))
    assert names == ["checkpoint_step_2.pt", "checkpoint_step_3.pt"]
    assert (tmp_path / "checkpoint_latest.pt").exists()
    meta = json.loads((tmp_path / "metadata.json").read_text())
    assert meta["last_step"] == 3
    sd = torch.load(tmp_path / "checkpoint_latest.pt", weights_only=False)
    assert set(sd) == {"step", "model_state_dict", "optimizer_state_dict", "dataloader_state", "val_loss",
                       "best_val_loss"}
    assert "output.weight" in sd["model_state_dict"] and "tok_embeddings.weight" in sd["model_state_dict"]
    model2 = setup_parallel(Gemma(cfg), ParallelContext())
    opt2 = configure_optimizer(model2, cfg, SchedulerConfig(), MuonAdamWConfig(matrix_optimizer="muon"))
    Checkpointer(CheckpointerConfig(checkpoint_dir=str(tmp_path)), is_main_process=True).load_checkpoint(
        model2, opt2, str(tmp_path / "checkpoint_latest.pt"))
    for (n, p), (_, q) in zip(model.state_dict().items(), model2.state_dict().items(), strict=True):
        assert torch.equal(p, q), n
    # identical next step from the restored optimizer state
    for mdl, o in ((model, opt), (model2, opt2)):
        o.zero_grad()
        mdl.loss(x, x, torch.ones(2, 16)).backward()
        o.step()
    for (n, p), (_, q) in zip(model.state_dict().items(), model2.state_dict().items(), strict=True):
        assert torch.allclose(p, q, atol=1e-6), n


def test_checkpoint_loads_into_reference_model(reference_mint, tmp_path):
    import mint.models.gemma as RG

    from mint_b200.models.gemma import Gemma, GemmaConfig
    from mint_b200.utils.checkpointer import consolidated_state_dict

    cfg = dict(embed_dim=32, hidden_dim=64, seq_length=16, vocab_size=50, n_layers=2, n_heads=2, n_kv_heads=1, head_dim=16)
    ours = Gemma(GemmaConfig(**cfg))
    ref = RG.Gemma(RG.GemmaConfig(**cfg), gradient_checkpointing=False)
    ref.load_state_dict(consolidated_state_dict(ours))
    x = torch.randint(0, 50, (1, 16))
    assert torch.allclose(ref(x), ours(x), atol=1e-5)


def test_qlora_nf4_roundtrip_and_training():
    from mint_b200.models.gemma import Gemma, GemmaConfig
    from mint_b200.sft.peft import LoRA, QLoRA
    from mint_b200.sft.peft.qlora import nf4_dequantize, nf4_quantize

    w = torch.randn(96, 64)
    q = nf4_quantize(w)
    err = (nf4_dequantize(q) - w).abs().mean() / w.abs().mean()
    assert err < 0.12
    assert q["packed"].dtype == torch.uint8 and q["packed"].numel() == w.numel() // 2
    for adapter in (LoRA, QLoRA):
        model = Gemma(GemmaConfig(embed_dim=64, hidden_dim=128, seq_length=16, vocab_size=50, n_layers=1, n_heads=2,
                                  n_kv_heads=2, head_dim=32))
        adapter.apply(model, target_modules=["wq", "wv"], r=4, alpha=8)
        trainable = [n for n, p in model.named_parameters() if p.requires_grad]
        assert trainable and all("lora" in n for n in trainable)
        x = torch.randint(0, 50, (2, 16))
        model.loss(x, x, torch.ones(2, 16)).backward()
        assert all(p.grad is not None for n, p in model.named_parameters() if p.requires_grad)


def test_exec_sandbox_timeout():
    from mint_b200.utils.exec import execute_code

    assert execute_code("print(1+1)").output.strip() == "2"
    res = execute_code("while True: pass", timeout=1)
    assert not res.success and "Timeout" in res.error


def test_step_profiler_windows(tmp_path):
    """wait 1, warmup 1, active 2, repeat 2: two recording windows, each with a trace and a kernel table."""
    import torch

    from mint_b200.utils.profiler import ProfilerConfig, StepProfiler

    cfg = ProfilerConfig(enabled=True, output_dir=str(tmp_path), schedule_wait=1, schedule_warmup=1,
                         schedule_active=2, schedule_repeat=2, activities=["cpu"], run_name="r",
                         profile_memory=False, with_flops=False)
    x = torch.randn(64, 64)
    with StepProfiler(cfg) as prof:
        for _ in range(12):
            (x @ x).sum()
            prof.step()
    files = sorted(p.name for p in (tmp_path / "r").iterdir())
    assert files == ["trace_rank0_w0.json", "trace_rank0_w0.kernels.txt",
                     "trace_rank0_w1.json", "trace_rank0_w1.kernels.txt"], files


def test_execute_code_isolated_process():
    from mint_b200.utils.exec import execute_code

    res = execute_code("import sys; print('out'); sys.exit(3)")
    assert not res.success and res.output.strip() == "out"
    res = execute_code("import os, time\nos.fork()\ntime.sleep(30)", timeout=1)
    assert not res.success and res.error.startswith("Timeout")
