"""CPU parity of the model, loss and optimizer math against the reference implementation."""

import pytest
import torch

from mint_b200.models.gemma import Gemma, GemmaConfig
from mint_b200.ops.cross_entropy import masked_cross_entropy

CFG = dict(embed_dim=64, hidden_dim=128, seq_length=32, vocab_size=100, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=16)


def _pair(reference_mint, **over):
    import mint.models.gemma as RG

    cfg = {**CFG, **over}
    torch.manual_seed(0)
    ref = RG.Gemma(RG.GemmaConfig(**cfg), gradient_checkpointing=False)
    with torch.no_grad():
        for p in ref.parameters():
            p.normal_(0, 0.1)
    ours = Gemma(GemmaConfig(**cfg))
    ours.load_state_dict(ref.state_dict(), strict=True)
    return ref, ours


@pytest.mark.parametrize("over", [{}, {"n_kv_heads": 4}, {"n_kv_heads": 1}, {"pad_vocab_multiple": 64}])
def test_forward_backward_matches_reference(reference_mint, over):
    ref, ours = _pair(reference_mint, **over)
    torch.manual_seed(1)
    x = torch.randint(0, 100, (2, 32))
    y = torch.randint(0, 100, (2, 32))
    m = (torch.rand(2, 32) > 0.3).float()
    lr, lo = ref(x), ours(x)
    assert torch.allclose(lr, lo, atol=1e-5)
    from mint.trainer.base import _masked_cross_entropy as rce

    vocab = 100 if over.get("pad_vocab_multiple", 1) > 1 else None
    l1 = rce(ref(x, unpad_logits=False), y, m, vocab)
    l2 = ours.loss(x, y, m)
    assert abs(l1.item() - l2.item()) < 1e-5
    l1.backward()
    l2.backward()
    for (n1, p1), (_n2, p2) in zip(ref.named_parameters(), ours.named_parameters(), strict=True):
        assert torch.allclose(p1.grad, p2.grad, atol=1e-5, rtol=1e-4), n1


def test_doc_ids_and_window_masks(reference_mint):
    ref, ours = _pair(reference_mint)
    x = torch.randint(0, 100, (2, 32))
    doc = (torch.arange(32) // 10).expand(2, -1)
    # the reference's flash_attn varlen path needs CUDA; its SDPA fallback is the oracle on CPU
    import mint.nn.flashattn as rf

    saved = rf.flash_attn_varlen_func
    rf.flash_attn_varlen_func = None
    try:
        assert torch.allclose(ref(x, doc_ids=doc), ours(x, doc_ids=doc), atol=1e-5)
    finally:
        rf.flash_attn_varlen_func = saved


def test_kv_cache_generate_matches_full_forward():
    torch.manual_seed(3)
    model = Gemma(GemmaConfig(**CFG)).eval()
    x = torch.randint(0, 100, (1, 8))
    full = model.generate(x, 6, temperature=0)
    cached = model.generate(x, 6, temperature=0, use_cache=True)
    assert torch.equal(full, cached)
    # HF-style kwargs accepted (ChatCORE)
    out = model.generate(x, 2, attention_mask=torch.ones_like(x), pad_token_id=0, do_sample=False, use_cache=True)
    assert out.shape == (1, 10)


def test_masked_ce_matches_reference(reference_mint):
    from mint.trainer.base import _masked_cross_entropy as rce

    torch.manual_seed(4)
    logits = torch.randn(2, 7, 128)
    t = torch.randint(0, 100, (2, 7))
    m = torch.tensor([[1, 1, 0, 1, 1, 1, 0], [0, 0, 0, 0, 0, 0, 0]]).float()
    assert torch.allclose(rce(logits, t, m, 100), masked_cross_entropy(logits, t, m, 100))


def test_positional_variants_run():
    for pos in ("nope", "alibi", "sinusoidal", "linear_rope"):
        model = Gemma(GemmaConfig(**CFG, pos_embedding=pos))
        x = torch.randint(0, 100, (2, 32))
        out = model(x)
        out.sum().backward()
        assert torch.isfinite(out).all()


def test_adamw_and_muon_math_match_reference(reference_mint):
    from mint.optim.muon_adamw import MuonAdamW as RefOpt

    from mint_b200.optim.muon_adamw import MuonAdamW

    torch.manual_seed(5)
    w0 = torch.randn(48, 32)
    s0 = torch.randn(32)
    grads = [(torch.randn(48, 32), torch.randn(32)) for _ in range(3)]

    def run(cls, compiled_off):
        w = torch.nn.Parameter(w0.clone())
        s = torch.nn.Parameter(s0.clone())
        groups = [
            {"kind": "muon", "params": [w], "lr": 0.02, "momentum": 0.95, "beta2": 0.9, "weight_decay": 0.1, "ns_steps": 5},
            {"kind": "adamw", "params": [s], "lr": 0.01, "betas": (0.8, 0.95), "eps": 1e-10, "weight_decay": 0.05},
        ]
        opt = cls(groups)
        if compiled_off:
            opt._fused_adam = opt._adamw_step_fused
        for gw, gs in grads:
            w.grad, s.grad = gw.clone(), gs.clone()
            opt.step()
        return w.detach(), s.detach()

    wr, sr = run(RefOpt, True)
    wo, so = run(MuonAdamW, False)
    assert torch.allclose(wr, wo, atol=1e-5)
    assert torch.allclose(sr, so, atol=1e-6)
