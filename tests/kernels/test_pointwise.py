"""Norm / RoPE / GeGLU / embedding / cross-entropy / AdamW kernels vs PyTorch fp32 references."""

import math

import pytest
import torch
import torch.nn.functional as F

from mint_b200.ops import add_rmsnorm, embedding, geglu, qk_norm_rope, rmsnorm, rope_cos_sin
from mint_b200.ops.cross_entropy import lm_head_cross_entropy, lm_head_token_logps, masked_cross_entropy

pytestmark = pytest.mark.gpu


def rms_ref(x, s, eps=1e-6):
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * (1 + s.float())


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("D", [64, 768, 2048])
def test_rmsnorm(dtype, D):
    torch.manual_seed(0)
    x = torch.randn(333, D, device="cuda", dtype=dtype, requires_grad=True)
    s = (0.1 * torch.randn(D, device="cuda")).requires_grad_()
    y = rmsnorm(x, s, out_dtype=torch.bfloat16)
    g = torch.randn_like(y)
    (y.float() * g.float()).sum().backward()
    gx, gs = x.grad.clone(), s.grad.clone()
    x2 = x.detach().clone().float().requires_grad_()
    s2 = s.detach().clone().requires_grad_()
    y2 = rms_ref(x2, s2)
    (y2 * g.float()).sum().backward()
    assert (y.float() - y2).abs().max() < 3e-2
    assert ((gx.float() - x2.grad).norm() / x2.grad.norm()) < 1e-2
    assert ((gs - s2.grad).norm() / s2.grad.norm()) < 1e-3


def test_add_rmsnorm():
    torch.manual_seed(1)
    D = 768
    res = torch.randn(500, D, device="cuda", requires_grad=True)
    a = torch.randn(500, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    post = (0.1 * torch.randn(D, device="cuda")).requires_grad_()
    pre = (0.1 * torch.randn(D, device="cuda")).requires_grad_()
    h, y = add_rmsnorm(res, a, post, pre, y_dtype=torch.bfloat16)
    gh, gy = torch.randn_like(h), torch.randn_like(y)
    ((h * gh).sum() + (y.float() * gy.float()).sum()).backward()
    out = [t.grad.clone() for t in (res, a, post, pre)]
    r2, a2 = res.detach().clone().requires_grad_(), a.detach().float().clone().requires_grad_()
    p2, q2 = post.detach().clone().requires_grad_(), pre.detach().clone().requires_grad_()
    h2 = r2 + rms_ref(a2, p2)
    y2 = rms_ref(h2, q2)
    ((h2 * gh).sum() + (y2 * gy.float()).sum()).backward()
    assert (h - h2).abs().max() < 2e-2
    assert (y.float() - y2).abs().max() < 5e-2
    for got, want in zip(out, (r2.grad, a2.grad, p2.grad, q2.grad)):
        assert ((got.float() - want).norm() / want.norm()) < 2e-2


@pytest.mark.parametrize("hq,hkv,D", [(6, 6, 128), (16, 4, 128), (4, 2, 16), (8, 1, 64)])
def test_qk_norm_rope(hq, hkv, D):
    torch.manual_seed(2)
    B, T = 2, 96
    qkv = torch.randn(B, T, (hq + 2 * hkv) * D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    qs = (0.1 * torch.randn(D, device="cuda")).requires_grad_()
    ks = (0.1 * torch.randn(D, device="cuda")).requires_grad_()
    cos, sin = rope_cos_sin(T + 8, D, 10000.0)
    cos, sin = cos.cuda(), sin.cuda()
    q, k, v = qk_norm_rope(qkv, hq, hkv, D, qs, ks, cos, sin, start_pos=4)
    gq, gk, gv = torch.randn_like(q), torch.randn_like(k), torch.randn_like(v)
    ((q.float() * gq.float()).sum() + (k.float() * gk.float()).sum() + (v.float() * gv.float()).sum()).backward()
    got = [qkv.grad.clone(), qs.grad.clone(), ks.grad.clone()]

    x = qkv.detach().float().clone().requires_grad_()
    qs2, ks2 = qs.detach().clone().requires_grad_(), ks.detach().clone().requires_grad_()
    q2 = rms_ref(x[..., : hq * D].reshape(B, T, hq, D), qs2)
    k2 = rms_ref(x[..., hq * D : (hq + hkv) * D].reshape(B, T, hkv, D), ks2)
    v2 = x[..., (hq + hkv) * D :].reshape(B, T, hkv, D)
    c = cos[4 : 4 + T][None, :, None, :]
    s = sin[4 : 4 + T][None, :, None, :]

    def rot(t):
        h = D // 2
        return torch.cat([t[..., :h] * c - t[..., h:] * s, t[..., :h] * s + t[..., h:] * c], -1)

    q2, k2 = rot(q2), rot(k2)
    ((q2 * gq.float()).sum() + (k2 * gk.float()).sum() + (v2 * gv.float()).sum()).backward()
    assert (q.float() - q2).abs().max() < 5e-2 and (k.float() - k2).abs().max() < 5e-2
    assert torch.equal(v.float(), v2)
    for a_, b_ in zip(got, (x.grad, qs2.grad, ks2.grad)):
        assert ((a_.float() - b_).norm() / b_.norm()) < 2e-2


def test_geglu():
    torch.manual_seed(3)
    ab = torch.randn(300, 2 * 3072, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    h = geglu(ab)
    g = torch.randn_like(h)
    (h.float() * g.float()).sum().backward()
    x = ab.detach().float().clone().requires_grad_()
    a, b = x.chunk(2, -1)
    h2 = F.gelu(a, approximate="tanh") * b
    (h2 * g.float()).sum().backward()
    assert (h.float() - h2).abs().max() < 5e-2
    assert ((ab.grad.float() - x.grad).norm() / x.grad.norm()) < 1e-2


def test_embedding():
    torch.manual_seed(4)
    w = torch.randn(1000, 768, device="cuda", requires_grad=True)
    ids = torch.randint(0, 1000, (4, 64), device="cuda")
    out = embedding(ids, w)
    g = torch.randn_like(out)
    (out * g).sum().backward()
    w2 = w.detach().clone().requires_grad_()
    out2 = F.embedding(ids, w2)
    (out2 * g).sum().backward()
    assert torch.equal(out, out2)
    assert (w.grad - w2.grad).abs().max() < 1e-4
    # vocab-parallel shard
    wshard = w.detach()[500:].clone()
    outp = embedding(ids, wshard, 500, vocab_parallel=True)
    exp = torch.where((ids >= 500)[..., None], F.embedding((ids - 500).clamp(min=0), wshard), 0.0)
    assert torch.equal(outp, exp)


@pytest.mark.parametrize("V,valid", [(65536, 65536), (50304, 50267), (1000, 1000)])
def test_lm_head_ce(V, valid):
    torch.manual_seed(5)
    M, D = 512, 256
    h = (torch.randn(M, D, device="cuda") * 0.5).requires_grad_()
    w = (torch.randn(V, D, device="cuda") * 0.1).requires_grad_()
    t = torch.randint(0, valid, (M,), device="cuda")
    m = (torch.rand(M, device="cuda") > 0.2).float()
    loss = lm_head_cross_entropy(h, w, t, m, valid, compute_dtype=torch.bfloat16)
    (loss * 0.7).backward()
    h2, w2 = h.detach().clone().requires_grad_(), w.detach().clone().requires_grad_()
    logits = h2.bfloat16().float() @ w2.bfloat16().float().t()
    l2 = masked_cross_entropy(logits, t, m, valid if V > valid else None)
    (l2 * 0.7).backward()
    assert abs(loss.item() - l2.item()) < 2e-2 * max(1, abs(l2.item()))
    assert ((h.grad - h2.grad).norm() / h2.grad.norm()) < 3e-2
    assert ((w.grad - w2.grad).norm() / w2.grad.norm()) < 3e-2


@pytest.mark.parametrize("V,valid", [(65536, 65536), (50304, 50267)])
def test_lm_head_token_logps(V, valid):
    """Fused DPO log-probs (LM-head GEMM + row statistics, in-place gradient with per-token weights)
    against fp32 log_softmax + gather, values and both input gradients."""
    torch.manual_seed(7)
    B, T, D = 2, 256, 256
    h = (torch.randn(B, T, D, device="cuda") * 0.5).requires_grad_()
    w = (torch.randn(V, D, device="cuda") * 0.1).requires_grad_()
    t = torch.randint(0, valid, (B, T), device="cuda")
    g = torch.randn(B, T, device="cuda")
    lp = lm_head_token_logps(h, w, t, valid, compute_dtype=torch.bfloat16)
    (lp * g).sum().backward()
    h2, w2 = h.detach().clone().requires_grad_(), w.detach().clone().requires_grad_()
    logits = h2.bfloat16().float() @ w2.bfloat16().float().t()
    if V > valid:
        logits = logits.masked_fill(torch.arange(V, device="cuda") >= valid, float("-inf"))
    lp2 = torch.log_softmax(logits, dim=-1).gather(-1, t.unsqueeze(-1)).squeeze(-1)
    (lp2 * g).sum().backward()
    assert lp.shape == (B, T) and lp.dtype == torch.float32
    assert (lp - lp2).abs().max().item() < 5e-2
    assert ((h.grad - h2.grad).norm() / h2.grad.norm()) < 3e-2
    assert ((w.grad - w2.grad).norm() / w2.grad.norm()) < 3e-2


def test_adamw_kernel():
    from mint_b200.optim.functional import adamw_update

    torch.manual_seed(6)
    n = 10007
    p = torch.randn(n, device="cuda")
    g = torch.randn(n, device="cuda")
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    pc, mc, vc = p.cpu().clone(), m.cpu().clone(), v.cpu().clone()
    for step in range(1, 4):
        adamw_update(p, g, m, v, step, 0.01, 0.8, 0.95, 1e-10, 0.1)
        # CPU reference path
        pc.mul_(1 - 0.01 * 0.1)
        mc.lerp_(g.cpu(), 0.2)
        vc.lerp_(g.cpu().square(), 0.05)
        denom = (vc / (1 - 0.95**step)).sqrt() + 1e-10
        pc.add_(mc / denom, alpha=-(0.01 / (1 - 0.8**step)))
    assert (p.cpu() - pc).abs().max() < 1e-5
    assert math.isfinite(p.sum().item())


@pytest.mark.parametrize("D", [256, 768, 1024])
def test_add_rmsnorm_without_pre(D):
    """h = res + rmsnorm(a) only (the block's post-FFN residual): register-resident backward for
    D <= 768, the general kernel above."""
    torch.manual_seed(2)
    res = torch.randn(300, D, device="cuda", requires_grad=True)
    a = torch.randn(300, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    post = (0.1 * torch.randn(D, device="cuda")).requires_grad_()
    h, _ = add_rmsnorm(res, a, post, None)
    gh = torch.randn_like(h)
    (h * gh).sum().backward()
    out = [t.grad.clone() for t in (res, a, post)]
    r2, a2 = res.detach().clone().requires_grad_(), a.detach().float().clone().requires_grad_()
    p2 = post.detach().clone().requires_grad_()
    h2 = r2 + rms_ref(a2, p2)
    (h2 * gh).sum().backward()
    for got, want in zip(out, (r2.grad, a2.grad, p2.grad)):
        assert ((got.float() - want).norm() / want.norm()) < 2e-2
