"""Run-to-run repeatability of the kernels (a race inside a kernel -- a missing barrier, a buffer
reused too early -- shows up as results that change between identical calls).

Deterministic by construction, so compared bitwise: attention forward (output and LSE), the
attention backward's dK / dV (each key tile is owned by one CTA), the LM-head cross-entropy loss
and the gradient of its input. The attention backward's dQ is summed with fp32 reduce-adds across
key tiles, whose order varies, so it is held to a tolerance far below the bf16 rounding."""

import pytest
import torch

from mint_b200.ops.attention import attention
from mint_b200.ops.cross_entropy import lm_head_cross_entropy

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("use_doc", [False, True])
def test_attention_repeatable(use_doc):
    torch.manual_seed(3)
    B, T, Hq, Hkv, D = 2, 1024, 4, 2, 128
    q0 = torch.randn(B, T, Hq, D, device="cuda", dtype=torch.bfloat16)
    k0 = torch.randn(B, T, Hkv, D, device="cuda", dtype=torch.bfloat16)
    v0 = torch.randn(B, T, Hkv, D, device="cuda", dtype=torch.bfloat16)
    do = torch.randn(B, T, Hq, D, device="cuda", dtype=torch.bfloat16)
    doc = (torch.arange(T, device="cuda") // 300).expand(B, -1).contiguous() if use_doc else None
    runs = []
    for _ in range(3):
        q, k, v = (t.clone().requires_grad_() for t in (q0, k0, v0))
        o = attention(q, k, v, causal=True, window_left=-1, doc_ids=doc)
        (o.float() * do.float()).sum().backward()
        runs.append((o.detach(), q.grad, k.grad, v.grad))
    for o, dq, dk, dv in runs[1:]:
        assert torch.equal(o, runs[0][0])
        assert torch.equal(dk, runs[0][2])
        assert torch.equal(dv, runs[0][3])
        rel = ((dq.float() - runs[0][1].float()).norm() / runs[0][1].float().norm()).item()
        assert rel < 1e-3, rel


def test_lm_head_ce_repeatable():
    torch.manual_seed(4)
    M, D, V = 1024, 256, 65536
    h0 = torch.randn(M, D, device="cuda") * 0.5
    w = torch.randn(V, D, device="cuda") * 0.1
    t = torch.randint(0, V, (M,), device="cuda")
    m = torch.ones(M, device="cuda")
    runs = []
    for _ in range(3):
        h = h0.clone().requires_grad_()
        loss = lm_head_cross_entropy(h, w, t, m, V, compute_dtype=torch.bfloat16)
        loss.backward()
        runs.append((loss.detach(), h.grad))
    for loss, dh in runs[1:]:
        assert torch.equal(loss, runs[0][0])
        assert torch.equal(dh, runs[0][1])
