"""tcgen05 FlashAttention forward/backward vs an fp32 PyTorch reference (causal, sliding window,
document masks, GQA/MQA, sequence lengths that are not tile multiples)."""

import math

import pytest
import torch

from mint_b200.ops.attention import attention, build_mask

pytestmark = pytest.mark.gpu


def ref_attention(q, k, v, causal, window, doc):
    B, T, Hq, D = q.shape
    Hkv = k.shape[2]
    qf, kf, vf = (t.float().transpose(1, 2) for t in (q, k, v))
    kf = kf.repeat_interleave(Hq // Hkv, dim=1)
    vf = vf.repeat_interleave(Hq // Hkv, dim=1)
    s = qf @ kf.transpose(-1, -2) / math.sqrt(D)
    mask = build_mask(T, T, q.device, causal=causal, window_left=window, doc_ids=doc, attn_mask=None)
    if mask is not None:
        s = s.masked_fill(~mask, float("-inf"))
    p = torch.softmax(s, dim=-1)
    return (p @ vf).transpose(1, 2)


CASES = [
    # B, T, Hq, Hkv, causal, window, doc
    (2, 256, 2, 2, True, -1, False),
    (1, 384, 4, 1, True, -1, False),
    (2, 200, 4, 2, True, -1, False),
    (1, 512, 2, 2, True, 100, False),
    (2, 300, 4, 4, True, -1, True),
    (1, 256, 2, 1, False, -1, False),
    (1, 1024, 6, 6, True, 256, False),
    (2, 640, 4, 2, True, -1, "unsorted"),
    (1, 1024, 2, 2, True, 300, True),
    (1, 384, 2, 2, False, -1, True),
]


@pytest.mark.parametrize("B,T,Hq,Hkv,causal,window,use_doc", CASES)
def test_flash_attention_fwd_bwd(B, T, Hq, Hkv, causal, window, use_doc):
    torch.manual_seed(0)
    D = 128
    q = torch.randn(B, T, Hq, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(B, T, Hkv, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(B, T, Hkv, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    doc = None
    if use_doc == "unsorted":  # ids repeat non-contiguously: per-element id comparison, no tile skipping
        doc = ((torch.arange(T, device="cuda") // 70) % 3).expand(B, -1).contiguous()
    elif use_doc:
        doc = (torch.arange(T, device="cuda") // 70).expand(B, -1).contiguous()
    o = attention(q, k, v, causal=causal, window_left=window, doc_ids=doc)
    do = torch.randn_like(o)
    (o.float() * do.float()).sum().backward()
    got = [t.grad.clone() for t in (q, k, v)]
    q2, k2, v2 = (t.detach().float().clone().requires_grad_() for t in (q, k, v))
    o2 = ref_attention(q2, k2, v2, causal, window, doc)
    (o2 * do.float()).sum().backward()
    err = (o.float() - o2).abs().max().item()
    assert err < 3e-2, f"fwd max err {err}"
    for name, a, b in zip("qkv", got, (q2.grad, k2.grad, v2.grad)):
        rel = ((a.float() - b).norm() / b.norm()).item()
        assert rel < 2e-2, f"d{name} rel err {rel}"
    from mint_b200.ops import _ext

    assert _ext.require().read_status(False) == 0


def test_flash_attention_matches_model_path_shapes():
    """d12 attention shape (6 heads x 128, T=2048) with the windowed layer's window T/4."""
    torch.manual_seed(1)
    q = torch.randn(1, 2048, 6, 128, device="cuda", dtype=torch.bfloat16)
    k = torch.randn_like(q)
    v = torch.randn_like(q)
    for window in (-1, 512):
        o = attention(q, k, v, causal=True, window_left=window)
        o2 = ref_attention(q, k, v, True, window, None)
        assert (o.float() - o2).abs().max().item() < 3e-2


@pytest.mark.parametrize("B,Tq,Tk,Hq,Hkv,window", [(2, 1, 777, 8, 2, -1), (1, 4, 1500, 4, 4, -1), (3, 1, 96, 16, 1, -1),
                                                    (2, 2, 2048, 8, 2, 300), (1, 16, 600, 2, 2, -1)])
def test_decode_attention_kv_cache(B, Tq, Tk, Hq, Hkv, window):
    """Split-KV decode kernel against an fp32 reference: queries at the last Tq positions of a KV
    cache prefix (bottom-right causal), the cache read in place through a strided batch view."""
    from mint_b200.ops import _ext

    torch.manual_seed(3)
    Tmax = Tk + 64
    kc = torch.randn(B + 1, Tmax, Hkv, 128, device="cuda", dtype=torch.bfloat16)
    vc = torch.randn_like(kc)
    k, v = kc[:B, :Tk], vc[:B, :Tk]
    q = torch.randn(B, Tq, Hq, 128, device="cuda", dtype=torch.bfloat16)
    _ext.reset_fallbacks()
    with torch.no_grad():
        out = attention(q, k, v, causal=True, window_left=window)
    assert not _ext.fallback_counts()
    qf, kf, vf = (t.float().transpose(1, 2) for t in (q, k, v))
    kf = kf.repeat_interleave(Hq // Hkv, dim=1)
    vf = vf.repeat_interleave(Hq // Hkv, dim=1)
    s = qf @ kf.transpose(-1, -2) / math.sqrt(128)
    mask = build_mask(Tq, Tk, q.device, causal=True, window_left=window, doc_ids=None, attn_mask=None)
    p = torch.softmax(s.masked_fill(~mask, float("-inf")), dim=-1)
    want = (p @ vf).transpose(1, 2)
    assert (out.float() - want).abs().max().item() < 2e-2
