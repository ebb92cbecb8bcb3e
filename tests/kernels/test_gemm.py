"""tcgen05 GEMM vs a PyTorch fp32 reference: every operand major-ness, bf16 / fp32 output, alpha/beta."""

import pytest
import torch

from mint_b200.ops.gemm import matmul

pytestmark = pytest.mark.gpu


def ref(a, b, ta, tb, alpha=1.0, beta=0.0, d=None):
    a_ = a.float().t() if ta else a.float()
    b_ = b.float().t() if tb else b.float()
    c = alpha * (a_ @ b_)
    if d is not None:
        c = c + beta * d.float()
    return c


@pytest.mark.parametrize("ta", [False, True])
@pytest.mark.parametrize("tb", [False, True])
@pytest.mark.parametrize("shape", [(256, 512, 256), (384, 640, 192), (1000, 776, 328), (128, 128, 64), (300, 2304, 768)])
def test_gemm_layouts(ta, tb, shape):
    torch.manual_seed(0)
    M, N, K = shape
    a = torch.randn((K, M) if ta else (M, K), device="cuda", dtype=torch.bfloat16)
    b = torch.randn((N, K) if tb else (K, N), device="cuda", dtype=torch.bfloat16)
    out = matmul(a, b, trans_a=ta, trans_b=tb, out_dtype=torch.float32)
    torch.cuda.synchronize()
    exp = ref(a, b, ta, tb)
    err = (out - exp).abs().max().item()
    assert err < 1e-2 * max(1.0, exp.abs().max().item() / 50), f"max err {err}"


@pytest.mark.parametrize("ta,tb", [(False, True), (False, False), (True, False)])
def test_gemm_bf16_out_alpha_beta(ta, tb):
    torch.manual_seed(1)
    M, N, K = 512, 768, 1024
    a = torch.randn((K, M) if ta else (M, K), device="cuda", dtype=torch.bfloat16)
    b = torch.randn((N, K) if tb else (K, N), device="cuda", dtype=torch.bfloat16)
    d = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
    out = matmul(a, b, trans_a=ta, trans_b=tb, alpha=0.5, beta=-1.5, d=d, out_dtype=torch.bfloat16)
    exp = ref(a, b, ta, tb, 0.5, -1.5, d)
    rel = ((out.float() - exp).norm() / exp.norm()).item()
    assert rel < 1e-2, rel


def test_gemm_fp32_accumulate_inplace():
    torch.manual_seed(2)
    M, N, K = 768, 512, 4096
    a = torch.randn(K, M, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(K, N, device="cuda", dtype=torch.bfloat16)
    c = torch.randn(M, N, device="cuda", dtype=torch.float32)
    c0 = c.clone()
    matmul(a, b, trans_a=True, beta=1.0, d=c, out=c)
    exp = a.float().t() @ b.float() + c0
    rel = ((c - exp).norm() / exp.norm()).item()
    assert rel < 2e-3, rel


def test_gemm_large_lm_head_shape():
    torch.manual_seed(3)
    M, N, K = 4096, 65536, 768
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16) * 0.5
    b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.5
    out = matmul(a, b, trans_b=True, out_dtype=torch.bfloat16)
    exp = a.float() @ b.float().t()
    rel = ((out.float() - exp).norm() / exp.norm()).item()
    assert rel < 1e-2, rel
    from mint_b200.ops import _ext
    assert _ext.require().read_status(False) == 0


def test_gemm_repeatable():
    torch.manual_seed(4)
    a = torch.randn(640, 512, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(384, 512, device="cuda", dtype=torch.bfloat16)
    x = matmul(a, b, trans_b=True, out_dtype=torch.float32)
    y = matmul(a, b, trans_b=True, out_dtype=torch.float32)
    assert torch.equal(x, y)


@pytest.mark.parametrize("shape", [(768, 768, 65536), (2304, 768, 16384), (300, 200, 1000), (128, 256, 64)])
def test_gemm_split_k_accumulate(shape):
    """Weight-gradient shape: tiny output, huge contraction -> split-K with fp32 vector reductions."""
    torch.manual_seed(5)
    M, N, K = shape
    a = torch.randn(K, M, device="cuda", dtype=torch.bfloat16)  # dy [tokens, out]
    b = torch.randn(K, N, device="cuda", dtype=torch.bfloat16)  # x  [tokens, in]
    c = torch.randn(M, N, device="cuda", dtype=torch.float32)
    c0 = c.clone()
    matmul(a, b, trans_a=True, out=c, accumulate=True)
    matmul(a, b, trans_a=True, out=c, accumulate=True)
    exp = c0 + 2 * (a.float().t() @ b.float())
    rel = ((c - exp).norm() / exp.norm()).item()
    assert rel < 2e-3, rel


def test_gemm_column_slice_operand():
    """A strided column slice (fused-QKV weight-gradient rows) is a valid TMA operand."""
    torch.manual_seed(6)
    dy = torch.randn(4096, 2304, device="cuda", dtype=torch.bfloat16)
    x = torch.randn(4096, 768, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(768, 768, device="cuda")
    matmul(dy[:, 768:1536], x, trans_a=True, out=out, accumulate=True)
    exp = dy[:, 768:1536].float().t() @ x.float()
    assert ((out - exp).norm() / exp.norm()).item() < 2e-3


def test_gemm_unaligned_operand_is_a_counted_fallback(monkeypatch):
    """Rows of 14 bytes cannot be described to TMA: the call still returns the right product, but
    it is counted and warned about, and raises under MINT_STRICT_KERNELS=1."""
    from mint_b200.ops import _ext

    _ext.reset_fallbacks()
    a = torch.randn(64, 7, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(7, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.warns(RuntimeWarning, match="matmul ran its PyTorch fallback"):
        c = matmul(a, b)
    torch.testing.assert_close(c.float(), ref(a, b, False, False), rtol=2e-2, atol=2e-2)
    assert sum(_ext.fallback_counts().values()) == 1
    monkeypatch.setenv("MINT_STRICT_KERNELS", "1")
    with pytest.raises(RuntimeError, match="no kernel path"):
        matmul(a, b)
    _ext.reset_fallbacks()


@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True)])
@pytest.mark.parametrize("shape", [(5, 192, 320, 256), (3, 768, 768, 3072), (24, 128, 96, 64)])
def test_gemm_batched(ta, tb, shape):
    """3-D operands: one launch for a stack of equally shaped GEMMs (batched Polar Express), with
    the beta * D epilogue reading each batch's own D."""
    torch.manual_seed(2)
    nb, M, N, K = shape
    a = torch.randn((nb, K, M) if ta else (nb, M, K), device="cuda", dtype=torch.bfloat16)
    b = torch.randn((nb, N, K) if tb else (nb, K, N), device="cuda", dtype=torch.bfloat16)
    d = torch.randn(nb, M, N, device="cuda", dtype=torch.bfloat16)
    out = matmul(a, b, trans_a=ta, trans_b=tb, alpha=0.5, beta=-1.5, d=d, out_dtype=torch.float32)
    torch.cuda.synchronize()
    for i in range(nb):
        exp = ref(a[i], b[i], ta, tb, 0.5, -1.5, d[i])
        err = (out[i] - exp).abs().max().item()
        assert err < 1e-2 * max(1.0, exp.abs().max().item() / 50), f"batch {i} max err {err}"


@pytest.mark.parametrize("ta", [False, True])
@pytest.mark.parametrize("tb", [False, True])
def test_gemm_cta_pair_layouts(ta, tb):
    """Shapes large enough for the CTA-pair kernel (256-row tiles on 2 SMs, tcgen05 cta_group::2),
    with a ragged M and N so both CTAs of a pair see clipped rows and columns."""
    torch.manual_seed(3)
    M, N, K = 4100, 2336, 640
    a = torch.randn((K, M) if ta else (M, K), device="cuda", dtype=torch.bfloat16)
    b = torch.randn((N, K) if tb else (K, N), device="cuda", dtype=torch.bfloat16)
    d = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
    out = matmul(a, b, trans_a=ta, trans_b=tb, alpha=0.25, beta=2.0, d=d, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    exp = ref(a, b, ta, tb, 0.25, 2.0, d)
    rel = ((out.float() - exp).norm() / exp.norm()).item()
    assert rel < 1e-2, f"rel err {rel}"


def test_gemm_cta_pair_accumulate():
    """Weight-gradient form (A MN-major, fp32 C accumulated through TMA reduce-adds) on the pair kernel."""
    torch.manual_seed(4)
    M, N, K = 4096, 2304, 512
    a = torch.randn(K, M, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(K, N, device="cuda", dtype=torch.bfloat16)
    out = torch.randn(M, N, device="cuda", dtype=torch.float32)
    start = out.clone()
    matmul(a, b, trans_a=True, out=out, accumulate=True)
    torch.cuda.synchronize()
    exp = start + a.float().t() @ b.float()
    err = (out - exp).abs().max().item()
    assert err < 5e-2, f"max err {err}"


def test_gemm_cta_pair_split_k_accumulate():
    """A weight-gradient shape with too few 256 x 256 tiles to fill the GPU: CTA pairs plus split-K,
    each split's partial tile TMA-reduce-added into the fp32 gradient."""
    torch.manual_seed(5)
    M, N, K = 2304, 768, 8192
    a = torch.randn(K, M, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(K, N, device="cuda", dtype=torch.bfloat16)
    out = torch.randn(M, N, device="cuda", dtype=torch.float32)
    start = out.clone()
    matmul(a, b, trans_a=True, out=out, accumulate=True)
    torch.cuda.synchronize()
    exp = start + a.float().t() @ b.float()
    rel = ((out - exp).norm() / exp.norm()).item()
    assert rel < 1e-4, f"rel err {rel}"


@pytest.mark.parametrize("fused_bwd", [False, True])
@pytest.mark.parametrize("M,d,F", [(1000, 256, 384), (4096, 768, 3072), (300, 128, 128)])
def test_geglu_mlp_fused(M, d, F, fused_bwd, monkeypatch):
    """GeGLU inside the GEMM epilogues (forward: fc1||fc2 GEMM writes ab and h; backward, opt-in:
    the fc3 input-gradient GEMM writes d[a|b]) against fp32 PyTorch: output and every gradient."""
    from mint_b200.ops import glu
    from mint_b200.ops.glu import _GeGLUMLPFn, geglu_mlp_fusable

    monkeypatch.setattr(glu, "_FUSED_BWD", fused_bwd)

    torch.manual_seed(11)
    x = (torch.randn(M, d, device="cuda") * 0.5).requires_grad_()
    w1 = (torch.randn(F, d, device="cuda") * d ** -0.5).requires_grad_()
    w2 = (torch.randn(F, d, device="cuda") * d ** -0.5).requires_grad_()
    w3 = (torch.randn(d, F, device="cuda") * F ** -0.5).requires_grad_()
    assert geglu_mlp_fusable(x, w1, w2, w3, torch.bfloat16)
    gy = torch.randn(M, d, device="cuda")
    y = _GeGLUMLPFn.apply(x, torch.bfloat16, w1, w2, w3)
    (y.float() * gy).sum().backward()
    xs, a1, a2, a3 = (t.detach().clone().requires_grad_() for t in (x, w1, w2, w3))
    xb = xs.bfloat16().float()
    a = xb @ a1.bfloat16().float().t()
    b = xb @ a2.bfloat16().float().t()
    h = torch.nn.functional.gelu(a, approximate="tanh") * b
    y2 = h @ a3.bfloat16().float().t()
    (y2 * gy).sum().backward()

    def rel(u, v):
        return ((u.float() - v.float()).norm() / v.float().norm()).item()

    assert rel(y, y2) < 2e-2
    for got, want in ((x.grad, xs.grad), (w1.grad, a1.grad), (w2.grad, a2.grad), (w3.grad, a3.grad)):
        assert rel(got, want) < 3e-2, rel(got, want)
