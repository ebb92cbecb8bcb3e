"""Optimizer kernels (csrc/optim_kernels.cu) against plain PyTorch fp32 references: the device-side
NorMuon stack, the multi-segment squared norm and clip coefficient, the batched fp32 -> bf16 weight
copies, AdamW with a device clip scale, the status-word gate of the update kernels, and the
FMA-pipe exponential used by attention (error bound and NaN propagation)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _C():
    from mint_b200.ops import _ext

    return _ext.require()


@pytest.mark.parametrize("shape,n", [((768, 768), 4), ((3072, 768), 3), ((768, 3072), 2), ((256, 512), 3)])
def test_normuon_stack_matches_eager(shape, n):
    from mint_b200.optim.functional import NorMuonStack, normuon_update_batched

    torch.manual_seed(0)
    rows, cols = shape
    dev = "cuda"
    params = [torch.randn(rows, cols, device=dev) * 0.02 for _ in range(n)]
    grads = [torch.randn(rows, cols, device=dev) * 1e-3 for _ in range(n)]
    sshape = (rows, 1) if rows >= cols else (1, cols)
    mb = torch.randn(n, rows, cols, device=dev) * 1e-3
    smb = torch.rand(n, *sshape, device=dev) * 1e-2
    scale = torch.tensor([0.7], device=dev)
    # eager fp32 reference on copies (the eager path orthogonalizes in fp32 on CPU)
    ref_p = [p.detach().cpu().clone() for p in params]
    ref_g = torch.stack([g.cpu() for g in grads]) * 0.7
    ref_mb, ref_smb = mb.cpu().clone(), smb.cpu().clone()
    normuon_update_batched(ref_p, ref_g, ref_mb, ref_smb, lr=0.02, momentum=0.95, beta2=0.9, wd=0.1, ns_steps=5)

    old = [p.detach().cpu().clone() for p in params]
    stack = NorMuonStack(params, grads, mb, smb.view(n, -1))
    stack.step(lr=0.02, momentum=0.95, beta2=0.9, wd=0.1, ns_steps=5, grad_scale=scale)
    torch.cuda.synchronize()
    assert torch.allclose(mb.cpu(), ref_mb, rtol=1e-5, atol=1e-8)
    # the second moments come from the bf16 Polar-Express output on the device (fp32 on the CPU)
    assert torch.allclose(smb.cpu(), ref_smb, rtol=5e-2, atol=1e-6)
    for p0, p, r in zip(old, params, ref_p):
        got, want = p.cpu() - p0, r - p0  # the two updates
        err = (got - want).norm() / want.norm()
        assert err < 5e-2, err.item()


def test_sumsq_multi_and_clip_coef():
    C = _C()
    torch.manual_seed(1)
    segs = [torch.randn(n, device="cuda") for n in (1, 7, 4096, 100003)]
    base = torch.randn(64 + 3, device="cuda")
    segs.append(base[3:])  # an unaligned start
    ptrs = torch.tensor([t.data_ptr() for t in segs], dtype=torch.int64, device="cuda")
    sizes = torch.tensor([t.numel() for t in segs], dtype=torch.int64, device="cuda")
    out = torch.zeros(1, device="cuda")
    C.sumsq_multi(ptrs, sizes, out, max(t.numel() for t in segs))
    want = sum(float(t.double().square().sum()) for t in segs)
    assert abs(float(out) - want) / want < 1e-5
    coef, norm = torch.empty(1, device="cuda"), torch.empty(1, device="cuda")
    C.clip_coef(out, 1.0, coef, norm)
    assert abs(float(norm) - want ** 0.5) / want ** 0.5 < 1e-5
    assert abs(float(coef) - min(1.0, 1.0 / (want ** 0.5 + 1e-6))) < 1e-6


def test_cast_multi():
    C = _C()
    torch.manual_seed(2)
    src = [torch.randn(n, device="cuda") for n in (8, 12, 3, 65536 + 4)]
    dst = [torch.empty(t.numel(), dtype=torch.bfloat16, device="cuda") for t in src]
    table = [torch.tensor([t.data_ptr() for t in lst], dtype=torch.int64, device="cuda") for lst in (src, dst)]
    sizes = torch.tensor([t.numel() for t in src], dtype=torch.int64, device="cuda")
    C.cast_multi(table[0], table[1], sizes, max(t.numel() for t in src))
    for s, d in zip(src, dst):
        assert torch.equal(d, s.to(torch.bfloat16))


def test_adamw_device_clip_scale():
    from mint_b200.optim.functional import adamw_update

    torch.manual_seed(3)
    n = 4099
    p, g = torch.randn(n, device="cuda"), torch.randn(n, device="cuda")
    m, v = torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    rp, rm, rv = p.cpu().clone(), m.cpu().clone(), v.cpu().clone()
    adamw_update(rp, g.cpu() * 0.25, rm, rv, 1, 1e-3, 0.9, 0.95, 1e-8, 0.1)
    adamw_update(p, g, m, v, 1, 1e-3, 0.9, 0.95, 1e-8, 0.1, grad_scale=torch.tensor([0.25], device="cuda"))
    assert torch.allclose(p.cpu(), rp, rtol=1e-5, atol=1e-7)
    assert torch.allclose(v.cpu(), rv, rtol=1e-5, atol=1e-12)


def test_update_kernels_skip_after_a_kernel_error():
    """A non-zero status word (here written by the test itself) makes AdamW leave its inputs alone."""
    from mint_b200.ops import _ext
    from mint_b200.optim.functional import adamw_update

    C = _C()
    _ext.check_device_status()  # start clean
    st = C.status_tensor()
    p, g = torch.randn(1024, device="cuda"), torch.randn(1024, device="cuda")
    m, v = torch.zeros(1024, device="cuda"), torch.zeros(1024, device="cuda")
    before = p.clone()
    st.fill_(1 << 3)
    try:
        adamw_update(p, g, m, v, 1, 1e-2, 0.9, 0.95, 1e-8, 0.0)
        torch.cuda.synchronize()
        assert torch.equal(p, before) and int(m.abs().sum()) == 0
        with pytest.raises(_ext.DeviceStatusError):
            _ext.check_device_status()
    finally:
        C.read_status(True)
    adamw_update(p, g, m, v, 1, 1e-2, 0.9, 0.95, 1e-8, 0.0)
    torch.cuda.synchronize()
    assert not torch.equal(p, before)


def test_wait_limit_roundtrip():
    from mint_b200.ops import _ext

    old = _ext.wait_limit()
    try:
        _ext.set_wait_limit(0.25)
        assert abs(_ext.wait_limit() - 0.25) < 1e-9
    finally:
        _ext.set_wait_limit(old)
    assert abs(_ext.wait_limit() - old) < 1e-9


def test_exp2_poly_bound_and_nan():
    C = _C()
    x = torch.linspace(-130.0, 0.0, 2_000_001, device="cuda")
    y = C.exp2_poly_eval(x)
    ref = torch.exp2(x.double())
    ok = x >= -125.0
    rel = ((y.double() - ref).abs() / ref)[ok]
    assert float(rel.max()) <= 1e-4
    assert torch.all(y[~ok] == 0)
    special = torch.tensor([float("nan"), float("-inf"), -126.0, 0.0], device="cuda")
    out = C.exp2_poly_eval(special).cpu()
    assert torch.isnan(out[0])
    assert out[1] == 0 and out[2] == 0 and abs(float(out[3]) - 1.0) < 1e-4
