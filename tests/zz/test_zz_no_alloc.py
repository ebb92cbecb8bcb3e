"""The allocation-free FlashAttention backward (`mint_flash_attn_bwd_noalloc`, a C symbol of the
extension library) against the regular `flash_attn_bwd` binding.

The C entry point exists for callers that cannot allocate device memory while they run (a
pre-planned runtime, a plugin inside another framework's memory pool, plain C code without
PyTorch's allocator): it takes every output from the caller and keeps its fp32 work buffers in
one fixed device array inside the library. This test calls it through ctypes exactly as such a
caller would, twice in a row on different shapes (so the second call must clear what the first
left in the shared array), and checks the gradients against the ATen-allocating binding.
"""

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_ROWS = 32768  # MINT_FLASH_ATTN_BWD_NOALLOC_MAX_ROWS


def _lib():
    from mint_b200.ops import _ext

    mod = _ext.require()
    lib = ctypes.CDLL(mod.__file__)
    fn = lib.mint_flash_attn_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = ([ctypes.c_void_p] * 10 + [ctypes.c_int] * 6 +
                   [ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t])
    return mod, fn


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _call(fn, dout, q, k, v, o, lse, doc, dq, dk, dv, causal, window, scale, status):
    B, T, Hq, _ = q.shape
    Hkv = k.shape[2]
    err = ctypes.create_string_buffer(512)
    rc = fn(_ptr(dout), _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(lse), _ptr(doc), _ptr(dq), _ptr(dk), _ptr(dv),
            B, T, Hq, Hkv, int(causal), window, scale, _ptr(status),
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), err, len(err))
    return rc, err.value.decode()


def _case(mod, fn, seed, B, T, Hq, Hkv, causal, window, use_doc):
    torch.manual_seed(seed)
    D = 128
    q = torch.randn(B, T, Hq, D, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(B, T, Hkv, D, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(B, T, Hkv, D, device="cuda", dtype=torch.bfloat16)
    doc = ((torch.arange(T, device="cuda") // 70).expand(B, -1).contiguous().int() if use_doc else None)
    scale = 1.0 / math.sqrt(D)
    o, lse = mod.flash_attn_fwd(q, k, v, doc, causal, window, scale)
    dout = torch.randn_like(o)
    want = mod.flash_attn_bwd(dout, q, k, v, o, lse, doc, causal, window, scale)

    dq = torch.full_like(q, float("nan"))
    dk = torch.full_like(k, float("nan"))
    dv = torch.full_like(v, float("nan"))
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc, msg = _call(fn, dout, q, k, v, o, lse, doc, dq, dk, dv, causal, window, scale, status)
    assert rc == 0, msg
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    for name, got, ref in zip(("dq", "dk", "dv"), (dq, dk, dv), want):
        assert torch.isfinite(got.float()).all(), name
        rel = ((got.float() - ref.float()).norm() / ref.float().norm()).item()
        assert rel < 2e-2, f"{name} rel err {rel}"


def test_noalloc_matches_allocating_binding_twice():
    mod, fn = _lib()
    # the first call fills a larger part of the shared accumulator than the second one uses
    _case(mod, fn, 0, 2, 1024, 8, 2, True, -1, False)
    _case(mod, fn, 1, 1, 640, 4, 1, True, 200, True)


def test_noalloc_rejects_sizes_above_the_limit():
    mod, fn = _lib()
    B, T, Hq, Hkv = 1, MAX_ROWS // 4 + 128, 4, 4  # B*T*Hq = MAX_ROWS + 512
    q = torch.zeros(B, T, Hq, 128, device="cuda", dtype=torch.bfloat16)
    k = torch.zeros(B, T, Hkv, 128, device="cuda", dtype=torch.bfloat16)
    lse = torch.zeros(B, Hq, T, device="cuda")
    out = torch.empty_like(q)
    rc, msg = _call(fn, q, q, k, k, q, lse, None, out, out, out, True, -1, 0.1, None)
    assert rc == 2 and "limit" in msg


def test_noalloc_internal_status_word_reads_clean():
    """Calls made with status == NULL report into a word inside the library; the companion C
    function reads (and can clear) it, so such callers still learn about a timed-out wait."""
    mod, fn = _lib()
    _case(mod, fn, 2, 1, 512, 4, 4, True, -1, False)
    lib = ctypes.CDLL(mod.__file__)
    read = lib.mint_flash_attn_bwd_noalloc_status
    read.restype = ctypes.c_int
    read.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_uint)]
    out = ctypes.c_uint(123)
    assert read(1, ctypes.byref(out)) == 0
    assert out.value == 0
