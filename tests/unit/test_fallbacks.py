"""Fallback accounting: a CUDA call that runs PyTorch code instead of a kernel is counted, warns
once per (op, reason) and raises under ``MINT_STRICT_KERNELS=1``."""

import warnings

import pytest

from mint_b200.ops import _ext


def test_fallback_counts_warns_once_and_strict_raises(monkeypatch):
    _ext.reset_fallbacks()
    monkeypatch.delenv("MINT_STRICT_KERNELS", raising=False)
    with warnings.catch_warnings(record=True) as rec:
        warnings.simplefilter("always")
        _ext.fallback("matmul", "odd stride")
        _ext.fallback("matmul", "odd stride")
        _ext.fallback("attention", "mask")
    assert [str(w.message) for w in rec] == [
        "mint_b200: matmul ran its PyTorch fallback on CUDA (odd stride)",
        "mint_b200: attention ran its PyTorch fallback on CUDA (mask)",
    ]
    assert _ext.fallback_counts() == {"matmul: odd stride": 2, "attention: mask": 1}
    monkeypatch.setenv("MINT_STRICT_KERNELS", "1")
    with pytest.raises(RuntimeError, match="no kernel path"):
        _ext.fallback("matmul", "odd stride")
    _ext.reset_fallbacks()
    assert _ext.fallback_counts() == {}
