"""Tensor ops of the framework.

Every op has a PyTorch reference implementation (CPU tensors, numerics oracles) and an
sm_100a CUDA implementation from ``mint_b200._C`` used for every CUDA tensor.
"""

from mint_b200.ops.attention import attention
from mint_b200.ops.cross_entropy import masked_cross_entropy, vocab_parallel_cross_entropy
from mint_b200.ops.embedding import embedding
from mint_b200.ops.glu import geglu
from mint_b200.ops.linear import linear
from mint_b200.ops.norm import add_rmsnorm, rmsnorm
from mint_b200.ops.rope import qk_norm_rope, rope_cos_sin

__all__ = [
    "add_rmsnorm",
    "attention",
    "embedding",
    "geglu",
    "linear",
    "masked_cross_entropy",
    "qk_norm_rope",
    "rmsnorm",
    "rope_cos_sin",
    "vocab_parallel_cross_entropy",
]
