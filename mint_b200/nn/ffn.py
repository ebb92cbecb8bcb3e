"""GeGLU feed-forward ``fc3(gelu_tanh(fc1 x) * fc2 x)`` (mint/nn/ffn.py:5-15).

On CUDA the whole MLP is two GEMMs with the GeGLU in their epilogues (``ops.glu.geglu_mlp``):
fc1 and fc2 run as one GEMM over ``[W1; W2]`` that also writes ``h``, and the backward's fc3
input-gradient GEMM writes ``d[a | b]`` directly. Under tensor parallelism with the fused
collectives, the GEMMs carry the collectives instead and GeGLU is a separate kernel.
"""

from __future__ import annotations

import torch
from torch import nn

from mint_b200.nn.base import compute_dtype
from mint_b200.ops.glu import geglu, geglu_mlp, geglu_mlp_fusable
from mint_b200.ops.linear import linear
from mint_b200.parallel import fused as fused_tp
from mint_b200.parallel import tp as tpc


class GLU(nn.Module):
    def __init__(self, embed_dim: int, hidden_dim: int, dtype: torch.dtype) -> None:
        super().__init__()
        self.fc1 = nn.Linear(embed_dim, hidden_dim, dtype=dtype, bias=False)
        self.fc2 = nn.Linear(embed_dim, hidden_dim, dtype=dtype, bias=False)
        self.fc3 = nn.Linear(hidden_dim, embed_dim, dtype=dtype, bias=False)
        self.tp: tpc.TPInfo | None = None

    def _fusable(self) -> bool:
        return all(type(m) is nn.Linear for m in (self.fc1, self.fc2, self.fc3))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        dt = compute_dtype(x)
        if self._fusable() and dt == torch.bfloat16 and fused_tp.enabled(self.tp, x):
            # fc1||fc2 GEMM with its all-gather (SP) / backward all-reduce (no SP), fc3 GEMM with its
            # reduce-scatter (SP) / all-reduce (no SP), as fused kernels
            ab = fused_tp.column_parallel_linear(x, (self.fc1.weight, self.fc2.weight), self.tp)
            return fused_tp.row_parallel_linear(geglu(ab), self.fc3.weight, self.tp)
        x = tpc.enter_column_parallel(x, self.tp)
        if self._fusable() and geglu_mlp_fusable(x, self.fc1.weight, self.fc2.weight, self.fc3.weight, dt):
            # GeGLU inside the fc1||fc2 GEMM's epilogue and its backward inside fc3's dgrad epilogue
            out = geglu_mlp(x, self.fc1.weight, self.fc2.weight, self.fc3.weight, compute_dtype=dt)
        elif self._fusable():
            ab = linear(x, self.fc1.weight, self.fc2.weight, compute_dtype=dt)
            h = geglu(ab)
            out = linear(h, self.fc3.weight, compute_dtype=dt)
        else:
            a = self.fc1(x)
            b = self.fc2(x)
            h = geglu(torch.cat([a, b], dim=-1))
            out = self.fc3(h)
        return tpc.exit_row_parallel(out, self.tp)
