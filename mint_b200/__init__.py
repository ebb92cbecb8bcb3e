"""mint_b200: a Blackwell-native (sm_100a) LLM training framework.

Public surface mirrors nagarajpoojari404/mint (CLI sub-commands, TOML schema,
Gemma-style decoder, MuonAdamW, ZeRO-0..3, TP/SP on a dp x tp mesh, checkpoint
layout). Hot ops run as hand-written sm_100a CUDA kernels from ``mint_b200._C``.
"""

__version__ = "0.1.0"
