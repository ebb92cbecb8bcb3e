"""Gemma-style decoder (mint/models/gemma.py:17-248) on the framework's fused ops.

Same ``GemmaConfig`` fields, module names and state-dict keys as the reference
(``tok_embeddings.weight``, ``blocks.{i}.{pre,post}_{attn,ffn}_norm.scale``,
``blocks.{i}.gqa.{wq,wk,wv,wo}.weight``, ``blocks.{i}.gqa.{q,k}_norm.scale``,
``blocks.{i}.ffn.fc{1,2,3}.weight``, ``norm.scale``, ``output.weight``), alternating
sliding-window ('S', even index) and global ('L') blocks, tied embeddings, optional vocab
padding, gradient checkpointing and sampling ``generate``.

Additions: ``loss()`` fuses the LM head with the masked cross-entropy (no logits tensor is
returned, the gradient logits are written in place); under tensor parallelism the embedding and
LM head are vocab-parallel and ``forward`` all-gathers the vocabulary shards.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import torch
import torch.distributed as dist
from torch import nn
from torch.utils.checkpoint import checkpoint

from mint_b200.kvcache.base import KVCache
from mint_b200.nn.base import ModelConfig, compute_dtype
from mint_b200.nn.blocks import GQAGluBlock
from mint_b200.nn.norm import RMSNorm
from mint_b200.ops.cross_entropy import lm_head_cross_entropy, lm_head_token_logps
from mint_b200.ops.embedding import embedding
from mint_b200.ops.linear import linear
from mint_b200.parallel import fused as fused_tp
from mint_b200.parallel import tp as tpc
from mint_b200.utils.logger import logger


def _default_tp_plan() -> dict[str, str]:
    return {
        "blocks.*.gqa.wq": "col",
        "blocks.*.gqa.wk": "col",
        "blocks.*.gqa.wv": "col",
        "blocks.*.gqa.wo": "row",
        "blocks.*.ffn.fc1": "col",
        "blocks.*.ffn.fc2": "col",
        "blocks.*.ffn.fc3": "row",
    }


@dataclass
class GemmaConfig(ModelConfig):
    embed_dim: int
    hidden_dim: int
    seq_length: int
    vocab_size: int
    n_layers: int
    dtype: torch.dtype = torch.float32
    n_heads: int = 12
    n_kv_heads: int = 4
    head_dim: int = 128
    rope_base_theta: int | float = 100000
    tie_weights: bool = True
    pad_vocab_multiple: int = 1
    tp_plan: dict[str, str] = field(default_factory=_default_tp_plan)
    # extensions (defaults reproduce the reference model exactly)
    pos_embedding: str = "rope"  # rope | linear_rope | nope | alibi | sinusoidal
    rope_scale_factor: float = 4.0  # LinearScaledRoPE interpolation factor
    window_divisor: int = 4  # 'S' blocks attend to seq_length // window_divisor keys
    attention_pattern: str = "SL"  # repeated over layers; 'S' windowed, 'L' global
    init_std: float = 0.0  # 0 -> PyTorch's default nn.Linear / nn.Embedding init (reference)


class Gemma(nn.Module):
    def __init__(self, config: GemmaConfig, *, gradient_checkpointing: bool = False) -> None:
        super().__init__()
        self.config = config
        self.gradient_checkpointing = gradient_checkpointing
        m = config.pad_vocab_multiple
        self.padded_vocab_size = (config.vocab_size + m - 1) // m * m
        self.tok_embeddings = nn.Embedding(self.padded_vocab_size, config.embed_dim, dtype=config.dtype)
        pattern = config.attention_pattern or "SL"
        self.blocks = nn.ModuleList(
            GQAGluBlock(
                n_heads=config.n_heads,
                n_kv_heads=config.n_kv_heads,
                head_dim=config.head_dim,
                embed_dim=config.embed_dim,
                hidden_dim=config.hidden_dim,
                seq_len=config.seq_length,
                rope_base_theta=config.rope_base_theta,
                dtype=config.dtype,
                attention_type=pattern[i % len(pattern)],
                pos_embedding=config.pos_embedding,
                rope_scale_factor=config.rope_scale_factor,
                window_divisor=config.window_divisor,
            )
            for i in range(config.n_layers)
        )
        self.norm = RMSNorm(config.embed_dim)
        self.output = nn.Linear(config.embed_dim, self.padded_vocab_size, bias=False, dtype=config.dtype)
        # set by mint_b200.parallel.apply_tp: vocab-parallel embedding / LM head
        self.tp: tpc.TPInfo | None = None
        self.vocab_start = 0
        # set by the ZeRO-3 engine: materializes sharded top-level parameters before a pass
        self._before_forward = None
        self.reset_parameters()

    def reset_parameters(self) -> None:
        # Module.to_empty breaks weight tying, so it is re-established after every re-init
        if self.config.tie_weights:
            self.output.weight = self.tok_embeddings.weight
        if self.config.init_std > 0 and not self.tok_embeddings.weight.is_meta:
            for p in self.parameters():
                if p.ndim == 2:
                    nn.init.normal_(p, std=self.config.init_std)

    # ------------------------------------------------------------------ forward pieces
    def _chainable(self) -> bool:
        """Blocks can pass the next norm's output along (see GQAGluBlock.forward_chain): plain blocks
        and norms without a shift, residual stream in fp32, parameters not sharded by ZeRO-3."""
        eng = getattr(self, "_grad_engine", None)
        if eng is not None and eng.level == 3 and eng.dp > 1:
            return False  # ZeRO-3 materializes a block's parameters only inside that block's own call
        norms = [self.norm] + [n for b in self.blocks if type(b) is GQAGluBlock
                               for n in (b.pre_attn_norm, b.post_attn_norm, b.pre_ffn_norm, b.post_ffn_norm)]
        return (
            len(self.blocks) > 0
            and all(type(b) is GQAGluBlock for b in self.blocks)
            and all(getattr(n, "shift", None) is None for n in norms)
            and self.tok_embeddings.weight.dtype == torch.float32
        )

    def _embed(self, input_ids: torch.Tensor) -> torch.Tensor:
        tp = self.tp
        w = self.tok_embeddings.weight
        if tpc.active(tp):
            h = embedding(input_ids, w, self.vocab_start, vocab_parallel=True)
            # rows outside this shard are zero: the TP group sums the partial lookups
            return tpc.reduce_scatter_seq(h, tp) if tp.sp else tpc.reduce_from_tp(h, tp)
        if type(self.tok_embeddings) is nn.Embedding:
            return embedding(input_ids, w)
        return self.tok_embeddings(input_ids)

    def _trunk(
        self,
        input_ids: torch.Tensor,
        kv_caches: list[KVCache] | None,
        start_pos: int,
        doc_ids: torch.Tensor | None,
        attn_mask: torch.Tensor | None,
    ) -> torch.Tensor:
        if self._before_forward is not None:
            self._before_forward()
        if tpc.active(self.tp):
            fused_tp.begin_forward(self.tp, input_ids.device)
        h = self._embed(input_ids)
        if kv_caches is None and self._chainable():
            # each block's closing residual-add kernel also applies the following norm
            blocks = list(self.blocks)
            xn = blocks[0].pre_attn_norm(h, out_dtype=compute_dtype(h))
            for i, block in enumerate(blocks):
                nxt = blocks[i + 1].pre_attn_norm if i + 1 < len(blocks) else self.norm
                kwargs = {"start_pos": start_pos, "base_attn_mask": attn_mask, "doc_ids": doc_ids, "xn": xn,
                          "next_norm": nxt, "chain": True}
                if self.gradient_checkpointing and self.training:
                    h, xn = checkpoint(block, h, use_reentrant=False, **kwargs)
                else:
                    h, xn = block(h, **kwargs)
            hn = xn
            tp = self.tp
            if tpc.active(tp):
                hn = tpc.gather_seq(hn, tp) if tp.sp else tpc.copy_to_tp(hn, tp)
            return hn
        for i, block in enumerate(self.blocks):
            kv_cache = kv_caches[i] if kv_caches is not None else None
            kwargs = {"kv_cache": kv_cache, "start_pos": start_pos, "base_attn_mask": attn_mask, "doc_ids": doc_ids}
            if self.gradient_checkpointing and self.training and kv_cache is None:
                h = checkpoint(block, h, use_reentrant=False, **kwargs)
            else:
                h = block(h, **kwargs)
        hn = self.norm(h, out_dtype=compute_dtype(h))
        tp = self.tp
        if tpc.active(tp):
            hn = tpc.gather_seq(hn, tp) if tp.sp else tpc.copy_to_tp(hn, tp)
        return hn

    def forward(
        self,
        input_ids: torch.Tensor,
        kv_caches: list[KVCache] | None = None,
        start_pos: int = 0,
        doc_ids: torch.Tensor | None = None,
        attn_mask: torch.Tensor | None = None,
        unpad_logits: bool = True,
    ) -> torch.Tensor:
        hn = self._trunk(input_ids, kv_caches, start_pos, doc_ids, attn_mask)
        if type(self.output) is nn.Linear:
            logits = linear(hn, self.output.weight, compute_dtype=compute_dtype(hn))
        else:
            logits = self.output(hn)
        tp = self.tp
        if tpc.active(tp):
            shards = [torch.empty_like(logits) for _ in range(tp.size)]
            dist.all_gather(shards, logits.contiguous(), group=tp.group)
            logits = torch.cat(shards, dim=-1)
        if unpad_logits and self.padded_vocab_size != self.config.vocab_size:
            logits = logits[..., : self.config.vocab_size]
        return logits

    def loss(
        self,
        input_ids: torch.Tensor,
        targets: torch.Tensor,
        loss_mask: torch.Tensor,
        doc_ids: torch.Tensor | None = None,
        attn_mask: torch.Tensor | None = None,
    ) -> torch.Tensor:
        """Masked next-token CE of the model on ``input_ids`` (fused LM head + CE)."""
        hn = self._trunk(input_ids, None, 0, doc_ids, attn_mask)
        tp = self.tp
        group = tp.group if tpc.active(tp) else None
        return lm_head_cross_entropy(
            hn, self.output.weight, targets, loss_mask, self.config.vocab_size,
            vocab_start=self.vocab_start, group=group, compute_dtype=compute_dtype(hn),
        )

    def token_logps(
        self,
        input_ids: torch.Tensor,
        targets: torch.Tensor,
        doc_ids: torch.Tensor | None = None,
        attn_mask: torch.Tensor | None = None,
    ) -> torch.Tensor:
        """fp32 ``log p(targets[b, t] | input_ids[b, :t+1])`` for every position, without
        materializing fp32 logits or a log-softmax (fused LM head + row statistics on CUDA).
        ``targets`` must hold valid token ids; positions to ignore are masked by the caller."""
        hn = self._trunk(input_ids, None, 0, doc_ids, attn_mask)
        tp = self.tp
        group = tp.group if tpc.active(tp) else None
        return lm_head_token_logps(
            hn, self.output.weight, targets, self.config.vocab_size,
            vocab_start=self.vocab_start, group=group, compute_dtype=compute_dtype(hn),
        )

    @torch.no_grad()
    def generate(
        self,
        input_ids: torch.Tensor,
        max_new_tokens: int,
        temperature: float = 1.0,
        top_k: int | None = None,
        top_p: float | None = None,
        eos_token_id: int | None = None,
        kv_caches: list[KVCache] | None = None,
        *,
        do_sample: bool | None = None,
        use_cache: bool = False,
        attention_mask: torch.Tensor | None = None,  # noqa: ARG002 - HF-style kwarg (ChatCORE), unpadded batches only
        pad_token_id: int | None = None,  # noqa: ARG002
        **_: Any,  # noqa: ANN401
    ) -> torch.Tensor:
        """Sample ``max_new_tokens`` tokens; ``temperature=0`` (or ``do_sample=False``) is greedy.

        Also accepts the HF-style keyword arguments the reference ChatCORE evaluator passes
        (mint/eval/dist/chatcore.py:91-99); ``use_cache=True`` allocates per-layer KV caches.
        """
        self.eval()
        if do_sample is False:
            temperature = 0.0
        if kv_caches is None and use_cache:
            dev = input_ids.device
            total = min(self.config.seq_length, input_ids.shape[1] + max_new_tokens)
            ref = self.blocks[0].gqa
            dt = self.tok_embeddings.weight.dtype if not torch.is_autocast_enabled(dev.type) else torch.get_autocast_dtype(dev.type)
            kv_caches = [
                KVCache(input_ids.shape[0], total, ref.n_kv_heads, ref.head_dim, dtype=dt, device=dev)
                for _ in self.blocks
            ]
        for step in range(max_new_tokens):
            if kv_caches is None:
                logits = self(input_ids[:, -self.config.seq_length :])
            elif step == 0:
                logits = self(input_ids, kv_caches=kv_caches)
            else:
                if input_ids.shape[1] > kv_caches[0].max_seq_len:
                    break
                logits = self(input_ids[:, -1:], kv_caches=kv_caches, start_pos=input_ids.shape[1] - 1)
            logits = logits[:, -1, :].float()
            if temperature == 0:
                next_token = logits.argmax(dim=-1, keepdim=True)
            else:
                logits = logits / temperature
                if top_k is not None:
                    v, _ = torch.topk(logits, min(top_k, logits.size(-1)))
                    logits[logits < v[:, [-1]]] = -float("inf")
                if top_p is not None:
                    sorted_logits, sorted_idx = torch.sort(logits, descending=True)
                    cum = torch.cumsum(torch.softmax(sorted_logits, dim=-1), dim=-1)
                    remove = cum > top_p
                    remove[..., 1:] = remove[..., :-1].clone()
                    remove[..., 0] = False
                    logits[remove.scatter(1, sorted_idx, remove)] = -float("inf")
                next_token = torch.multinomial(torch.softmax(logits, dim=-1), num_samples=1)
            input_ids = torch.cat([input_ids, next_token], dim=1)
            if eos_token_id is not None and (next_token == eos_token_id).all():
                break
        return input_ids

    def get_num_params(self, *, non_embedding: bool = True) -> int:
        n = sum(p.numel() for p in self.parameters())
        if non_embedding:
            n -= self.tok_embeddings.weight.numel()
        return n


def configure_optimizer(
    model: nn.Module,
    model_cfg: GemmaConfig,
    sched_cfg: Any,  # noqa: ANN401 - SchedulerConfig
    optim_cfg: Any,  # noqa: ANN401 - MuonAdamWConfig
    dp_group: dist.ProcessGroup | None = None,
):  # noqa: ANN201
    """Param groups lm_head / embedding / scalar / matrix (mint/models/gemma.py:177-248).

    ``optim_cfg.matrix_optimizer == "adamw"`` (default) reproduces the reference, which routes
    every group to AdamW. ``"muon"`` sends 2-D block matrices to NorMuon with Polar-Express
    orthogonalization of whole matrices.
    """
    from mint_b200.optim.dist_muon_adamw import DistMuonAdamW  # noqa: PLC0415

    groups: dict[str, list[nn.Parameter]] = {"lm_head": [], "embedding": [], "scalar": [], "matrix": []}
    for name, param in model.named_parameters():
        if not param.requires_grad:
            continue
        if "tok_embeddings" in name:
            groups["embedding"].append(param)
        elif "output" in name:
            groups["lm_head"].append(param)
        elif len(getattr(param, "_orig_shape", param.shape)) == 2:
            groups["matrix"].append(param)
        else:
            groups["scalar"].append(param)

    lr_scale = (model_cfg.embed_dim / 768) ** -0.5
    logger.info(f"Scaling AdamW LRs by {lr_scale:.6f}")
    hyper = {
        "lm_head": (sched_cfg.unembedding_lr * lr_scale, optim_cfg.adamw_beta2_lm_head, sched_cfg.weight_decay_lm_head),
        "embedding": (sched_cfg.embedding_lr * lr_scale, optim_cfg.adamw_beta2_embedding, sched_cfg.weight_decay_embedding),
        "scalar": (sched_cfg.scalar_lr * sched_cfg.scalar_lr_multiplier, optim_cfg.adamw_beta2_scalar, sched_cfg.weight_decay_scalar),
        "matrix": (sched_cfg.matrix_lr, optim_cfg.adamw_beta2_scalar, sched_cfg.weight_decay),
    }
    use_muon = getattr(optim_cfg, "matrix_optimizer", "adamw") == "muon"
    param_groups = []
    for kind, params in groups.items():
        if not params:
            continue
        lr, beta2, wd = hyper[kind]
        logger.info(f"{kind}: {len(params)} tensors, lr={lr:.6f}")
        if kind == "matrix" and use_muon:
            param_groups.append({
                "kind": "muon", "name": kind, "params": params, "lr": lr, "initial_lr": lr,
                "momentum": optim_cfg.muon_momentum, "beta2": optim_cfg.muon_beta2,
                "ns_steps": optim_cfg.muon_ns_steps, "weight_decay": wd,
            })
        else:
            param_groups.append({
                "kind": "adamw", "name": kind, "params": params, "lr": lr, "initial_lr": lr,
                "betas": (optim_cfg.adamw_beta1, beta2), "eps": optim_cfg.adamw_eps, "weight_decay": wd,
            })
    return DistMuonAdamW(param_groups, group=dp_group)
