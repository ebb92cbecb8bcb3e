"""``mint gen-config``: derive a model / schedule config from scaling laws
(scripts/utils/gen_config_from_scaling_law.py). Chinchilla tokens = ratio x params, batch
``B = B_ref (D/D_ref)^0.383`` rounded to a power of two, ``lr = lr_ref sqrt(B/B_ref)``,
``wd = wd_ref sqrt(B/B_ref) D_ref/D``, warmup ``max(100, 2%)``, warmdown ratio 0.65.

The reference writes a flat YAML file that its own TOML loader cannot read; this writes a TOML
file in the ``[model] / [train] / [train.sched] / [optim] / [device] / [dl]`` schema.
"""

from __future__ import annotations

import argparse
import math


def _model_dim(depth: int, aspect: int, head_dim: int) -> int:
    return (depth * aspect + head_dim - 1) // head_dim * head_dim


def scaling_params(depth: int, aspect: int, head_dim: int) -> int:
    d = _model_dim(depth, aspect, head_dim)
    return 4 * depth * d * d


def calculate_hyperparams(depth_ref: int, depth_target: int, aspect_ratio: int, head_dim: int, seq_length: int,
                          param_data_ratio: float, B_ref: int, lr_ref: float, wd_ref: float,  # noqa: N803
                          vocab_size: int = 50258) -> dict:
    embed = _model_dim(depth_target, aspect_ratio, head_dim)
    n_ref, n_tgt = scaling_params(depth_ref, aspect_ratio, head_dim), scaling_params(depth_target, aspect_ratio, head_dim)
    d_ref, d_tgt = param_data_ratio * n_ref, param_data_ratio * n_tgt
    b = 2 ** round(math.log2(B_ref * (d_tgt / d_ref) ** 0.383))
    rb = b / B_ref
    iters = int(d_tgt / b)
    return {
        "embed_dim": embed, "hidden_dim": 4 * embed, "seq_length": seq_length, "vocab_size": vocab_size,
        "n_layers": depth_target, "n_heads": embed // head_dim, "n_kv_heads": embed // head_dim, "head_dim": head_dim,
        "batch_size": b, "train_num_steps": iters, "matrix_lr": lr_ref * math.sqrt(rb),
        "weight_decay": wd_ref * math.sqrt(rb) * (d_ref / d_tgt), "warmup_steps": max(100, int(0.02 * iters)),
        "warmdown_ratio": 0.65, "scaling_params": n_tgt, "training_tokens": d_tgt,
    }


def calculate_optimal_depth_from_flops(target_flops: float, aspect_ratio: int, head_dim: int, seq_length: int,  # noqa: ARG001
                                       param_data_ratio: float, vocab_size: int = 50258) -> int:  # noqa: ARG001
    optimal = math.sqrt(target_flops / (6 * param_data_ratio))
    return min(range(1, 101), key=lambda d: abs(scaling_params(d, aspect_ratio, head_dim) - optimal))


def to_toml(p: dict) -> str:
    seqs = max(1, p["batch_size"] // p["seq_length"])
    return f"""[model]
embed_dim = {p['embed_dim']}
hidden_dim = {p['hidden_dim']}
seq_length = {p['seq_length']}
vocab_size = {p['vocab_size']}
n_layers = {p['n_layers']}
n_heads = {p['n_heads']}
n_kv_heads = {p['n_kv_heads']}
head_dim = {p['head_dim']}
rope_base_theta = 100000
tie_weights = true

[train]
mixed_precision = true
use_meta_device = true
compile_model = false
train_num_steps = {p['train_num_steps']}
grad_clip = 1.0
log_every_n_steps = 1
eval_every_n_steps = 100
eval_num_steps = 10
core_eval_every_n_step = 500
gradient_accumulation_steps = 1

[train.ckpt]
checkpoint_dir = "checkpoints"
save_checkpoint_every_n_steps = 200
keep_last_n_checkpoints = 1
load_best_checkpoint = false

[train.lg]
wandb_enabled = true
wandb_project = "goda"

[train.sched]
unembedding_lr = 0.004
embedding_lr = 0.2
matrix_lr = {p['matrix_lr']:.8g}
scalar_lr = 0.5
weight_decay = {p['weight_decay']:.8g}
weight_decay_lm_head = 0.01
weight_decay_embedding = 0.001
weight_decay_scalar = 0.05
scalar_lr_multiplier = 0.01
warmup_steps = {p['warmup_steps']}
warmdown_ratio = {p['warmdown_ratio']}
final_lr_frac = 0.1
muon_momentum_warmup_steps = 400
muon_momentum_start = 0.85
muon_momentum_peak = 0.97
muon_momentum_final = 0.9

[optim]
muon_momentum = 0.95
muon_beta2 = 0.9
muon_ns_steps = 5
adamw_beta1 = 0.8
adamw_beta2_lm_head = 0.96
adamw_beta2_embedding = 0.995
adamw_beta2_scalar = 0.95
adamw_eps = 1.0e-10

[device]
mixed_precision = true
tp_size = 1
ddp_level = 0
sp = false

[dl]
data_dir = "data/climbmix"
batch_size = {seqs}
buffer_size = 1000
tokenizer_batch_size = 128
seq_length = {p['seq_length']}
"""


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--depth-ref", type=int, default=12)
    ap.add_argument("--depth-target", type=int, default=None)
    ap.add_argument("--flops", type=float, default=None, help="Total compute budget in FLOPs")
    ap.add_argument("--mfu", type=float, default=None, help="Model FLOPs Utilization (0-1)")
    ap.add_argument("--aspect-ratio", type=int, default=64)
    ap.add_argument("--head-dim", type=int, default=128)
    ap.add_argument("--seq-length", type=int, default=512)
    ap.add_argument("--param-data-ratio", type=float, default=20)
    ap.add_argument("--B-ref", type=int, default=524288)
    ap.add_argument("--lr-ref", type=float, default=0.02)
    ap.add_argument("--wd-ref", type=float, default=0.0)
    ap.add_argument("--vocab-size", type=int, default=50258)
    ap.add_argument("--output", type=str, default=None)
    a = ap.parse_args()
    if a.flops is not None:
        eff = a.flops * (a.mfu if a.mfu is not None else 1.0)
        depth = calculate_optimal_depth_from_flops(eff, a.aspect_ratio, a.head_dim, a.seq_length, a.param_data_ratio,
                                                   a.vocab_size)
    elif a.depth_target is not None:
        depth = a.depth_target
    else:
        ap.error("Either --depth-target or --flops must be specified")
    res = calculate_hyperparams(a.depth_ref, depth, a.aspect_ratio, a.head_dim, a.seq_length, a.param_data_ratio,
                                a.B_ref, a.lr_ref, a.wd_ref, a.vocab_size)
    for k in ("n_layers", "embed_dim", "hidden_dim", "n_heads", "scaling_params", "training_tokens", "batch_size",
              "matrix_lr", "weight_decay", "train_num_steps", "warmup_steps"):
        print(f"{k}: {res[k]}")
    out = a.output or f"config_d{depth}.toml"
    with open(out, "w") as fh:
        fh.write(to_toml(res))
    print(f"Config saved to: {out}")


if __name__ == "__main__":
    main()
