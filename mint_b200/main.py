"""``mint`` command-line dispatcher (mint/main.py:19-53): same nine sub-commands and flags.

    python -m mint_b200 pretrain --config configs/d12_b200.toml
    torchrun --nproc-per-node 8 -m mint_b200 pretrain --config configs/d12_b200_tp2_zero2.toml
"""

from __future__ import annotations

import importlib
import sys

_COMMANDS: dict[str, tuple[str, str]] = {
    "sft": ("mint_b200.scripts.sfttrain", "SFT training for Gemma model (TikToken tokenizer)"),
    "dpo": ("mint_b200.scripts.dpo", "DPO training for Gemma model (TikToken tokenizer)"),
    "pretrain": ("mint_b200.scripts.pretrain", "Pre-training for Gemma model with distributed dataloader"),
    "chat": ("mint_b200.scripts.chat", "Chat with any HuggingFace causal LM or a mint checkpoint"),
    "download-climbmix": ("mint_b200.scripts.utils.async_download_climbmix", "Async download of ClimbMix"),
    "download-eval": ("mint_b200.scripts.utils.download_eval_bundle", "Download evaluation benchmarks bundle"),
    "prepare-dpo": ("mint_b200.scripts.utils.prepare_dpo_dataset", "Prepare anthropic/hh-rlhf DPO dataset"),
    "stream-train": ("mint_b200.scripts.utils.train_with_streaming_download", "Train while downloading"),
    "gen-config": ("mint_b200.scripts.utils.gen_config_from_scaling_law", "Generate model config from scaling laws"),
}


def _print_help() -> None:
    print("usage: mint <command> [args ...]\n")
    print("Available commands:")
    width = max(map(len, _COMMANDS))
    for cmd, (_, desc) in _COMMANDS.items():
        print(f"  {cmd:<{width}}  {desc}")
    print("\nRun `mint <command> --help` for command-specific options.")


def app() -> None:
    if len(sys.argv) < 2 or sys.argv[1] in {"-h", "--help"}:
        _print_help()
        sys.exit(0)
    cmd = sys.argv[1]
    if cmd not in _COMMANDS:
        print(f"mint: unknown command '{cmd}'\n", file=sys.stderr)
        _print_help()
        sys.exit(1)
    sys.argv = [f"mint {cmd}", *sys.argv[2:]]
    importlib.import_module(_COMMANDS[cmd][0]).main()


if __name__ == "__main__":
    app()
