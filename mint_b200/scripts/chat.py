"""``mint chat``: interactive chat with a HuggingFace causal LM (scripts/chat.py), or with a mint
checkpoint (``--checkpoint`` + ``--config``) through ``Gemma.generate`` with a KV cache."""

from __future__ import annotations

import argparse
import sys
from typing import Any


def _hf_loop(args: argparse.Namespace) -> None:
    from transformers import AutoModelForCausalLM, AutoTokenizer  # noqa: PLC0415

    tok = AutoTokenizer.from_pretrained(args.model_name, trust_remote_code=True)
    model: Any = AutoModelForCausalLM.from_pretrained(args.model_name, trust_remote_code=True, device_map="auto")
    model.eval()
    history: list[dict] = [{"role": "system", "content": args.system}]
    while True:
        try:
            text = input("You: ").strip()
        except (KeyboardInterrupt, EOFError):
            sys.exit(0)
        if not text:
            continue
        if text.lower() == "quit":
            sys.exit(0)
        if text.lower() == "reset":
            history = history[:1]
            continue
        history.append({"role": "user", "content": text})
        enc = tok.apply_chat_template(history, add_generation_prompt=True, return_tensors="pt", return_dict=True)
        ids = enc["input_ids"].to(model.device)
        out = model.generate(ids, attention_mask=enc["attention_mask"].to(model.device),
                             max_new_tokens=args.max_new_tokens, temperature=args.temperature, top_p=args.top_p,
                             do_sample=args.temperature > 0, pad_token_id=tok.eos_token_id)
        reply = tok.decode(out[0][ids.shape[-1]:], skip_special_tokens=True).strip()
        print(f"Assistant: {reply}\n")
        history = history[:1] if args.no_history else [*history, {"role": "assistant", "content": reply}]


def _mint_loop(args: argparse.Namespace) -> None:
    import torch  # noqa: PLC0415

    from mint_b200.models.gemma import Gemma, GemmaConfig  # noqa: PLC0415
    from mint_b200.scripts.pretrain import MetaConfig  # noqa: PLC0415
    from mint_b200.tokenizer import TikTokenizer  # noqa: PLC0415
    from mint_b200.utils.checkpointer import Checkpointer  # noqa: PLC0415

    cfg: GemmaConfig = MetaConfig.from_toml(args.config).model
    dev = torch.device("cuda" if torch.cuda.is_available() else "cpu")
    model = Gemma(cfg).to(dev)
    Checkpointer.load_model(model, args.checkpoint)
    tok = TikTokenizer()
    conv: list[dict] = []
    while True:
        try:
            text = input("You: ").strip()
        except (KeyboardInterrupt, EOFError):
            sys.exit(0)
        if text.lower() == "quit":
            sys.exit(0)
        conv.append({"role": "user", "content": text})
        ids, _ = tok.render_conversation({"messages": conv}, cfg.seq_length - args.max_new_tokens)
        ids.append(tok.encode_special("<|assistant_start|>"))
        inp = torch.tensor([ids], device=dev)
        with torch.autocast(dev.type, dtype=torch.bfloat16, enabled=dev.type == "cuda"):
            out = model.generate(inp, args.max_new_tokens, temperature=args.temperature, top_p=args.top_p,
                                 eos_token_id=tok.encode_special("<|assistant_end|>"), use_cache=True)
        reply = tok.decode(out[0, inp.shape[1]:].cpu())[0]
        print(f"Assistant: {reply}\n")
        conv = [] if args.no_history else [*conv, {"role": "assistant", "content": reply}]


def main() -> None:
    p = argparse.ArgumentParser(description="Chat with a causal LM")
    p.add_argument("--model-name", type=str, default="Qwen/Qwen2-0.5B-Instruct")
    p.add_argument("--max-new-tokens", type=int, default=512)
    p.add_argument("--temperature", type=float, default=0.7)
    p.add_argument("--top-p", type=float, default=0.9)
    p.add_argument("--system", type=str, default="You are a helpful assistant.")
    p.add_argument("--no-history", action="store_true")
    p.add_argument("--checkpoint", type=str, default=None, help="mint checkpoint (uses Gemma instead of HF)")
    p.add_argument("--config", type=str, default=None, help="TOML config matching --checkpoint")
    args = p.parse_args()
    if args.checkpoint:
        _mint_loop(args)
    else:
        _hf_loop(args)


if __name__ == "__main__":
    main()
