"""Tokenizers (mint/tokenizer/__init__.py:10-434).

``TikTokenizer`` reproduces the reference ids exactly: GPT-2 BPE (max id 50256), BOS = max+1,
PAD = max+2, eight chat specials max+3..max+10, vocab = max+11 = 50267, chat rendering with a
loss mask (assistant text and python calls 1; user turns, python outputs and BOS 0).

The GPT-2 BPE ranks are fetched by tiktoken on first use. Offline, point
``MINT_TIKTOKEN_FILE`` at a ``.tiktoken`` ranks file, or pass ``encoding=`` (e.g.
:func:`byte_level_encoding`, 256 byte tokens, used by the tests).
"""

from __future__ import annotations

import base64
import copy
import os
from abc import ABC, abstractmethod
from typing import Any

import torch

_GPT2_PAT = r"""'(?:[sdmt]|ll|ve|re)| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+"""

SPECIAL_NAMES = [
    "<|user_start|>", "<|user_end|>", "<|assistant_start|>", "<|assistant_end|>",
    "<|python_start|>", "<|python_end|>", "<|output_start|>", "<|output_end|>",
]


class Tokenizer(ABC):
    @property
    @abstractmethod
    def bos_token(self) -> int: ...

    @property
    @abstractmethod
    def eos_token(self) -> int: ...

    @property
    @abstractmethod
    def pad_token(self) -> int: ...

    @property
    @abstractmethod
    def vocab_size(self) -> int: ...

    @abstractmethod
    def encode(self, batch: list[str], *, add_bos: bool = True, add_eos: bool = False, padding: bool = True,
               max_length: int | None = None) -> torch.Tensor: ...

    @abstractmethod
    def encode_to_list(self, batch: list[str], *, add_bos: bool = True, add_eos: bool = False,
                       padding: bool = True, max_length: int | None = None) -> list[Any]: ...

    @abstractmethod
    def decode(self, batch: torch.Tensor, *, skip_special_tokens: bool = True) -> list[str]: ...

    @abstractmethod
    def encode_special(self, token: str) -> int: ...

    @abstractmethod
    def render_conversation(self, conversation: dict, max_tokens: int = 2048) -> tuple[list[int], list[int]]: ...


def byte_level_encoding(name: str = "bytes"):  # noqa: ANN201
    """A tiktoken Encoding with 256 single-byte tokens and the GPT-2 split pattern (no network)."""
    import tiktoken  # noqa: PLC0415

    ranks = {bytes([i]): i for i in range(256)}
    return tiktoken.Encoding(name=name, pat_str=_GPT2_PAT, mergeable_ranks=ranks, special_tokens={})


def _load_encoding(model_name: str):  # noqa: ANN202
    import tiktoken  # noqa: PLC0415

    path = os.environ.get("MINT_TIKTOKEN_FILE")
    if path:
        ranks = {}
        with open(path, "rb") as fh:
            for line in fh:
                if line.strip():
                    tok, rank = line.split()
                    ranks[base64.b64decode(tok)] = int(rank)
        eot = len(ranks)
        return tiktoken.Encoding(name=model_name, pat_str=_GPT2_PAT, mergeable_ranks=ranks,
                                 special_tokens={"<|endoftext|>": eot})
    return tiktoken.encoding_for_model(model_name=model_name)


class TikTokenizer(Tokenizer):
    def __init__(self, model_name: str = "gpt-2", encoding: Any = None) -> None:  # noqa: ANN401
        self.encoding = encoding if encoding is not None else _load_encoding(model_name)
        mx = self.encoding.max_token_value
        self._bos_token = mx + 1
        self._pad_token = mx + 2
        try:
            self._eos_token = self.encoding.eot_token
        except (AttributeError, KeyError):
            self._eos_token = mx
        self.special_tokens = {name: mx + 3 + i for i, name in enumerate(SPECIAL_NAMES)}

    @property
    def bos_token(self) -> int:
        return self._bos_token

    @property
    def eos_token(self) -> int:
        return self._eos_token

    @property
    def pad_token(self) -> int:
        return self._pad_token

    @property
    def vocab_size(self) -> int:
        return self.encoding.max_token_value + 11

    def encode(self, batch: list[str], *, add_bos: bool = True, add_eos: bool = False, padding: bool = True,
               max_length: int | None = None) -> torch.Tensor:
        return torch.tensor(self.encode_to_list(batch, add_bos=add_bos, add_eos=add_eos, padding=padding,
                                                max_length=max_length), dtype=torch.long)

    def encode_to_list(self, batch: list[str], *, add_bos: bool = True, add_eos: bool = False,
                       padding: bool = True, max_length: int | None = None) -> list[Any]:
        encoded = self.encoding.encode_batch(batch, disallowed_special=())
        out = []
        for toks in encoded:
            toks = list(toks)
            if max_length is not None:
                toks = toks[: max_length - int(add_bos) - int(add_eos)]
            if add_bos:
                toks = [self.bos_token, *toks]
            if add_eos:
                toks = [*toks, self.eos_token]
            out.append(toks)
        if padding and out:
            width = max(len(s) for s in out)
            return [s + [self.pad_token] * (width - len(s)) for s in out]
        return out

    def decode(self, batch: torch.Tensor, *, skip_special_tokens: bool = True) -> list[str]:
        if batch.dim() == 1:
            batch = batch.unsqueeze(0)
        rows = batch.tolist()
        if skip_special_tokens:
            special = {self.bos_token, self.eos_token, self.pad_token, *self.special_tokens.values()}
            rows = [[t for t in r if t not in special] for r in rows]
        mx = self.encoding.max_token_value
        rows = [[t for t in r if t <= mx] for r in rows]
        return self.encoding.decode_batch(rows)

    def encode_special(self, token: str) -> int:
        return self.special_tokens[token]

    def render_conversation(self, conversation: dict, max_tokens: int = 2048) -> tuple[list[int], list[int]]:
        ids: list[int] = []
        mask: list[int] = []

        def add(tok: int | list[int], m: int) -> None:
            toks = [tok] if isinstance(tok, int) else tok
            ids.extend(toks)
            mask.extend([m] * len(toks))

        messages = conversation["messages"]
        if messages[0]["role"] == "system":
            conversation = copy.deepcopy(conversation)
            messages = conversation["messages"]
            messages[1]["content"] = messages[0]["content"] + "\n\n" + messages[1]["content"]
            messages = messages[1:]
        sp = self.special_tokens
        add(self.bos_token, 0)
        for message in messages:
            content = message["content"]
            if message["role"] == "user":
                add(sp["<|user_start|>"], 0)
                add(self.encoding.encode(content, disallowed_special=()), 0)
                add(sp["<|user_end|>"], 0)
            elif message["role"] == "assistant":
                add(sp["<|assistant_start|>"], 0)
                if isinstance(content, str):
                    add(self.encoding.encode(content, disallowed_special=()), 1)
                elif isinstance(content, list):
                    for part in content:
                        toks = self.encoding.encode(part["text"], disallowed_special=())
                        if part["type"] == "text":
                            add(toks, 1)
                        elif part["type"] == "python":
                            add(sp["<|python_start|>"], 1)
                            add(toks, 1)
                            add(sp["<|python_end|>"], 1)
                        elif part["type"] == "python_output":
                            add(sp["<|output_start|>"], 0)
                            add(toks, 0)
                            add(sp["<|output_end|>"], 0)
                add(sp["<|assistant_end|>"], 1)
        return ids[:max_tokens], mask[:max_tokens]


class HFTokenizer(Tokenizer):
    """Thin wrapper over a HuggingFace tokenizer (deprecated in the reference, kept for API parity)."""

    def __init__(self, hf_tokenizer: Any) -> None:  # noqa: ANN401
        self.tok = hf_tokenizer
        if self.tok.pad_token_id is None:
            self.tok.pad_token = self.tok.eos_token

    @property
    def bos_token(self) -> int:
        return self.tok.bos_token_id if self.tok.bos_token_id is not None else self.tok.eos_token_id

    @property
    def eos_token(self) -> int:
        return self.tok.eos_token_id

    @property
    def pad_token(self) -> int:
        return self.tok.pad_token_id

    @property
    def vocab_size(self) -> int:
        return len(self.tok)

    def encode(self, batch: list[str], *, add_bos: bool = True, add_eos: bool = False, padding: bool = True,
               max_length: int | None = None) -> torch.Tensor:
        return torch.tensor(self.encode_to_list(batch, add_bos=add_bos, add_eos=add_eos, padding=padding,
                                                max_length=max_length), dtype=torch.long)

    def encode_to_list(self, batch: list[str], *, add_bos: bool = True, add_eos: bool = False,
                       padding: bool = True, max_length: int | None = None) -> list[Any]:
        out = []
        for text in batch:
            toks = self.tok.encode(text, add_special_tokens=False)
            if max_length is not None:
                toks = toks[: max_length - int(add_bos) - int(add_eos)]
            if add_bos:
                toks = [self.bos_token, *toks]
            if add_eos:
                toks = [*toks, self.eos_token]
            out.append(toks)
        if padding and out:
            width = max(len(s) for s in out)
            return [s + [self.pad_token] * (width - len(s)) for s in out]
        return out

    def decode(self, batch: torch.Tensor, *, skip_special_tokens: bool = True) -> list[str]:
        if batch.dim() == 1:
            batch = batch.unsqueeze(0)
        return self.tok.batch_decode(batch.tolist(), skip_special_tokens=skip_special_tokens)

    def encode_special(self, token: str) -> int:
        return self.tok.convert_tokens_to_ids(token)

    def render_conversation(self, conversation: dict, max_tokens: int = 2048) -> tuple[list[int], list[int]]:
        ids: list[int] = [self.bos_token]
        mask: list[int] = [0]
        for m in conversation["messages"]:
            content = m["content"] if isinstance(m["content"], str) else "".join(p["text"] for p in m["content"])
            toks = self.tok.encode(content, add_special_tokens=False)
            ids.extend(toks)
            mask.extend([1 if m["role"] == "assistant" else 0] * len(toks))
        return ids[:max_tokens], mask[:max_tokens]
