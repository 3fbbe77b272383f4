"""Tokenizer loading for the server.

``load_tokenizer(path)`` reads a Hugging Face ``tokenizer.json`` (or this
framework's compiled tokenizer format) into the C++ ``Tokenizer``. With no
path, ``byte_level_tokenizer(vocab_size)`` builds a synthetic byte-level BPE
tokenizer: the 256 byte tokens (GPT-2 byte-to-unicode alphabet), the chat
template tags of the "glm" and "deepseek" styles as special tokens, and no
merges; it encodes any UTF-8 text, one token per byte, inside ``vocab_size``.
"""
from __future__ import annotations

import json
from pathlib import Path

from ..core import core

GLM_SPECIALS = ("[gMASK]", "<sop>", "<|system|>", "<|user|>", "<|assistant|>", "<|observation|>", "<think>",
                "</think>", "<tool_response>", "</tool_response>", "<|endoftext|>")
DEEPSEEK_SPECIALS = ("<｜begin▁of▁sentence｜>", "<｜end▁of▁sentence｜>",
                     "<｜User｜>", "<｜Assistant｜>", "<｜tool▁output｜>")


def _byte_alphabet() -> list[str]:
    """GPT-2 byte-to-unicode map: printable bytes map to themselves, the rest to 256+n."""
    keep = list(range(ord("!"), ord("~") + 1)) + list(range(0xA1, 0xAD)) + list(range(0xAE, 0x100))
    out, n = {}, 0
    for b in range(256):
        if b in keep:
            out[b] = chr(b)
        else:
            out[b] = chr(256 + n)
            n += 1
    return [out[b] for b in range(256)]


def byte_level_tokenizer_json(vocab_size: int = 1024, specials=GLM_SPECIALS + DEEPSEEK_SPECIALS) -> str:
    if vocab_size < 256 + len(specials):
        raise ValueError(f"vocab_size {vocab_size} cannot hold 256 bytes + {len(specials)} specials")
    vocab = {ch: i for i, ch in enumerate(_byte_alphabet())}
    added = []
    for i, s in enumerate(specials):
        vocab[s] = 256 + i
        added.append({"id": 256 + i, "content": s, "special": True})
    return json.dumps({
        "model": {"type": "BPE", "vocab": vocab, "merges": []},
        "pre_tokenizer": {"type": "ByteLevel", "add_prefix_space": False},
        "added_tokens": added,
    })


def byte_level_tokenizer(vocab_size: int = 1024):
    return core().Tokenizer.from_hf_json(byte_level_tokenizer_json(vocab_size))


def load_tokenizer(path: str | None, vocab_size: int = 1024):
    if not path:
        return byte_level_tokenizer(vocab_size)
    data = Path(path).read_bytes()
    if data[:1] == b"{":
        return core().Tokenizer.from_hf_json(data.decode("utf-8"))
    return core().Tokenizer.from_compiled(data)
