"""Tokenizers for the rollout/workflow layer.

``load_tokenizer(path)`` returns a Hugging Face tokenizer when ``path`` holds
tokenizer files, otherwise ``ByteTokenizer``: UTF-8 bytes mapped to ids
``[offset, offset+256)`` with a few special ids below ``offset``.  Synthetic
benchmark workloads use raw token ids and need no tokenizer at all.
"""

from __future__ import annotations

import os
from typing import List, Optional


class ByteTokenizer:
    pad_token_id = 0
    eos_token_id = 1
    bos_token_id = 2
    offset = 4

    def __init__(self, vocab_size: int = 1024):
        if vocab_size < self.offset + 256:
            raise ValueError("ByteTokenizer needs vocab_size >= 260")
        self.vocab_size = vocab_size
        self.pad_token = "<pad>"
        self.eos_token = "<eos>"

    def encode(self, text: str, add_special_tokens: bool = False) -> List[int]:
        return [b + self.offset for b in text.encode("utf-8")]

    def decode(self, ids: List[int], skip_special_tokens: bool = True) -> str:
        data = bytes(int(i) - self.offset for i in ids if self.offset <= int(i) < self.offset + 256)
        return data.decode("utf-8", errors="replace")

    def __call__(self, text: str, **_):
        return {"input_ids": self.encode(text)}

    def apply_chat_template(self, messages, tokenize: bool = False, add_generation_prompt: bool = True, **_):
        text = "".join(f"<|{m['role']}|>\n{m['content']}\n" for m in messages)
        if add_generation_prompt:
            text += "<|assistant|>\n"
        return self.encode(text) if tokenize else text


def load_tokenizer(path: Optional[str], vocab_size: int = 151936):
    if path and os.path.isdir(path) and any(os.path.exists(os.path.join(path, f))
                                            for f in ("tokenizer.json", "tokenizer_config.json")):
        from transformers import AutoTokenizer

        tok = AutoTokenizer.from_pretrained(path, trust_remote_code=True)
        if tok.pad_token is None:
            tok.pad_token = tok.eos_token
        return tok
    return ByteTokenizer(vocab_size)
