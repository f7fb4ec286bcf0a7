"""Tokenizers for the server: a local Hugging Face tokenizer, or a byte-level fallback.

No network is assumed: a tokenizer is only loaded from a local directory.
Without one, text is encoded as UTF-8 bytes shifted past three special ids
(0 pad, 1 bos, 2 eos) -- enough to drive random-init models end to end.
"""
from __future__ import annotations

import os
from typing import List, Optional


class ByteTokenizer:
    pad_token_id, bos_token_id, eos_token_id = 0, 1, 2
    offset = 3

    def encode(self, text: str) -> List[int]:
        return [b + self.offset for b in text.encode("utf-8")]

    def decode(self, ids) -> str:
        return bytes(i - self.offset for i in ids if self.offset <= i < self.offset + 256).decode("utf-8",
                                                                                            errors="replace")

    def apply_chat_template(self, messages) -> List[int]:
        text = "".join(f"<|{m.get('role', 'user')}|>\n{m.get('content', '')}\n" for m in messages) + "<|assistant|>\n"
        return [self.bos_token_id] + self.encode(text)


class HFTokenizer:
    def __init__(self, path: str):
        from transformers import AutoTokenizer

        self.tok = AutoTokenizer.from_pretrained(path, local_files_only=True)
        self.eos_token_id = self.tok.eos_token_id

    def encode(self, text: str) -> List[int]:
        return list(self.tok.encode(text))

    def decode(self, ids) -> str:
        return self.tok.decode(list(ids), skip_special_tokens=True)

    def apply_chat_template(self, messages) -> List[int]:
        if getattr(self.tok, "chat_template", None):
            return list(self.tok.apply_chat_template(messages, add_generation_prompt=True, tokenize=True))
        return ByteTokenizer.apply_chat_template(ByteTokenizer(), messages)


def load_tokenizer(path: Optional[str]):
    if path and os.path.isdir(path):
        return HFTokenizer(path)
    return ByteTokenizer()
