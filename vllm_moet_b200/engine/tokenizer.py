"""Byte-level tokenizer for synthetic (random-init) models: token = byte + 3
(0 = pad, 1 = bos, 2 = eos); ids above 258 decode to nothing."""
from __future__ import annotations


class ByteTokenizer:
    pad_token_id, bos_token_id, eos_token_id = 0, 1, 2

    def __init__(self, vocab_size: int):
        if vocab_size < 259:
            raise ValueError("byte tokenizer needs vocab >= 259")
        self.vocab_size = vocab_size

    def encode(self, text: str) -> list:
        return [b + 3 for b in text.encode("utf-8")]

    def decode(self, ids) -> str:
        return bytes(i - 3 for i in ids if 3 <= i < 259).decode("utf-8", errors="replace")

    def apply_chat_template(self, messages, add_generation_prompt=True) -> list:
        text = "".join(f"<|{m['role']}|>{m['content']}" for m in messages)
        if add_generation_prompt:
            text += "<|assistant|>"
        return [self.bos_token_id] + self.encode(text)
