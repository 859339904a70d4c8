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


class HFTokenizer:
    """A checkpoint's own tokenizer (tokenizer.json / tokenizer_config.json, local files
    only) behind the interface the engine uses: encode (no special tokens), decode
    (special tokens skipped), bos / eos / pad ids."""

    def __init__(self, path: str):
        from transformers import AutoTokenizer
        self.tok = AutoTokenizer.from_pretrained(path, local_files_only=True, trust_remote_code=False)
        self.bos_token_id = self.tok.bos_token_id if self.tok.bos_token_id is not None else 0
        self.eos_token_id = self.tok.eos_token_id if self.tok.eos_token_id is not None else -1
        self.pad_token_id = self.tok.pad_token_id if self.tok.pad_token_id is not None else 0
        self.vocab_size = len(self.tok)

    def encode(self, text: str) -> list:
        return list(self.tok.encode(text, add_special_tokens=False))

    def decode(self, ids) -> str:
        return self.tok.decode(list(ids), skip_special_tokens=True)

    def apply_chat_template(self, messages, add_generation_prompt=True) -> list:
        if getattr(self.tok, "chat_template", None):
            return list(self.tok.apply_chat_template(messages, add_generation_prompt=add_generation_prompt,
                                                     tokenize=True))
        text = "".join(f"<|{m['role']}|>{m['content']}" for m in messages)
        return [self.bos_token_id] + self.encode(text + ("<|assistant|>" if add_generation_prompt else ""))


def tokenizer_for(cfg_vocab: int, checkpoint: str = None):
    """The checkpoint's tokenizer when it ships one, else the byte tokenizer."""
    import os
    if checkpoint and any(os.path.exists(os.path.join(checkpoint, f))
                          for f in ("tokenizer.json", "tokenizer_config.json", "tokenizer.model")):
        return HFTokenizer(checkpoint)
    return ByteTokenizer(cfg_vocab)
