"""Tokenizers for the server: a byte-level tokenizer (no files needed; ids 3..258 = bytes) and a loader for a
local Hugging Face tokenizer directory (no network access is attempted)."""
from __future__ import annotations


class ByteTokenizer:
    """UTF-8 bytes shifted by 3 (0 = pad, 1 = bos/eos, 2 = unk). Decoding drops ids outside the byte range."""
    offset = 3
    eos_token_id = 1

    def encode(self, text: str) -> list:
        return [b + self.offset for b in text.encode("utf-8")]

    def decode(self, ids) -> str:
        return bytes(int(i) - self.offset for i in ids if self.offset <= int(i) < 256 + self.offset).decode(
            "utf-8", errors="replace")


class HFTokenizer:
    def __init__(self, path: str):
        from transformers import AutoTokenizer
        self.tok = AutoTokenizer.from_pretrained(path, local_files_only=True)
        self.eos_token_id = self.tok.eos_token_id

    def encode(self, text: str) -> list:
        return self.tok(text, add_special_tokens=False).input_ids

    def decode(self, ids) -> str:
        return self.tok.decode(list(ids))


def load_tokenizer(path: str | None):
    return HFTokenizer(path) if path else ByteTokenizer()
