"""Tokenizer front-end: the model's HF `tokenizer.json` when present, else a byte-level tokenizer.

Parity: the coordinator loads `tokenizer.json` from the model directory (rust/src/distributed/
coordinator.rs:~890, rust/src/infer.rs:62-66). Random-init benchmark models have no tokenizer, so a
deterministic byte-level fallback (UTF-8 bytes offset into the vocabulary) keeps the HTTP API usable
with them.
"""

from __future__ import annotations

import logging
import os
from typing import List, Optional


class ByteTokenizer:
    OFFSET = 3

    def __init__(self, vocab_size: int):
        self.vocab_size = vocab_size

    def encode(self, text: str) -> List[int]:
        ids = [b + self.OFFSET for b in text.encode("utf-8")]
        return [i % self.vocab_size for i in ids] or [self.OFFSET % self.vocab_size]

    def decode(self, ids: List[int]) -> str:
        bs = bytes(((i - self.OFFSET) % 256) for i in ids if i >= self.OFFSET)
        return bs.decode("utf-8", errors="replace")


class HfTokenizer:
    def __init__(self, path: str):
        from tokenizers import Tokenizer
        self.tok = Tokenizer.from_file(path)

    def encode(self, text: str) -> List[int]:
        return self.tok.encode(text).ids

    def decode(self, ids: List[int]) -> str:
        return self.tok.decode(ids)


def load_tokenizer(model_dir: Optional[str], vocab_size: int):
    if model_dir:
        p = os.path.join(model_dir, "tokenizer.json")
        if os.path.exists(p):
            try:
                return HfTokenizer(p)
            except Exception as e:  # any parse / import failure: say so, then fall back
                logging.getLogger("hcp.tokenizer").warning(
                    "could not load %s (%s: %s); using the byte tokenizer", p,
                    type(e).__name__, e)
    return ByteTokenizer(vocab_size)
