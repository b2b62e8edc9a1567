"""Tokenizers: HF tokenizers from local checkpoint directories, a byte-level fallback.

There is no network access in the serving path: `load_tokenizer` reads a local
directory (tokenizer.json / tokenizer_config.json) through transformers, and
otherwise returns `ByteTokenizer`, which maps UTF-8 bytes to ids 3..258 so that
random-init benchmark models and tests can still accept text.

Reference parity: core/tokenizer.py:19 (cached get_tokenizer), the Rust
batch_tokenize_fast of rust_core/src/lib.rs:1501-1558.
"""
from __future__ import annotations

import functools
import os
from typing import List, Optional, Sequence


class ByteTokenizer:
    """UTF-8 byte-level tokenizer: 0 = pad, 1 = bos, 2 = eos, bytes at 3..258."""

    pad_token_id = 0
    bos_token_id = 1
    eos_token_id = 2
    OFFSET = 3

    def __init__(self, vocab_size: int = 259):
        self.vocab_size = max(259, vocab_size)

    def encode(self, text: str, add_special_tokens: bool = False) -> List[int]:
        ids = [b + self.OFFSET for b in text.encode("utf-8")]
        return ([self.bos_token_id] + ids) if add_special_tokens else ids

    def decode(self, ids: Sequence[int], skip_special_tokens: bool = True) -> str:
        out = bytearray()
        for i in ids:
            i = int(i)
            if self.OFFSET <= i < self.OFFSET + 256:
                out.append(i - self.OFFSET)
            elif not skip_special_tokens and i < self.OFFSET:
                out.extend(f"<{i}>".encode())
            elif i >= self.OFFSET + 256:
                # ids outside the byte range (random models sample the whole vocabulary)
                out.extend(chr(0x4E00 + (i % 20000)).encode("utf-8"))
        return out.decode("utf-8", errors="replace")

    def batch_encode(self, texts: Sequence[str]) -> List[List[int]]:
        return [self.encode(t) for t in texts]

    def __call__(self, text, **kw):
        if isinstance(text, str):
            return {"input_ids": self.encode(text)}
        return {"input_ids": self.batch_encode(text)}


class HFTokenizer:
    """transformers tokenizer loaded from a local directory (local_files_only)."""

    def __init__(self, path: str):
        from transformers import AutoTokenizer
        self.tok = AutoTokenizer.from_pretrained(path, local_files_only=True)
        self.eos_token_id = self.tok.eos_token_id
        self.pad_token_id = self.tok.pad_token_id if self.tok.pad_token_id is not None else self.eos_token_id
        self.bos_token_id = self.tok.bos_token_id
        self.vocab_size = len(self.tok)

    def encode(self, text: str, add_special_tokens: bool = False) -> List[int]:
        return self.tok.encode(text, add_special_tokens=add_special_tokens)

    def decode(self, ids: Sequence[int], skip_special_tokens: bool = True) -> str:
        return self.tok.decode(list(ids), skip_special_tokens=skip_special_tokens)

    def batch_encode(self, texts: Sequence[str]) -> List[List[int]]:
        return [list(x) for x in self.tok(list(texts), add_special_tokens=False)["input_ids"]]

    def apply_chat_template(self, messages, **kw):
        return self.tok.apply_chat_template(messages, tokenize=False, add_generation_prompt=True, **kw)


@functools.lru_cache(maxsize=8)
def load_tokenizer(name_or_path: Optional[str], vocab_size: int = 259):
    if name_or_path and os.path.isdir(name_or_path) and any(
            os.path.exists(os.path.join(name_or_path, f)) for f in ("tokenizer.json", "tokenizer_config.json",
                                                                     "vocab.json", "tokenizer.model")):
        try:
            return HFTokenizer(name_or_path)
        except Exception:
            pass
    return ByteTokenizer(vocab_size)
