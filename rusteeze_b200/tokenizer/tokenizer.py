"""Tokenizer wrapper and incremental detokenizer.

The reference wraps the Rust `tokenizers` crate (crates/rusteeze-tokenizer/
src/tokenizer.rs:25-205: load from file or directory, encode/encode_batch,
decode, special tokens) and streams text with a decoder that re-decodes the
whole prefix on every token (tokenizer.rs:425-486, quadratic in length).
Here:
  * `HFTokenizer` loads `tokenizer.json` through the Python `tokenizers`
    package (same library) plus special tokens from `tokenizer_config.json`.
  * `ByteTokenizer` is a deterministic byte-level tokenizer for random-init
    benchmark models that ship no vocabulary: ids 0..2 are <pad>/<s>/</s>
    and ids 3..258 are bytes; ids above 258 decode to nothing.
  * `IncrementalDetokenizer` decodes only a sliding window of tokens
    (prefix-offset / read-offset method), so streaming costs O(1) per token,
    and holds back text that ends in an incomplete UTF-8 sequence.
"""
from __future__ import annotations

import json
import os
from typing import List, Optional, Sequence

from rusteeze_b200.core.errors import ModelLoadError


class BaseTokenizer:
    bos_token_id: Optional[int] = None
    eos_token_id: Optional[int] = None
    pad_token_id: Optional[int] = None
    bos_token: str = ""
    eos_token: str = ""
    chat_template: Optional[str] = None
    name: str = "tokenizer"

    def encode(self, text: str, add_special_tokens: bool = True) -> List[int]:
        raise NotImplementedError

    def decode(self, ids: Sequence[int], skip_special_tokens: bool = True) -> str:
        raise NotImplementedError

    def encode_batch(self, texts: Sequence[str], add_special_tokens: bool = True) -> List[List[int]]:
        return [self.encode(t, add_special_tokens) for t in texts]

    @property
    def vocab_size(self) -> int:
        raise NotImplementedError

    def all_special_ids(self) -> List[int]:
        return [i for i in (self.bos_token_id, self.eos_token_id, self.pad_token_id) if i is not None]


class ByteTokenizer(BaseTokenizer):
    OFFSET = 3

    def __init__(self, vocab_size: int = 32000, name: str = "byte"):
        self._vocab = max(vocab_size, 259)
        self.pad_token_id, self.bos_token_id, self.eos_token_id = 0, 1, 2
        self.bos_token, self.eos_token = "<s>", "</s>"
        self.name = name

    @property
    def vocab_size(self) -> int:
        return self._vocab

    def encode(self, text: str, add_special_tokens: bool = True) -> List[int]:
        ids = [b + self.OFFSET for b in text.encode("utf-8")]
        return ([self.bos_token_id] + ids) if add_special_tokens else ids

    def decode(self, ids: Sequence[int], skip_special_tokens: bool = True) -> str:
        out = bytearray()
        for i in ids:
            if self.OFFSET <= i < self.OFFSET + 256:
                out.append(i - self.OFFSET)
            elif not skip_special_tokens and i in (1, 2):
                out.extend((self.bos_token if i == 1 else self.eos_token).encode())
        return out.decode("utf-8", errors="replace")


class HFTokenizer(BaseTokenizer):
    def __init__(self, path: str):
        from tokenizers import Tokenizer
        tj = os.path.join(path, "tokenizer.json") if os.path.isdir(path) else path
        if not os.path.exists(tj):
            raise ModelLoadError(f"tokenizer.json not found at {tj}")
        self.tk = Tokenizer.from_file(tj)
        self.name = os.path.basename(os.path.dirname(os.path.abspath(tj)))
        cfg = {}
        d = os.path.dirname(os.path.abspath(tj))
        tc = os.path.join(d, "tokenizer_config.json")
        if os.path.exists(tc):
            with open(tc) as f:
                cfg = json.load(f)

        def tok_str(v):
            if isinstance(v, dict):
                return v.get("content", "")
            return v or ""

        self.bos_token = tok_str(cfg.get("bos_token"))
        self.eos_token = tok_str(cfg.get("eos_token"))
        self.chat_template = cfg.get("chat_template")
        self.add_bos = cfg.get("add_bos_token", True)
        self.bos_token_id = self.tk.token_to_id(self.bos_token) if self.bos_token else None
        self.eos_token_id = self.tk.token_to_id(self.eos_token) if self.eos_token else None
        pad = tok_str(cfg.get("pad_token"))
        self.pad_token_id = self.tk.token_to_id(pad) if pad else None

    @property
    def vocab_size(self) -> int:
        return self.tk.get_vocab_size(with_added_tokens=True)

    def encode(self, text: str, add_special_tokens: bool = True) -> List[int]:
        return self.tk.encode(text, add_special_tokens=add_special_tokens).ids

    def encode_batch(self, texts, add_special_tokens: bool = True):
        return [e.ids for e in self.tk.encode_batch(list(texts), add_special_tokens=add_special_tokens)]

    def decode(self, ids: Sequence[int], skip_special_tokens: bool = True) -> str:
        return self.tk.decode(list(ids), skip_special_tokens=skip_special_tokens)


def load_tokenizer(path: Optional[str], vocab_size: int = 32000) -> BaseTokenizer:
    if path and (os.path.exists(os.path.join(path, "tokenizer.json")) or path.endswith(".json")):
        return HFTokenizer(path)
    return ByteTokenizer(vocab_size)


class IncrementalDetokenizer:
    """Streaming detokenizer with prefix/read offsets.

    After each new token, decodes tokens[prefix_offset:] and
    tokens[prefix_offset:read_offset] and emits the difference; offsets then
    slide forward, so each step touches only a few tokens.  Text ending in
    U+FFFD (an incomplete multi-byte character) is held back."""

    def __init__(self, tokenizer: BaseTokenizer, prompt_ids: Sequence[int], skip_special_tokens: bool = True):
        self.tok = tokenizer
        self.skip = skip_special_tokens
        self.ids: List[int] = list(prompt_ids[-6:])
        self.prefix_offset = 0
        self.read_offset = len(self.ids)
        self.text = ""

    def clone(self) -> "IncrementalDetokenizer":
        c = IncrementalDetokenizer.__new__(IncrementalDetokenizer)
        c.tok, c.skip, c.ids = self.tok, self.skip, list(self.ids)
        c.prefix_offset, c.read_offset, c.text = self.prefix_offset, self.read_offset, self.text
        return c

    def step(self, new_id: int) -> str:
        self.ids.append(int(new_id))
        prefix = self.tok.decode(self.ids[self.prefix_offset:self.read_offset], self.skip)
        full = self.tok.decode(self.ids[self.prefix_offset:], self.skip)
        # advance when new text appeared, or when a run of tokens that decode to
        # nothing (special / unmapped ids) would otherwise grow the window forever
        stalled = len(self.ids) - self.prefix_offset > 8 and full == prefix
        if (len(full) > len(prefix) or stalled) and not full.endswith("�"):
            delta = full[len(prefix):]
            self.prefix_offset = self.read_offset
            self.read_offset = len(self.ids)
            self.text += delta
            # keep the id list short
            if self.prefix_offset > 64:
                cut = self.prefix_offset
                self.ids = self.ids[cut:]
                self.read_offset -= cut
                self.prefix_offset = 0
            return delta
        return ""

    def extend(self, new_ids) -> str:
        """Feeds many tokens at once and returns the text they add: the concatenation
        of what `step` would have returned for them one by one, with one decode of the
        window instead of two per token.  Used for outputs whose text nobody reads
        until the request finishes.  Where the window ends in an incomplete character
        the tokens go through `step` so the held-back tail is handled exactly."""
        new_ids = [int(t) for t in new_ids]
        if not new_ids:
            return ""
        n0 = len(self.ids)
        self.ids.extend(new_ids)
        prefix = self.tok.decode(self.ids[self.prefix_offset:self.read_offset], self.skip)
        full = self.tok.decode(self.ids[self.prefix_offset:], self.skip)
        if full.endswith("�") or "�" in full[len(prefix):] or not full.startswith(prefix):
            del self.ids[n0:]
            return "".join(self.step(t) for t in new_ids)
        delta = full[len(prefix):]
        self.prefix_offset = max(self.read_offset, len(self.ids) - 6)
        self.read_offset = len(self.ids)
        self.text += delta
        if self.prefix_offset > 64:
            cut = self.prefix_offset
            self.ids = self.ids[cut:]
            self.read_offset -= cut
            self.prefix_offset = 0
        return delta
