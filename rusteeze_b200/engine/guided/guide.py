"""Guided (structured) decoding: which tokens may come next.

`GuidedDecodingParams` (choice, regex, JSON schema, JSON object) compiles to one regex
and its lazily built DFA (`regex_fsm.RegexFSM`, cached per pattern).  A `TokenIndex`
holds, per tokenizer, the text of every token and a character trie over those texts
(built on the first guided request: about 1 s and 115 MB of host memory for a
128K-token vocabulary).
The tokens allowed in a DFA state are found by walking the trie and the DFA together,
cutting a branch as soon as the DFA dies, so shared token prefixes are stepped once (or,
in states where most characters loop back, by a vectorised check of whole tokens); the
resulting boolean mask is cached per (pattern, state): about 1-15 ms the first time for a
128K-token vocabulary, microseconds after.  A `Guide` is one sequence's
position in its DFA: the sampler masks the row's logits with `guide.mask()`, and the
engine advances the guide with every token the sequence takes.

End of output: where the DFA accepts, the EOS ids are allowed too; where it accepts and
cannot continue, only EOS is.  A request with `ignore_eos` ends ("stop") when its guide
can no longer continue.  Where no token of the vocabulary can continue a partial match
(the pattern needs a character no whole-character token spells), EOS is allowed and the
request ends ("stop") rather than leave the constraint.

Tokens whose text is empty (special tokens) or not whole characters (a byte-level
tokenizer's partial UTF-8 bytes) are never allowed, so guided outputs are spelled with
whole-character tokens.
"""
from __future__ import annotations

import threading
from collections import OrderedDict
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

from rusteeze_b200.engine.guided.json_schema import any_object, schema_to_regex
from rusteeze_b200.engine.guided.regex_fsm import RegexFSM

MASK_CACHE_STATES = 2048


def guide_pattern(g) -> str:
    """The regex of a `GuidedDecodingParams` (exactly one constraint must be set)."""
    import re
    kinds = [k for k in ("choice", "regex", "json_schema", "json_object", "grammar")
             if getattr(g, k, None) not in (None, False, [], "")]
    if len(kinds) != 1:
        raise ValueError(f"guided decoding needs exactly one of choice / regex / json_schema / json_object, "
                         f"got {kinds or 'none'}")
    k = kinds[0]
    if k == "choice":
        return "(" + "|".join(re.escape(str(c)) for c in g.choice) + ")"
    if k == "regex":
        return g.regex
    if k == "json_schema":
        return schema_to_regex(g.json_schema)
    if k == "json_object":
        return any_object()
    raise ValueError("grammar-guided decoding is not supported; use regex, choice or json_schema")


class TokenIndex:
    """Token texts and the character trie over them, for one tokenizer."""

    def __init__(self, tokenizer, vocab_size: int):
        self.vocab_size = vocab_size
        # a token's text is what it adds after other text: decoded alone, a SentencePiece
        # token drops its leading space ("▁hello" -> "hello"), so each token is decoded
        # after a fixed plain prefix token and the prefix's own text is cut off
        prefix, ptext = self._prefix(tokenizer)
        texts: List[str] = []
        for i in range(vocab_size):
            try:
                if prefix is not None:
                    full = tokenizer.decode([prefix, i], True)
                    t = full[len(ptext):] if full.startswith(ptext) else tokenizer.decode([i], True)
                else:
                    t = tokenizer.decode([i], True)
            except Exception:  # noqa: BLE001 -- ids the tokenizer does not know
                t = ""
            texts.append("" if "�" in t else t)
        self.texts = texts
        # trie: node = [children dict, token ids ending here]
        root: list = [{}, []]
        for i, t in enumerate(texts):
            if not t:
                continue
            node = root
            for ch in t:
                nxt = node[0].get(ch)
                if nxt is None:
                    nxt = node[0][ch] = [{}, []]
                node = nxt
            node[1].append(i)
        self.root = root
        # each token's text as indices into the vocabulary's alphabet (CSR), for the
        # self-loop shortcut below
        alphabet = sorted({ch for t in texts for ch in t})
        pos = {ch: i for i, ch in enumerate(alphabet)}
        self.alphabet = alphabet
        self.tok_ids = np.array([i for i, t in enumerate(texts) if t], dtype=np.int64)
        lens = np.array([len(texts[i]) for i in self.tok_ids], dtype=np.int64)
        self.starts = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
        self.flat = np.fromiter((pos[ch] for i in self.tok_ids for ch in texts[i]), dtype=np.int64,
                                count=int(lens.sum()))

    @staticmethod
    def _prefix(tokenizer):
        """A token that decodes to plain text on its own ("a"), or (None, "")."""
        try:
            ids = tokenizer.encode("a", add_special_tokens=False)
        except Exception:  # noqa: BLE001
            return None, ""
        if len(ids) != 1:
            return None, ""
        t = tokenizer.decode(ids, True)
        return (ids[0], t) if t else (None, "")

    def allowed(self, fsm: RegexFSM, state: int) -> np.ndarray:
        """Bool mask [vocab]: tokens whose whole text keeps the DFA alive from `state`.

        Where most characters lead from `state` back to `state` (inside a JSON string,
        say), a token made only of such characters is allowed as a whole and only the
        others are walked one by one; elsewhere the trie and the DFA are walked together,
        a branch ending where the DFA dies."""
        n = len(self.tok_ids)
        if n > 4096 and state >= 0:
            loops = np.fromiter((fsm.step(state, ch) == state for ch in self.alphabet), dtype=bool,
                                count=len(self.alphabet))
            if loops.mean() > 0.5:
                whole = np.logical_and.reduceat(loops[self.flat], self.starts)
                others = self.tok_ids[~whole]
                if len(others) <= n // 4:
                    mask = np.zeros(self.vocab_size, dtype=bool)
                    mask[self.tok_ids[whole]] = True
                    walk, texts = fsm.walk, self.texts
                    for i in others.tolist():
                        if walk(state, texts[i]) >= 0:
                            mask[i] = True
                    return mask
        mask = np.zeros(self.vocab_size, dtype=bool)
        stack = [(self.root, state)]
        step = fsm.step
        while stack:
            node, st = stack.pop()
            for ch, child in node[0].items():
                ns = step(st, ch)
                if ns < 0:
                    continue
                if child[1]:
                    mask[child[1]] = True
                if child[0]:
                    stack.append((child, ns))
        return mask


_lock = threading.Lock()
_fsms: Dict[str, RegexFSM] = {}
_indexes: Dict[Tuple[int, int], TokenIndex] = {}
_masks: "OrderedDict[Tuple[str, int, int], np.ndarray]" = OrderedDict()


def fsm_for(pattern: str) -> RegexFSM:
    with _lock:
        f = _fsms.get(pattern)
        if f is None:
            f = _fsms[pattern] = RegexFSM(pattern)
        return f


def index_for(tokenizer, vocab_size: int) -> TokenIndex:
    key = (id(tokenizer), vocab_size)
    with _lock:
        ix = _indexes.get(key)
    if ix is None:
        ix = TokenIndex(tokenizer, vocab_size)
        with _lock:
            _indexes[key] = ix
    return ix


class Guide:
    """One sequence's position in its constraint's DFA."""

    __slots__ = ("fsm", "index", "state", "eos_ids")

    def __init__(self, fsm: RegexFSM, index: TokenIndex, eos_ids: Sequence[int], state: Optional[int] = None):
        self.fsm, self.index, self.eos_ids = fsm, index, tuple(eos_ids)
        self.state = fsm.start if state is None else state

    def copy(self) -> "Guide":
        return Guide(self.fsm, self.index, self.eos_ids, self.state)

    @property
    def complete(self) -> bool:
        """The output matches and nothing can follow."""
        return self.fsm.accepting(self.state) and not self.fsm.can_continue(self.state)

    def mask(self, allow_eos: bool = True) -> np.ndarray:
        key = (self.fsm.pattern, id(self.index), self.state)
        with _lock:
            m = _masks.get(key)
            if m is not None:
                _masks.move_to_end(key)
        if m is None:
            m = self.index.allowed(self.fsm, self.state) if self.state >= 0 else \
                np.zeros(self.index.vocab_size, dtype=bool)
            with _lock:
                _masks[key] = m
                while len(_masks) > MASK_CACHE_STATES:
                    _masks.popitem(last=False)
        # EOS where the output is a match, and where no token can continue it (a dead end
        # the vocabulary cannot spell: the request then ends instead of leaving the constraint)
        if allow_eos and (self.fsm.accepting(self.state) or not m.any()):
            m = m.copy()
            for e in self.eos_ids:
                if 0 <= e < m.shape[0]:
                    m[e] = True
        return m

    def stuck(self) -> bool:
        """No token can continue the output and it is not a complete match."""
        if self.state < 0:
            return True
        return not self.fsm.accepting(self.state) and not self.mask(allow_eos=False).any()

    def advance(self, tok: int) -> None:
        if tok in self.eos_ids:
            return
        t = self.index.texts[tok] if 0 <= tok < len(self.index.texts) else ""
        self.state = self.fsm.walk(self.state, t) if t else -1
