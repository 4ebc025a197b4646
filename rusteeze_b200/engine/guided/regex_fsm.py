"""A regular-expression automaton for constrained decoding.

A pattern is parsed into a syntax tree, built into a Thompson NFA over character sets,
and run as a DFA whose states (epsilon-closed NFA state sets) and transitions are made on
first use and then memoised, so a guide pays for the states its outputs actually visit.
The language is the pattern's full match (`re.fullmatch`).

Syntax: literals; escapes \\d \\D \\w \\W \\s \\S \\t \\n \\r \\f \\v \\xHH \\uXXXX and
escaped punctuation; `.` (any character but newline); classes `[a-z_]`, `[^...]` with
escapes; groups `( )`, `(?: )`, `(?P<name> )`; alternation `|`; quantifiers `* + ?
{n} {n,} {n,m}` (a trailing `?` or `+` is accepted and changes nothing: the language is
the same); `^` at the start and `$` at the end.  Back-references and look-arounds are
refused (they are not regular).
"""
from __future__ import annotations

import bisect
import threading
from typing import Dict, FrozenSet, List, Optional, Tuple

MAX_CP = 0x10FFFF
MAX_NFA_STATES = 400_000
MAX_REPEAT = 1000

Ranges = Tuple[Tuple[int, int], ...]


def _norm(ranges) -> Ranges:
    rs = sorted(ranges)
    out: List[List[int]] = []
    for a, b in rs:
        if out and a <= out[-1][1] + 1:
            out[-1][1] = max(out[-1][1], b)
        else:
            out.append([a, b])
    return tuple((a, b) for a, b in out)


def _negate(r: Ranges) -> Ranges:
    out, lo = [], 0
    for a, b in r:
        if a > lo:
            out.append((lo, a - 1))
        lo = b + 1
    if lo <= MAX_CP:
        out.append((lo, MAX_CP))
    return tuple(out)


_DIGIT = ((48, 57),)
_WORD = _norm([(48, 57), (65, 90), (95, 95), (97, 122)])
_SPACE = _norm([(9, 13), (32, 32)])
_DOT = _negate(((10, 10),))
_CLASS_ESC = {"d": _DIGIT, "D": _negate(_DIGIT), "w": _WORD, "W": _negate(_WORD), "s": _SPACE,
              "S": _negate(_SPACE)}
_CHAR_ESC = {"t": "\t", "n": "\n", "r": "\r", "f": "\f", "v": "\v", "0": "\0"}


class RegexError(ValueError):
    pass


class _Parser:
    """Recursive-descent parser to (kind, ...) tuples: ("set", ranges), ("cat", [..]),
    ("alt", [..]), ("rep", node, lo, hi or None)."""

    def __init__(self, pattern: str):
        self.p = pattern
        self.i = 0

    def parse(self):
        if self.p.startswith("^"):
            self.i = 1
        node = self._alt()
        if self.i != len(self.p):
            raise RegexError(f"unexpected {self.p[self.i]!r} at {self.i}")
        return node

    def _peek(self) -> Optional[str]:
        return self.p[self.i] if self.i < len(self.p) else None

    def _alt(self):
        parts = [self._cat()]
        while self._peek() == "|":
            self.i += 1
            parts.append(self._cat())
        return parts[0] if len(parts) == 1 else ("alt", parts)

    def _cat(self):
        items = []
        while True:
            c = self._peek()
            if c is None or c in "|)":
                break
            if c == "$" and self.i == len(self.p) - 1:
                self.i += 1
                break
            items.append(self._quant(self._atom()))
        return items[0] if len(items) == 1 else ("cat", items)

    def _quant(self, node):
        while True:
            c = self._peek()
            if c == "*":
                lo, hi = 0, None
                self.i += 1
            elif c == "+":
                lo, hi = 1, None
                self.i += 1
            elif c == "?":
                lo, hi = 0, 1
                self.i += 1
            elif c == "{" and self._counted() is not None:
                lo, hi = self._counted(consume=True)
            else:
                return node
            if self._peek() in ("?", "+"):
                self.i += 1               # lazy / possessive: the same language
            if (hi if hi is not None else lo) > MAX_REPEAT:
                raise RegexError(f"repetition bound above {MAX_REPEAT}")
            node = ("rep", node, lo, hi)

    def _counted(self, consume: bool = False):
        j = self.p.find("}", self.i)
        if j < 0:
            return None
        body = self.p[self.i + 1:j]
        try:
            if "," in body:
                a, b = body.split(",", 1)
                lo, hi = int(a), (int(b) if b.strip() else None)
            else:
                lo = hi = int(body)
        except ValueError:
            return None
        if hi is not None and hi < lo:
            raise RegexError(f"bad repetition {{{body}}}")
        if consume:
            self.i = j + 1
        return lo, hi

    def _escape(self, in_class: bool):
        self.i += 1
        if self.i >= len(self.p):
            raise RegexError("trailing backslash")
        c = self.p[self.i]
        self.i += 1
        if c in _CLASS_ESC:
            return _CLASS_ESC[c]
        if c in _CHAR_ESC:
            return ((ord(_CHAR_ESC[c]),) * 2,)
        if c in "xu":
            n = 2 if c == "x" else 4
            h = self.p[self.i:self.i + n]
            if len(h) != n:
                raise RegexError(f"bad \\{c} escape")
            self.i += n
            v = int(h, 16)
            return ((v, v),)
        if c.isdigit() or (c in "bBAZz" and not in_class):
            raise RegexError(f"\\{c} is not supported")
        return ((ord(c), ord(c)),)

    def _class(self):
        self.i += 1
        neg = self._peek() == "^"
        if neg:
            self.i += 1
        ranges = []
        first = True
        while True:
            c = self._peek()
            if c is None:
                raise RegexError("unterminated character class")
            if c == "]" and not first:
                self.i += 1
                break
            first = False
            if c == "\\":
                r = self._escape(True)
            else:
                self.i += 1
                r = ((ord(c), ord(c)),)
            if (len(r) == 1 and r[0][0] == r[0][1] and self._peek() == "-" and self.i + 1 < len(self.p)
                    and self.p[self.i + 1] != "]"):
                self.i += 1
                c2 = self._peek()
                if c2 == "\\":
                    r2 = self._escape(True)
                else:
                    self.i += 1
                    r2 = ((ord(c2), ord(c2)),)
                if len(r2) != 1 or r2[0][0] != r2[0][1] or r2[0][0] < r[0][0]:
                    raise RegexError("bad range in character class")
                r = ((r[0][0], r2[0][0]),)
            ranges.extend(r)
        rs = _norm(ranges)
        return ("set", _negate(rs) if neg else rs)

    def _atom(self):
        c = self._peek()
        if c == "(":
            self.i += 1
            if self.p.startswith("?:", self.i):
                self.i += 2
            elif self.p.startswith("?P<", self.i):
                j = self.p.find(">", self.i)
                if j < 0:
                    raise RegexError("bad group name")
                self.i = j + 1
            elif self._peek() == "?":
                raise RegexError("look-arounds and inline flags are not supported")
            node = self._alt()
            if self._peek() != ")":
                raise RegexError("missing )")
            self.i += 1
            return node
        if c == "[":
            return self._class()
        if c == ".":
            self.i += 1
            return ("set", _DOT)
        if c == "\\":
            return ("set", self._escape(False))
        if c in "*+?":
            raise RegexError(f"nothing to repeat at {self.i}")
        self.i += 1
        return ("set", ((ord(c), ord(c)),))


class _NFA:
    def __init__(self):
        self.eps: List[List[int]] = []
        self.edges: List[List[Tuple[int, int]]] = []      # (charset id, target)
        self.sets: List[Ranges] = []
        self._set_ids: Dict[Ranges, int] = {}

    def new(self) -> int:
        if len(self.eps) >= MAX_NFA_STATES:
            raise RegexError("pattern too large")
        self.eps.append([])
        self.edges.append([])
        return len(self.eps) - 1

    def set_id(self, r: Ranges) -> int:
        k = self._set_ids.get(r)
        if k is None:
            k = self._set_ids[r] = len(self.sets)
            self.sets.append(r)
        return k

    def build(self, node) -> Tuple[int, int]:
        """Fragment (start, end) for a syntax node."""
        kind = node[0]
        if kind == "set":
            s, e = self.new(), self.new()
            self.edges[s].append((self.set_id(node[1]), e))
            return s, e
        if kind == "cat":
            if not node[1]:                    # the empty pattern: only the empty string
                s = self.new()
                return s, s
            s, e = self.build(node[1][0])
            for sub in node[1][1:]:
                s2, e2 = self.build(sub)
                self.eps[e].append(s2)
                e = e2
            return s, e
        if kind == "alt":
            s, e = self.new(), self.new()
            for sub in node[1]:
                s2, e2 = self.build(sub)
                self.eps[s].append(s2)
                self.eps[e2].append(e)
            return s, e
        if kind == "rep":
            _, sub, lo, hi = node
            s = cur = self.new()
            for _ in range(lo):
                a, b = self.build(sub)
                self.eps[cur].append(a)
                cur = b
            if hi is None:
                a, b = self.build(sub)
                self.eps[cur].append(a)
                self.eps[b].append(a)
                e = self.new()
                self.eps[cur].append(e)
                self.eps[b].append(e)
                return s, e
            e = self.new()
            self.eps[cur].append(e)
            for _ in range(hi - lo):
                a, b = self.build(sub)
                self.eps[cur].append(a)
                self.eps[b].append(e)
                cur = b
            return s, e
        raise RegexError(f"unknown node {kind}")


def _contains(r: Ranges, cp: int) -> bool:
    i = bisect.bisect_right(r, (cp, MAX_CP + 1)) - 1
    return i >= 0 and r[i][0] <= cp <= r[i][1]


class RegexFSM:
    """DFA of a pattern, built lazily.  States are small ints; -1 is the dead state."""

    DEAD = -1

    def __init__(self, pattern: str):
        self.pattern = pattern
        tree = _Parser(pattern).parse()
        nfa = _NFA()
        s, e = nfa.build(tree)
        self._nfa = nfa
        self._final = e
        self._sets: List[FrozenSet[int]] = []
        self._ids: Dict[FrozenSet[int], int] = {}
        self._trans: List[Dict[str, int]] = []
        self._accept: List[bool] = []
        self._live: List[bool] = []
        # states and transitions are added on first use; engines on several threads (data-
        # parallel replicas in one process) may share one automaton
        self._lock = threading.Lock()
        self.start = self._state(self._closure([s]))

    def _closure(self, states) -> FrozenSet[int]:
        seen = set(states)
        stack = list(states)
        eps = self._nfa.eps
        while stack:
            x = stack.pop()
            for y in eps[x]:
                if y not in seen:
                    seen.add(y)
                    stack.append(y)
        return frozenset(seen)

    def _state(self, ss: FrozenSet[int]) -> int:
        k = self._ids.get(ss)
        if k is None:
            k = self._ids[ss] = len(self._sets)
            self._sets.append(ss)
            self._trans.append({})
            self._accept.append(self._final in ss)
            self._live.append(any(self._nfa.edges[x] for x in ss))
        return k

    @property
    def num_states(self) -> int:
        return len(self._sets)

    def step(self, state: int, ch: str) -> int:
        if state < 0:
            return -1
        t = self._trans[state]
        nxt = t.get(ch)
        if nxt is not None:
            return nxt
        cp = ord(ch)
        sets, edges = self._nfa.sets, self._nfa.edges
        with self._lock:
            nxt = t.get(ch)
            if nxt is None:
                targets = [y for x in self._sets[state] for sid, y in edges[x] if _contains(sets[sid], cp)]
                nxt = self._state(self._closure(targets)) if targets else -1
                t[ch] = nxt
        return nxt

    def walk(self, state: int, text: str) -> int:
        for ch in text:
            state = self.step(state, ch)
            if state < 0:
                return -1
        return state

    def accepting(self, state: int) -> bool:
        return state >= 0 and self._accept[state]

    def can_continue(self, state: int) -> bool:
        """Whether some character leads on from `state` (if not, the match is complete)."""
        return state >= 0 and self._live[state]

    def fullmatch(self, text: str) -> bool:
        return self.accepting(self.walk(self.start, text))
