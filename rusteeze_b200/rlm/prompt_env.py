"""RLM REPL environment: operation parsing, execution and limits.

The model drives the environment with one operation per turn, written as a
function-call line anywhere in its output (matched case-insensitively; the
first recognised line wins; anything else is THINK).  Operation set and
limits follow crates/rusteeze-engine/src/prompt_env.rs (ops :27-62, limits:
50 iterations, depth 3, 1000 sub-calls, 600 s session :459-476, metadata
prompts :329-449, adaptive chunking :1239-1318) and the parser of
crates/rusteeze-engine/src/recursive_engine.rs:591-754:

  PEEK(start, end)              bytes [start, end) of the prompt (UTF-8 safe)
  DECOMPOSE(chunk, overlap)     prompt -> __chunks__ (sentence/paragraph aware)
  SEARCH(pattern)               regex search over the prompt (the reference
                                does a case-insensitive substring match,
                                prompt_env.rs:823-831; invalid regexes and
                                ones at risk of catastrophic backtracking
                                fall back to that)
  SET_VAR(name, value) / GET_VAR(name)
  SUBCALL(text, instruction)    one sub-model call on literal text
  SUBCALL_VAR(var, instruction) one sub-model call on a variable
  BATCH_SUBCALL(listvar, instr) one sub-call per list item -- submitted
                                CONCURRENTLY so they batch on the GPU
  TRANSFORM(src, dst, op)       split/join/filter/sort/count/truncate/grep,
                                map_subcall(instr) / reduce_subcall(instr)
  FINAL(value) / FINAL_VAR(name)
"""
from __future__ import annotations

import re
import time
from dataclasses import dataclass, field
from typing import List, Optional, Tuple

from rusteeze_b200.rlm.variable_store import VariableStore


@dataclass
class EnvLimits:
    max_iterations: int = 50
    max_depth: int = 3
    max_subcalls: int = 1000
    session_timeout_s: float = 600.0
    max_peek_bytes: int = 16000
    max_search_results: int = 20


# ----------------------------------------------------------------------------- operations
@dataclass
class Op:
    kind: str
    args: Tuple = ()


@dataclass
class PendingSubcall:
    prompt: str
    instruction: str
    target_var: Optional[str] = None       # where the result is stored
    index: Optional[int] = None


@dataclass
class ExecResult:
    stdout: str = ""
    subcalls: List[PendingSubcall] = field(default_factory=list)
    batch_target: Optional[str] = None     # BATCH_SUBCALL / map result list var
    reduce: Optional[Tuple[str, str]] = None  # (target var, instruction) for reduce_subcall
    error: Optional[str] = None
    final: bool = False


_OPS = ["FINAL_VAR", "FINAL", "PEEK", "DECOMPOSE", "SUBCALL_VAR", "SUBCALL", "BATCH_SUBCALL", "SET_VAR",
        "GET_VAR", "SEARCH", "REGEX_SEARCH", "TRANSFORM"]
_NARGS = {"PEEK": 2, "DECOMPOSE": 2, "SUBCALL_VAR": 2, "SUBCALL": 2, "BATCH_SUBCALL": 2, "SET_VAR": 2,
          "TRANSFORM": 3}


_NAME = r"[A-Za-z_][A-Za-z0-9_]{0,63}"
# every character `str.splitlines` breaks a line at
_EOL = r"\n\r\x0b\x0c\x1c\x1d\x1e\x85\u2028\u2029"
_TEXT = rf"[^{_EOL}]{{1,1000}}"            # free text: may hold commas and parentheses
_INT = r"[0-9]{1,9}"
_SEP = r", ?"
# one operation line, as `parse_model_output` reads it: the regex the orchestrator's
# turns are constrained to (guided decoding), so every turn parses to an operation
OP_PATTERN = "(" + "|".join([
    rf"PEEK\({_INT}{_SEP}{_INT}\)",
    rf"SEARCH\({_TEXT}\)",
    rf"DECOMPOSE\({_INT}({_SEP}{_INT})?\)",
    rf"SUBCALL\([^,{_EOL}]{{1,1000}},{_TEXT}\)",
    rf"SUBCALL_VAR\({_NAME}{_SEP}{_TEXT}\)",
    rf"BATCH_SUBCALL\({_NAME}{_SEP}{_TEXT}\)",
    rf"SET_VAR\({_NAME}{_SEP}{_TEXT}\)",
    rf"GET_VAR\({_NAME}\)",
    rf"TRANSFORM\({_NAME}{_SEP}{_NAME}{_SEP}{_TEXT}\)",
    rf"FINAL\({_TEXT}\)",
    rf"FINAL_VAR\({_NAME}\)",
]) + ")"


def _strip(s: str) -> str:
    return s.strip().strip('"').strip("'")


def parse_model_output(text: str) -> Op:
    for raw in text.strip().splitlines():
        line = raw.strip()
        up = line.upper()
        for op in _OPS:
            if up.startswith(op + "(") and line.endswith(")"):
                inner = line[len(op) + 1:-1]
                n = _NARGS.get(op, 1)
                parts = inner.split(",", n - 1) if n > 1 else [inner]
                if len(parts) != n:
                    continue
                args = tuple(_strip(p) for p in parts)
                if op == "REGEX_SEARCH":
                    op = "SEARCH"
                if op in ("PEEK",):
                    try:
                        args = (int(args[0]), int(args[1]))
                    except ValueError:
                        continue
                if op == "DECOMPOSE":
                    try:
                        args = (int(args[0] or 8000), int(args[1] or 200))
                    except ValueError:
                        args = (8000, 200)
                return Op(op, args)
        # DECOMPOSE(chunk) with a single argument
        m = re.match(r"(?i)^DECOMPOSE\((\d+)\)$", line)
        if m:
            return Op("DECOMPOSE", (int(m.group(1)), 200))
    t = text.strip()
    return Op("THINK", (t[:200] + "..." if len(t) > 200 else t,))


# ----------------------------------------------------------------------------- model-written regexes
_MAX_PATTERN = 512


_REGEX_WORKER = (
    "import json,re,sys\n"
    "d=json.loads(sys.stdin.read())\n"
    "rx=re.compile(d['p'],d['f'])\n"
    "if d['lines']:\n"
    "    out=[k for k,ln in enumerate(d['t'].splitlines()) if rx.search(ln)]\n"
    "else:\n"
    "    out=[]\n"
    "    for m in rx.finditer(d['t']):\n"
    "        out.append([m.start(),m.group(0)])\n"
    "        if len(out)>=d['k']:\n"
    "            break\n"
    "sys.stdout.write(json.dumps(out))\n")
REGEX_TIMEOUT_S = 2.0


def _repeats(pat: str) -> bool:
    """Repetition, alternation, several optional items or a backreference: the
    constructs whose backtracking can take super-linear time."""
    optional = len(re.findall(r"(?<!\()\?", pat))
    return any(ch in pat for ch in "*+{|") or optional > 4 or bool(re.search(r"\\[1-9]", pat))


def model_regex(pat: str, text: str, flags: int, lines: bool = False, limit: int = 20):
    """Runs a regex written by the model over `text`: the first `limit` matches as
    (position, match) pairs, or with `lines` the indices of the matching lines.
    Returns None when the pattern is invalid, longer than 512 characters or did not
    finish within REGEX_TIMEOUT_S (the caller then matches it as a plain substring).

    Python's `re` backtracks and has no time limit: nested repeats ((a+)+) take
    exponential time and even `a*a*b` takes minutes over a 20k-character prompt, which
    would stall the engine thread.  Patterns without any repetition or alternation run
    here; the others run in a child interpreter that is killed at the time limit."""
    if len(pat) > _MAX_PATTERN:
        return None
    try:
        rx = re.compile(pat, flags)
    except re.error:
        return None
    if not _repeats(pat):
        if lines:
            return [k for k, ln in enumerate(text.splitlines()) if rx.search(ln)]
        return [(m.start(), m.group(0)) for _, m in zip(range(limit), rx.finditer(text))]
    import json
    import subprocess
    import sys
    try:
        r = subprocess.run([sys.executable, "-I", "-S", "-c", _REGEX_WORKER],
                           input=json.dumps({"p": pat, "f": int(flags), "t": text, "lines": lines, "k": limit}),
                           capture_output=True, text=True, timeout=REGEX_TIMEOUT_S)
    except (subprocess.TimeoutExpired, OSError):
        return None
    if r.returncode != 0:
        return None
    out = json.loads(r.stdout)
    return out if lines else [(int(a), str(b)) for a, b in out]


# ----------------------------------------------------------------------------- chunking
def _break_point(text: str, start: int, target: int) -> int:
    lo = max(start, target - 200)
    region = text[lo:target]
    p = region.rfind("\n\n")
    if p >= 0:
        return lo + p + 2
    best = -1
    for mk in (". ", "! ", "? ", ".\n", "!\n", "?\n"):
        q = region.rfind(mk)
        if q >= 0:
            best = max(best, q + len(mk))
    if best >= 0:
        return lo + best
    for mk in ("\n", " "):
        q = region.rfind(mk)
        if q >= 0:
            return lo + q + 1
    return target


def adaptive_chunk(text: str, chunk: int, overlap: int) -> List[str]:
    """Chunks of about `chunk` characters, cut at paragraph > sentence > line >
    word boundaries, consecutive chunks overlapping by `overlap` characters."""
    if not text:
        return []
    if len(text) <= chunk:
        return [text]
    out, pos = [], 0
    overlap = max(0, min(overlap, chunk // 2))
    while pos < len(text):
        end = min(pos + chunk, len(text))
        bp = _break_point(text, pos, end) if end < len(text) else end
        if bp <= pos:
            bp = end
        out.append(text[pos:bp])
        if bp >= len(text):
            break
        nxt = bp - overlap if bp - overlap > pos else bp
        pos = nxt
    return out


def utf8_slice(text: str, start: int, end: int) -> str:
    b = text.encode("utf-8")
    return b[max(0, start):max(0, end)].decode("utf-8", errors="ignore")


# ----------------------------------------------------------------------------- environment
class PromptEnvironment:
    PROMPT_VAR = "__prompt__"
    CHUNKS_VAR = "__chunks__"

    def __init__(self, prompt: str, limits: Optional[EnvLimits] = None, depth: int = 0,
                 store: Optional[VariableStore] = None):
        self.limits = limits or EnvLimits()
        self.depth = depth
        self.store = store or VariableStore()
        self.store.set(self.PROMPT_VAR, prompt)
        self.iteration = 0
        self.subcalls_made = 0
        self.started = time.monotonic()
        self.history: List[str] = []

    @property
    def prompt(self) -> str:
        return self.store.get(self.PROMPT_VAR)

    def timed_out(self) -> bool:
        return time.monotonic() - self.started > self.limits.session_timeout_s

    def is_terminated(self) -> bool:
        return self.store.is_terminated()

    def initial_metadata(self) -> str:
        p = self.prompt
        return (f"The user prompt is stored in variable {self.PROMPT_VAR} ({len(p)} characters, "
                f"{len(p.encode('utf-8'))} bytes, {p.count(chr(10)) + 1} lines).\n"
                f"Preview: {p[:300]!r}\nVariables:\n{self.store.metadata_block()}")

    def iteration_metadata(self, last_stdout: str) -> str:
        return (f"Iteration {self.iteration}/{self.limits.max_iterations}, depth {self.depth}, "
                f"sub-calls {self.subcalls_made}/{self.limits.max_subcalls}.\nVariables:\n"
                f"{self.store.metadata_block()}\nLast result:\n{last_stdout[:2000]}")

    def _budget(self, n: int) -> Optional[str]:
        if self.subcalls_made + n > self.limits.max_subcalls:
            return f"sub-call limit {self.limits.max_subcalls} reached"
        return None

    def execute(self, op: Op) -> ExecResult:
        k, a = op.kind, op.args
        st = self.store
        try:
            if k == "FINAL":
                st.set_final(a[0])
                return ExecResult(stdout="final answer set", final=True)
            if k == "FINAL_VAR":
                st.set_final_var(a[0])
                return ExecResult(stdout=f"final answer is variable {a[0]}", final=True)
            if k == "PEEK":
                s, e = a
                e = min(e, s + self.limits.max_peek_bytes)
                return ExecResult(stdout=utf8_slice(self.prompt, s, e))
            if k == "DECOMPOSE":
                chunks = adaptive_chunk(self.prompt, max(1, a[0]), a[1])
                st.set(self.CHUNKS_VAR, chunks)
                return ExecResult(stdout=f"{len(chunks)} chunks stored in {self.CHUNKS_VAR}")
            if k == "SEARCH":
                pat = a[0]
                hits = model_regex(pat, self.prompt, re.IGNORECASE | re.MULTILINE,
                                   limit=self.limits.max_search_results)
                if hits is None:
                    low, lp = self.prompt.lower(), pat.lower()
                    hits, i = [], low.find(lp)
                    while i >= 0 and len(hits) < self.limits.max_search_results:
                        hits.append((i, self.prompt[i:i + len(pat)]))
                        i = low.find(lp, i + 1)
                lines = [f"@{pos}: ...{self.prompt[max(0, pos - 60):pos + min(len(g), 200) + 60]!r}..."
                         for pos, g in hits]
                return ExecResult(stdout=f"{len(hits)} match(es)\n" + "\n".join(lines))
            if k == "SET_VAR":
                st.set(a[0], a[1])
                return ExecResult(stdout=f"{a[0]} set")
            if k == "GET_VAR":
                v = st.get(a[0])
                return ExecResult(stdout=str(v)[:4000])
            if k == "SUBCALL":
                err = self._budget(1)
                if err:
                    return ExecResult(error=err)
                return ExecResult(subcalls=[PendingSubcall(a[0], a[1], target_var=f"__subcall_{self.subcalls_made}")])
            if k == "SUBCALL_VAR":
                err = self._budget(1)
                if err:
                    return ExecResult(error=err)
                v = st.get(a[0])
                return ExecResult(subcalls=[PendingSubcall(v if isinstance(v, str) else str(v), a[1],
                                                           target_var=f"{a[0]}__result")])
            if k == "BATCH_SUBCALL":
                items = st.get(a[0])
                if not isinstance(items, (list, tuple)):
                    items = [items]
                err = self._budget(len(items))
                if err:
                    return ExecResult(error=err)
                return ExecResult(subcalls=[PendingSubcall(str(x), a[1], index=i) for i, x in enumerate(items)],
                                  batch_target=f"{a[0]}__results")
            if k == "TRANSFORM":
                return self._transform(a[0], a[1], a[2])
            if k == "THINK":
                return ExecResult(stdout="(no operation recognised; thought recorded)")
        except KeyError as e:
            return ExecResult(error=f"unknown variable {e.args[0]!r}")
        except Exception as e:  # noqa: BLE001 -- reported back to the model
            return ExecResult(error=f"{k} failed: {e}")
        return ExecResult(error=f"unsupported operation {k}")

    def _transform(self, src: str, dst: str, op: str) -> ExecResult:
        st = self.store
        v = st.get(src)
        o = op.strip()
        name, arg = o, None
        m = re.match(r"^(\w+)\s*(?:\((.*)\))?\s*(.*)$", o, re.S)
        if m:
            name = m.group(1).lower()
            arg = m.group(2) if m.group(2) is not None else (m.group(3) or None)
        if name in ("map_subcall", "map"):
            items = v if isinstance(v, list) else [v]
            err = self._budget(len(items))
            if err:
                return ExecResult(error=err)
            return ExecResult(subcalls=[PendingSubcall(str(x), arg or "", index=i) for i, x in enumerate(items)],
                              batch_target=dst)
        if name in ("reduce_subcall", "reduce"):
            err = self._budget(1)
            if err:
                return ExecResult(error=err)
            items = v if isinstance(v, list) else [v]
            joined = "\n---\n".join(map(str, items))
            return ExecResult(subcalls=[PendingSubcall(joined, arg or "", target_var=dst)])
        if name == "split":
            res = str(v).split(arg if arg else ",")
        elif name == "join":
            res = (arg if arg is not None else "\n").join(map(str, v if isinstance(v, list) else [v]))
        elif name in ("filter", "filter_contains"):
            kw = (arg or "").lower()
            res = [x for x in (v if isinstance(v, list) else str(v).splitlines()) if kw in str(x).lower()]
        elif name == "sort":
            res = sorted(v if isinstance(v, list) else str(v).splitlines(), key=str)
        elif name == "count":
            res = len(v) if isinstance(v, (list, str, dict)) else 1
        elif name == "truncate":
            n = int(arg) if arg and arg.isdigit() else 1000
            res = str(v)[:n] if not isinstance(v, list) else v[:n]
        elif name == "grep":
            text_lines = str(v).splitlines()
            idx = model_regex(arg or "", str(v), re.IGNORECASE, lines=True)
            if idx is not None:
                res = "\n".join(text_lines[k] for k in idx)
            else:
                kw = (arg or "").lower()
                res = "\n".join(ln for ln in text_lines if kw in ln.lower())
        else:
            return ExecResult(error=f"unknown transform {op!r}")
        st.set(dst, res)
        return ExecResult(stdout=f"{dst} = {st.meta(dst).describe()}")

    def store_subcall_result(self, sc: PendingSubcall, text: str) -> None:
        if sc.target_var:
            self.store.set(sc.target_var, text)

    def store_batch_results(self, target: str, results: List[str]) -> None:
        self.store.set(target, list(results))
