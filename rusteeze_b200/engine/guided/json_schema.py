"""JSON Schema (a common subset) and "any JSON object" as regular expressions for the
guided-decoding automaton.

Supported: `type` string / integer / number / boolean / null / object / array (or a list
of types); `enum`, `const`; `anyOf` / `oneOf`; `$ref` to `#/definitions/...` or
`#/$defs/...` (not recursive); strings with `minLength` / `maxLength` / `pattern`;
arrays with `items`, `minItems` / `maxItems`; objects with `properties` (written in the
schema's order), `required` (optional properties may be left out), no other keys.  A
schema without a type admits any JSON value of bounded depth.

Bounds that keep every output finite (a guided output must be able to end): integers have
at most 16 digits, fractions at most 16, exponents at most 3; between tokens the output may
put one space (`{"a": 1, "b": 2}` and `{"a":1,"b":2}` are both allowed, newlines are not);
values without a schema nest at most `ANY_DEPTH` levels.
"""
from __future__ import annotations

import json
import re
from typing import Any, Dict, List, Optional

WS = "[ ]?"
STRING_CHAR = r'([^"\\\x00-\x1f]|\\["\\/bfnrt]|\\u[0-9a-fA-F]{4})'
STRING = f'"{STRING_CHAR}*"'
INTEGER = r"-?(0|[1-9][0-9]{0,15})"
NUMBER = INTEGER + r"(\.[0-9]{1,16})?([eE][+-]?[0-9]{1,3})?"
BOOLEAN = "(true|false)"
NULL = "null"
ANY_DEPTH = 3
_MAX_BOUND = 1000          # counted repetitions the automaton unrolls


class SchemaError(ValueError):
    pass


def _lit(v: Any) -> str:
    """A JSON literal as a regex."""
    return re.escape(json.dumps(v, ensure_ascii=False, separators=(",", ":")))


def _alt(parts: List[str]) -> str:
    return "(" + "|".join(parts) + ")"


def _list(item: str, lo: int = 0, hi: Optional[int] = None) -> str:
    """`[` items `]` with lo..hi items separated by commas."""
    sep = f"{WS},{WS}"
    if hi == 0:
        return rf"\[{WS}\]"
    more_lo = max(0, lo - 1)
    more = f"({sep}{item})" + ("{%d,}" % more_lo if hi is None else "{%d,%d}" % (more_lo, hi - 1))
    body = f"{item}{more}"
    if lo == 0:
        body = f"({body})?"
    return rf"\[{WS}{body}{WS}\]"


def any_value(depth: int = ANY_DEPTH) -> str:
    """Any JSON value nesting at most `depth` objects / arrays."""
    scalars = [STRING, NUMBER, BOOLEAN, NULL]
    if depth <= 0:
        return _alt(scalars)
    inner = any_value(depth - 1)
    kv = f"{STRING}{WS}:{WS}{inner}"
    obj = rf"\{{{WS}({kv}({WS},{WS}{kv})*)?{WS}\}}"
    return _alt(scalars + [obj, _list(inner)])


def any_object(depth: int = ANY_DEPTH) -> str:
    """A JSON object (response_format json_object) nesting at most `depth` levels."""
    inner = any_value(depth - 1)
    kv = f"{STRING}{WS}:{WS}{inner}"
    return rf"\{{{WS}({kv}({WS},{WS}{kv})*)?{WS}\}}"


class _Compiler:
    def __init__(self, root: Dict):
        self.root = root
        self.stack: List[str] = []

    def _resolve(self, ref: str) -> Dict:
        if not ref.startswith("#/"):
            raise SchemaError(f"only local $ref is supported, got {ref!r}")
        node: Any = self.root
        for part in ref[2:].split("/"):
            if not isinstance(node, dict) or part not in node:
                raise SchemaError(f"unresolvable $ref {ref!r}")
            node = node[part]
        return node

    def value(self, s: Any) -> str:
        if s is True or s == {}:
            return any_value()
        if not isinstance(s, dict):
            raise SchemaError(f"a schema must be an object, got {s!r}")
        if "$ref" in s:
            ref = s["$ref"]
            if ref in self.stack:
                raise SchemaError(f"recursive $ref {ref!r} is not supported")
            self.stack.append(ref)
            try:
                return self.value(self._resolve(ref))
            finally:
                self.stack.pop()
        if "const" in s:
            return _lit(s["const"])
        if "enum" in s:
            if not isinstance(s["enum"], list) or not s["enum"]:
                raise SchemaError("enum must be a non-empty list")
            return _alt([_lit(v) for v in s["enum"]])
        for key in ("anyOf", "oneOf"):
            if key in s:
                if not isinstance(s[key], list) or not s[key]:
                    raise SchemaError(f"{key} must be a non-empty list")
                return _alt([self.value(x) for x in s[key]])
        t = s.get("type")
        if isinstance(t, list):
            return _alt([self.value(dict(s, type=x)) for x in t])
        if t is None:
            if "properties" in s:
                t = "object"
            elif "items" in s:
                t = "array"
            else:
                return any_value()
        if t == "string":
            if "pattern" in s:
                p = s["pattern"]
                return '"(' + (p[1:] if p.startswith("^") else p).rstrip("$") + ')"'
            lo, hi = int(s.get("minLength", 0)), s.get("maxLength")
            if max(lo, int(hi or 0)) > _MAX_BOUND:
                raise SchemaError(f"minLength / maxLength above {_MAX_BOUND} are not supported")
            if lo == 0 and hi is None:
                return STRING
            return f'"{STRING_CHAR}' + ("{%d,}" % lo if hi is None else "{%d,%d}" % (lo, int(hi))) + '"'
        if t == "integer":
            return INTEGER
        if t == "number":
            return NUMBER
        if t == "boolean":
            return BOOLEAN
        if t == "null":
            return NULL
        if t == "array":
            item = self.value(s.get("items", {}))
            lo = int(s.get("minItems", 0))
            hi = s.get("maxItems")
            if max(lo, int(hi or 0)) > _MAX_BOUND:
                raise SchemaError(f"minItems / maxItems above {_MAX_BOUND} are not supported")
            return _list(item, lo, None if hi is None else int(hi))
        if t == "object":
            return self.obj(s)
        raise SchemaError(f"unsupported type {t!r}")

    def obj(self, s: Dict) -> str:
        props = s.get("properties") or {}
        if not props:
            return any_object()
        req = set(s.get("required", []))
        kvs = [(f"{_lit(k)}{WS}:{WS}{self.value(v)}", k in req) for k, v in props.items()]
        sep = f"{WS},{WS}"
        first_req = next((i for i, (_, r) in enumerate(kvs) if r), None)
        if first_req is None:
            # all optional: choose which property comes first, the rest each optional
            alts = []
            for i in range(len(kvs)):
                alts.append(kvs[i][0] + "".join(f"({sep}{kv})?" for kv, _ in kvs[i + 1:]))
            body = f"({_alt(alts)})?"
        else:
            body = "".join(f"({kv}{sep})?" for kv, _ in kvs[:first_req]) + kvs[first_req][0]
            for kv, r in kvs[first_req + 1:]:
                body += f"{sep}{kv}" if r else f"({sep}{kv})?"
        return rf"\{{{WS}{body}{WS}\}}"


def schema_to_regex(schema: Any) -> str:
    """The regex of a schema; a schema this subset cannot express, or a malformed one,
    raises SchemaError (a ValueError: the client's mistake, not the server's)."""
    if isinstance(schema, str):
        schema = json.loads(schema)
    try:
        return _Compiler(schema if isinstance(schema, dict) else {}).value(schema)
    except SchemaError:
        raise
    except (TypeError, AttributeError, KeyError, IndexError, ValueError) as e:
        raise SchemaError(f"malformed JSON schema: {e}") from None
