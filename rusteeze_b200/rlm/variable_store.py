"""Typed variable store of the RLM REPL.

Semantics from crates/rusteeze-engine/src/variable_store.rs: typed values
(text, tokens, number, bool, list, map, null; :27-78), constant-size
metadata so a 10M-character prompt never enters the model context, only its
description (:239-338), a memory limit (1 GiB default, :358-420), the
`Final` / `FinalVar` termination slots (:600-700) and a debug snapshot
(:701-713).
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional

from rusteeze_b200.core.errors import InvalidRequestError

PREVIEW_CHARS = 120


def _size(v: Any) -> int:
    if v is None:
        return 0
    if isinstance(v, str):
        return len(v.encode("utf-8", errors="ignore"))
    if isinstance(v, (bool, int, float)):
        return 8
    if isinstance(v, (list, tuple)):
        return sum(_size(x) for x in v) + 8 * len(v)
    if isinstance(v, dict):
        return sum(_size(k) + _size(x) for k, x in v.items())
    return len(str(v))


def type_name(v: Any) -> str:
    if v is None:
        return "null"
    if isinstance(v, bool):
        return "bool"
    if isinstance(v, (int, float)):
        return "number"
    if isinstance(v, str):
        return "text"
    if isinstance(v, (list, tuple)):
        if v and all(isinstance(x, int) and not isinstance(x, bool) for x in v):
            return "tokens"
        return "list"
    if isinstance(v, dict):
        return "map"
    return "text"


@dataclass
class VarMeta:
    name: str
    type: str
    length: int
    bytes: int
    preview: str

    def describe(self) -> str:
        unit = {"text": "chars", "list": "items", "tokens": "tokens", "map": "keys"}.get(self.type, "")
        p = self.preview.replace("\n", " ")
        return f"{self.name}: {self.type}" + (f" ({self.length} {unit})" if unit else "") + (f' "{p}"' if p else "")


@dataclass
class VariableStore:
    memory_limit: int = 1 << 30
    _vars: Dict[str, Any] = field(default_factory=dict)
    _bytes: int = 0
    final: Optional[str] = None
    final_var: Optional[str] = None

    def set(self, name: str, value: Any) -> None:
        new = _size(value)
        old = _size(self._vars.get(name))
        if self._bytes - old + new > self.memory_limit:
            raise InvalidRequestError(f"variable store memory limit ({self.memory_limit} bytes) exceeded by {name!r}")
        self._vars[name] = value
        self._bytes += new - old

    def get(self, name: str) -> Any:
        if name not in self._vars:
            raise KeyError(name)
        return self._vars[name]

    def has(self, name: str) -> bool:
        return name in self._vars

    def delete(self, name: str) -> None:
        if name in self._vars:
            self._bytes -= _size(self._vars.pop(name))

    def names(self) -> List[str]:
        return list(self._vars)

    @property
    def used_bytes(self) -> int:
        return self._bytes

    def meta(self, name: str) -> VarMeta:
        v = self._vars[name]
        t = type_name(v)
        if isinstance(v, str):
            n, prev = len(v), v[:PREVIEW_CHARS]
        elif isinstance(v, (list, tuple, dict)):
            n = len(v)
            prev = (str(v[0])[:PREVIEW_CHARS] if isinstance(v, (list, tuple)) and v else
                    ", ".join(list(map(str, v.keys()))[:8]) if isinstance(v, dict) else "")
        else:
            n, prev = 1, str(v)[:PREVIEW_CHARS]
        return VarMeta(name, t, n, _size(v), prev)

    def metadata_block(self, exclude_internal: bool = False) -> str:
        lines = [self.meta(n).describe() for n in self._vars if not (exclude_internal and n.startswith("__"))]
        return "\n".join(lines) if lines else "(no variables)"

    # ---- termination
    def set_final(self, value: str) -> None:
        self.final = value

    def set_final_var(self, name: str) -> None:
        if name not in self._vars:
            raise KeyError(name)
        self.final_var = name

    def final_value(self) -> Optional[str]:
        if self.final is not None:
            return self.final
        if self.final_var is not None:
            v = self._vars[self.final_var]
            return v if isinstance(v, str) else json.dumps(v)
        return None

    def is_terminated(self) -> bool:
        return self.final is not None or self.final_var is not None

    def snapshot(self) -> Dict[str, Any]:
        return {"vars": {n: self.meta(n).__dict__ for n in self._vars}, "bytes": self._bytes,
                "final": self.final, "final_var": self.final_var}
