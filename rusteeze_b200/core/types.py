"""Enums and small value types shared across layers.

Counterparts of crates/rusteeze-core/src/types.rs: `RequestStatus` (:100),
`FinishReason` (:149-183), `TokenUsage` (:230), `PerformanceMetrics`
(:276-318), `ModelArchitecture` (:344), `QuantizationType` (:393).
"""
from __future__ import annotations

import enum
import itertools
import time
from dataclasses import dataclass, field
from typing import Optional

_req_counter = itertools.count()


def new_request_id(prefix: str = "req") -> str:
    return f"{prefix}-{int(time.time() * 1000):x}-{next(_req_counter)}"


class RequestStatus(str, enum.Enum):
    WAITING = "waiting"
    RUNNING = "running"
    SWAPPED = "swapped"
    FINISHED_STOPPED = "finished_stopped"
    FINISHED_LENGTH = "finished_length"
    FINISHED_ABORTED = "finished_aborted"
    FINISHED_IGNORED = "finished_ignored"

    @property
    def is_finished(self) -> bool:
        return self.value.startswith("finished")


class FinishReason(str, enum.Enum):
    STOP = "stop"
    LENGTH = "length"
    ABORT = "abort"
    CONTENT_FILTER = "content_filter"
    TOOL_CALLS = "tool_calls"


class Role(str, enum.Enum):
    SYSTEM = "system"
    USER = "user"
    ASSISTANT = "assistant"
    TOOL = "tool"


class ModelArchitecture(str, enum.Enum):
    LLAMA = "llama"
    MISTRAL = "mistral"
    MIXTRAL = "mixtral"
    QWEN2 = "qwen2"
    PHI3 = "phi3"
    GEMMA = "gemma"
    GEMMA2 = "gemma2"

    @classmethod
    def from_hf(cls, model_type: str, architectures=None) -> "ModelArchitecture":
        mt = (model_type or "").lower()
        table = {"llama": cls.LLAMA, "mistral": cls.MISTRAL, "mixtral": cls.MIXTRAL,
                 "qwen2": cls.QWEN2, "phi3": cls.PHI3, "gemma": cls.GEMMA,
                 "gemma2": cls.GEMMA2}
        if mt in table:
            return table[mt]
        for a in architectures or []:
            al = a.lower()
            for k, v in sorted(table.items(), key=lambda kv: -len(kv[0])):
                if al.startswith(k):
                    return v
        from rusteeze_b200.core.errors import ModelLoadError
        raise ModelLoadError(f"unsupported model_type {model_type!r} / {architectures}")


class QuantizationType(str, enum.Enum):
    NONE = "none"
    FP8_BLOCK = "fp8_block"     # e4m3 weights, 128x128 weight scales, 1x128 activation scales


@dataclass
class TokenUsage:
    prompt_tokens: int = 0
    completion_tokens: int = 0

    @property
    def total_tokens(self) -> int:
        return self.prompt_tokens + self.completion_tokens

    def to_dict(self) -> dict:
        return {"prompt_tokens": self.prompt_tokens,
                "completion_tokens": self.completion_tokens,
                "total_tokens": self.total_tokens}


@dataclass
class RequestMetrics:
    """Per-request timing (seconds, `time.monotonic()` clock)."""
    arrival_time: float = field(default_factory=time.monotonic)
    first_scheduled_time: Optional[float] = None
    first_token_time: Optional[float] = None
    last_token_time: Optional[float] = None
    finished_time: Optional[float] = None
    num_generated: int = 0

    @property
    def ttft(self) -> Optional[float]:
        if self.first_token_time is None:
            return None
        return self.first_token_time - self.arrival_time

    @property
    def tpot(self) -> Optional[float]:
        """Mean time per output token after the first."""
        if self.first_token_time is None or self.last_token_time is None or self.num_generated < 2:
            return None
        return (self.last_token_time - self.first_token_time) / (self.num_generated - 1)

    @property
    def queue_time(self) -> Optional[float]:
        if self.first_scheduled_time is None:
            return None
        return self.first_scheduled_time - self.arrival_time

    @property
    def e2e_latency(self) -> Optional[float]:
        if self.finished_time is None:
            return None
        return self.finished_time - self.arrival_time
