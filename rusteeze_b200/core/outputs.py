"""Engine outputs returned by `LLMEngine.step()` and `LLM.generate()`.

Counterpart of the reference's generation response types
(crates/rusteeze-core/src/response.rs:12,199) at the engine boundary; the
OpenAI wire format lives in `rusteeze_b200.api.schemas`.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional

from rusteeze_b200.core.types import RequestMetrics


@dataclass
class CompletionOutput:
    index: int
    text: str
    token_ids: List[int]
    cumulative_logprob: Optional[float] = None
    logprobs: Optional[List[Dict[int, float]]] = None
    finish_reason: Optional[str] = None
    stop_reason: Optional[object] = None

    def finished(self) -> bool:
        return self.finish_reason is not None


@dataclass
class RequestOutput:
    request_id: str
    prompt: Optional[str]
    prompt_token_ids: List[int]
    outputs: List[CompletionOutput]
    finished: bool
    metrics: Optional[RequestMetrics] = None
    num_cached_tokens: int = 0
    # text appended since the previous RequestOutput for this request (streaming)
    delta_text: List[str] = field(default_factory=list)
    # per prompt token: None for the first, else {token id: logprob} with the prompt's own
    # token and the `prompt_logprobs` most likely ones (when the request asked for them)
    prompt_logprobs: Optional[List[Optional[Dict[int, float]]]] = None
