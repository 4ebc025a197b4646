"""OpenAI-compatible request/response models.

Chat types follow crates/rusteeze-api/src/types.rs:8-331 (ChatCompletionRequest,
ChatMessage, responses, chunks with deltas, logprobs, usage, models, health);
the legacy completions request follows crates/rusteeze-core/src/request.rs:
525-594 (prompt as string / list of strings / token ids / list of token id
lists, echo, best_of, logprobs) plus the `RusteezeExtensions` fields
(request.rs:489-523: priority, min_tokens, stop_token_ids, ignore_eos,
use_prefix_cache) and beam search (`use_beam_search`, `length_penalty`,
`early_stopping`, sampling.rs:76-80) accepted at top level as vLLM does.
"""
from __future__ import annotations

import time
from typing import Any, Dict, List, Literal, Optional, Union

from pydantic import BaseModel, ConfigDict, Field


class StreamOptions(BaseModel):
    include_usage: bool = False


class ContentPart(BaseModel):
    model_config = ConfigDict(extra="allow")
    type: str = "text"
    text: Optional[str] = None


class ChatMessage(BaseModel):
    model_config = ConfigDict(extra="allow")
    role: str
    content: Optional[Union[str, List[ContentPart]]] = ""
    name: Optional[str] = None
    # assistant turns that called tools, and the id a tool result answers
    tool_calls: Optional[List[Dict[str, Any]]] = None
    tool_call_id: Optional[str] = None


class _SamplingFields(BaseModel):
    model_config = ConfigDict(extra="ignore")
    model: str = ""
    max_tokens: Optional[int] = None
    temperature: Optional[float] = None
    top_p: Optional[float] = None
    top_k: Optional[int] = None
    min_p: Optional[float] = None
    n: int = 1
    best_of: Optional[int] = None
    stream: bool = False
    stream_options: Optional[StreamOptions] = None
    stop: Optional[Union[str, List[str]]] = None
    presence_penalty: Optional[float] = None
    frequency_penalty: Optional[float] = None
    repetition_penalty: Optional[float] = None
    logit_bias: Optional[Dict[str, float]] = None
    seed: Optional[int] = None
    user: Optional[str] = None
    # extensions
    priority: int = 0
    min_tokens: int = 0
    stop_token_ids: Optional[List[int]] = None
    ignore_eos: bool = False
    skip_special_tokens: bool = True
    include_stop_str_in_output: bool = False
    # beam search (sampling.rs:76-80): `best_of` (or `n`) is the width
    use_beam_search: bool = False
    length_penalty: float = 1.0
    early_stopping: Union[bool, Literal["never"]] = False
    # structured output: OpenAI `response_format` ({"type": "json_object"} or
    # {"type": "json_schema", "json_schema": {"schema": ...}}) and vLLM's guided_* fields
    response_format: Optional[Dict[str, Any]] = None
    guided_json: Optional[Union[Dict[str, Any], str]] = None
    guided_regex: Optional[str] = None
    guided_choice: Optional[List[str]] = None


class ChatCompletionRequest(_SamplingFields):
    messages: List[ChatMessage]
    logprobs: Optional[bool] = False
    top_logprobs: Optional[int] = None
    max_completion_tokens: Optional[int] = None
    add_generation_prompt: bool = True
    chat_template: Optional[str] = None
    tools: Optional[List[Dict[str, Any]]] = None
    tool_choice: Optional[Any] = None


class CompletionRequest(_SamplingFields):
    prompt: Union[str, List[str], List[int], List[List[int]]]
    echo: bool = False
    logprobs: Optional[int] = None
    suffix: Optional[str] = None


class EmbeddingRequest(BaseModel):
    """crates/rusteeze-core/src/request.rs:627-672 (types the reference never routes), plus
    `pooling` and `normalize`."""
    model_config = ConfigDict(extra="ignore")
    model: str = ""
    input: Union[str, List[str], List[int], List[List[int]]]
    encoding_format: Literal["float", "base64"] = "float"
    dimensions: Optional[int] = None
    user: Optional[str] = None
    pooling: Literal["last", "mean"] = "last"
    normalize: bool = True


class TokenizeRequest(BaseModel):
    """`/tokenize`: a prompt, or chat messages rendered with the server's chat template."""
    model_config = ConfigDict(extra="ignore")
    model: str = ""
    prompt: Optional[str] = None
    messages: Optional[List[ChatMessage]] = None
    add_special_tokens: bool = True
    add_generation_prompt: bool = True


class DetokenizeRequest(BaseModel):
    model_config = ConfigDict(extra="ignore")
    model: str = ""
    tokens: List[int]
    skip_special_tokens: bool = False


class EmbeddingData(BaseModel):
    object: Literal["embedding"] = "embedding"
    embedding: Union[List[float], str]
    index: int


class EmbeddingUsage(BaseModel):
    prompt_tokens: int = 0
    total_tokens: int = 0


class EmbeddingResponse(BaseModel):
    object: Literal["list"] = "list"
    data: List[EmbeddingData]
    model: str
    usage: EmbeddingUsage


class Usage(BaseModel):
    prompt_tokens: int = 0
    completion_tokens: int = 0
    total_tokens: int = 0


class TopLogProb(BaseModel):
    token: str
    logprob: float
    bytes: Optional[List[int]] = None


class TokenLogProb(TopLogProb):
    top_logprobs: List[TopLogProb] = Field(default_factory=list)


class ChatLogProbs(BaseModel):
    content: Optional[List[TokenLogProb]] = None


class ChatChoice(BaseModel):
    index: int
    message: ChatMessage
    finish_reason: Optional[str] = None
    logprobs: Optional[ChatLogProbs] = None


class ChatCompletionResponse(BaseModel):
    id: str
    object: Literal["chat.completion"] = "chat.completion"
    created: int = Field(default_factory=lambda: int(time.time()))
    model: str
    choices: List[ChatChoice]
    usage: Usage
    system_fingerprint: Optional[str] = None


class ChatDelta(BaseModel):
    role: Optional[str] = None
    content: Optional[str] = None
    tool_calls: Optional[List[Dict[str, Any]]] = None


class ChatChunkChoice(BaseModel):
    index: int
    delta: ChatDelta
    finish_reason: Optional[str] = None
    logprobs: Optional[ChatLogProbs] = None


class ChatCompletionChunk(BaseModel):
    id: str
    object: Literal["chat.completion.chunk"] = "chat.completion.chunk"
    created: int = Field(default_factory=lambda: int(time.time()))
    model: str
    choices: List[ChatChunkChoice]
    usage: Optional[Usage] = None
    system_fingerprint: Optional[str] = None


class CompletionLogProbs(BaseModel):
    tokens: List[str] = Field(default_factory=list)
    token_logprobs: List[Optional[float]] = Field(default_factory=list)
    top_logprobs: List[Optional[Dict[str, float]]] = Field(default_factory=list)
    text_offset: List[int] = Field(default_factory=list)


class CompletionChoice(BaseModel):
    index: int
    text: str
    finish_reason: Optional[str] = None
    logprobs: Optional[CompletionLogProbs] = None


class CompletionResponse(BaseModel):
    id: str
    object: Literal["text_completion"] = "text_completion"
    created: int = Field(default_factory=lambda: int(time.time()))
    model: str
    choices: List[CompletionChoice]
    usage: Usage
    system_fingerprint: Optional[str] = None


class ModelCard(BaseModel):
    id: str
    object: Literal["model"] = "model"
    created: int = Field(default_factory=lambda: int(time.time()))
    owned_by: str = "rusteeze"
    max_model_len: Optional[int] = None


class ModelList(BaseModel):
    object: Literal["list"] = "list"
    data: List[ModelCard]


class HealthResponse(BaseModel):
    status: str
    version: str
    uptime_seconds: int
    requests_processed: int
    waiting_requests: int
    running_requests: int
    gpu_memory_usage: float
    kv_cache_usage: float
