"""Sampling parameters for text generation.

Field set, defaults and validation ranges follow the reference's
`SamplingParams` (crates/rusteeze-core/src/sampling.rs:25-186, validation
:318-383, strategy selection :424-445).  Here the struct is also the unit that
the GPU sampler packs into a per-row parameter tensor (see
`rusteeze_b200.engine.sampler`).
"""
from __future__ import annotations

import math

import enum
from dataclasses import dataclass, field, asdict
from typing import Dict, List, Optional

from rusteeze_b200.core.errors import InvalidRequestError

# Upper bounds the reference does not have (sampling.rs:357-383 checks only the lower
# ones): one request must not be able to make the engine build an unbounded number of
# sequences, or return a vocabulary-sized logprob table for every token.
MAX_BEST_OF = 256
MAX_LOGPROBS = 20


class SamplingStrategy(str, enum.Enum):
    GREEDY = "greedy"
    RANDOM = "random"
    TOP_K = "top_k"
    TOP_P = "top_p"
    TOP_K_TOP_P = "top_k_top_p"
    MIN_P = "min_p"
    TYPICAL_P = "typical_p"
    MIROSTAT = "mirostat"
    BEAM_SEARCH = "beam_search"


class EarlyStoppingMode(str, enum.Enum):
    FALSE = "false"
    TRUE = "true"
    NEVER = "never"


@dataclass
class GuidedDecodingParams:
    """Structured-output constraints (crates/rusteeze-core/src/sampling.rs:148, declared
    there and not applied): exactly one of `choice`, `regex`, `json_schema` or
    `json_object` (any JSON object) is enforced as a per-step token mask
    (engine/guided); `grammar` is refused."""
    json_schema: Optional[dict] = None
    regex: Optional[str] = None
    choice: Optional[List[str]] = None
    grammar: Optional[str] = None
    json_object: bool = False


@dataclass
class SamplingParams:
    n: int = 1
    max_tokens: Optional[int] = 16
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = -1
    min_p: float = 0.0
    typical_p: float = 0.0
    frequency_penalty: float = 0.0
    presence_penalty: float = 0.0
    repetition_penalty: float = 1.0
    length_penalty: float = 1.0
    best_of: Optional[int] = None
    use_beam_search: bool = False
    early_stopping: EarlyStoppingMode = EarlyStoppingMode.FALSE
    stop: List[str] = field(default_factory=list)
    stop_token_ids: List[int] = field(default_factory=list)
    include_stop_str_in_output: bool = False
    skip_special_tokens: bool = True
    spaces_between_special_tokens: bool = False
    seed: Optional[int] = None
    logit_bias: Dict[int, float] = field(default_factory=dict)
    logprobs: Optional[int] = None
    prompt_logprobs: Optional[int] = None
    ignore_eos: bool = False
    min_tokens: int = 0
    eta_cutoff: float = 0.0
    epsilon_cutoff: float = 0.0
    mirostat_mode: int = 0
    mirostat_tau: float = 5.0
    mirostat_eta: float = 0.1
    guided_decoding: Optional[GuidedDecodingParams] = None
    # "delta": the engine returns an output for the request after every step (streaming);
    # "final_only": one output when it finishes, and its text is detokenised once then
    # (unless stop strings need it token by token) -- offline batches and non-streaming
    # API requests read nothing in between
    output_kind: str = "delta"

    def __post_init__(self) -> None:
        if isinstance(self.stop, str):
            self.stop = [self.stop]
        if self.best_of is None:
            self.best_of = self.n
        self.logit_bias = {int(k): float(v) for k, v in (self.logit_bias or {}).items()}
        self.validate()

    # ---- constructors -------------------------------------------------
    @classmethod
    def greedy(cls, **kw) -> "SamplingParams":
        kw.setdefault("temperature", 0.0)
        return cls(**kw)

    @classmethod
    def beam_search(cls, num_beams: int, **kw) -> "SamplingParams":
        return cls(n=1, best_of=num_beams, use_beam_search=True, temperature=0.0, **kw)

    # ---- validation (ranges as in sampling.rs:318-383) ----------------
    def validate(self) -> None:
        def bad(msg: str) -> None:
            raise InvalidRequestError(msg, param="sampling_params")

        for name in ("temperature", "top_p", "min_p", "typical_p", "frequency_penalty", "presence_penalty",
                     "repetition_penalty", "length_penalty", "eta_cutoff", "epsilon_cutoff", "mirostat_tau",
                     "mirostat_eta"):
            v = getattr(self, name)
            if not math.isfinite(v):
                bad(f"{name} must be a finite number, got {v}")
        if self.temperature < 0.0:
            bad(f"temperature must be >= 0, got {self.temperature}")
        if not 0.0 <= self.epsilon_cutoff < 1.0:
            bad(f"epsilon_cutoff must be in [0, 1), got {self.epsilon_cutoff}")
        if not 0.0 <= self.eta_cutoff < 1.0:
            bad(f"eta_cutoff must be in [0, 1), got {self.eta_cutoff}")
        if self.mirostat_tau < 0.0:
            bad(f"mirostat_tau must be >= 0, got {self.mirostat_tau}")
        if not 0.0 <= self.top_p <= 1.0:
            bad(f"top_p must be in [0, 1], got {self.top_p}")
        if self.top_k == 0 or self.top_k < -1 or self.top_k > 2 ** 31 - 1:
            bad(f"top_k must be -1 (disabled) or in [1, 2**31 - 1], got {self.top_k}")
        if not 0.0 <= self.min_p <= 1.0:
            bad(f"min_p must be in [0, 1], got {self.min_p}")
        if not 0.0 <= self.typical_p <= 1.0:
            bad(f"typical_p must be in [0, 1], got {self.typical_p}")
        if not -2.0 <= self.frequency_penalty <= 2.0:
            bad(f"frequency_penalty must be in [-2, 2], got {self.frequency_penalty}")
        if not -2.0 <= self.presence_penalty <= 2.0:
            bad(f"presence_penalty must be in [-2, 2], got {self.presence_penalty}")
        if not -100.0 <= self.length_penalty <= 100.0:
            bad(f"length_penalty must be in [-100, 100], got {self.length_penalty}")
        if self.repetition_penalty <= 0.0:
            bad(f"repetition_penalty must be > 0, got {self.repetition_penalty}")
        if self.n < 1:
            bad(f"n must be >= 1, got {self.n}")
        if self.best_of < self.n:
            bad(f"best_of ({self.best_of}) must be >= n ({self.n})")
        if self.best_of > MAX_BEST_OF:
            bad(f"best_of / n must be <= {MAX_BEST_OF}, got {self.best_of}")
        if self.max_tokens is not None and self.max_tokens < 1:
            bad(f"max_tokens must be >= 1, got {self.max_tokens}")
        if self.min_tokens < 0:
            bad(f"min_tokens must be >= 0, got {self.min_tokens}")
        if self.max_tokens is not None and self.min_tokens > self.max_tokens:
            bad(f"min_tokens ({self.min_tokens}) must be <= max_tokens ({self.max_tokens})")
        for name in ("logprobs", "prompt_logprobs"):
            v = getattr(self, name)
            if v is not None and not 0 <= v <= MAX_LOGPROBS:
                bad(f"{name} must be in [0, {MAX_LOGPROBS}], got {v}")
        if self.output_kind not in ("delta", "final_only"):
            bad(f"output_kind must be 'delta' or 'final_only', got {self.output_kind!r}")
        if self.mirostat_mode not in (0, 1, 2):
            bad(f"mirostat_mode must be 0, 1 or 2, got {self.mirostat_mode}")
        if self.use_beam_search:
            if self.temperature != 0.0:
                bad("beam search requires temperature 0")
            if self.top_p < 1.0:
                bad("beam search requires top_p 1")
            if self.top_k > 0:
                bad("beam search requires top_k disabled")
        for tok, b in self.logit_bias.items():
            if not -100.0 <= b <= 100.0:
                bad(f"logit_bias for token {tok} must be in [-100, 100], got {b}")

    # ---- queries ------------------------------------------------------
    @property
    def is_greedy(self) -> bool:
        return self.temperature == 0.0 or self.top_k == 1

    def is_deterministic(self) -> bool:
        return self.temperature == 0.0 or self.use_beam_search

    def wants_logprobs(self) -> bool:
        return self.logprobs is not None or self.prompt_logprobs is not None

    def has_penalties(self) -> bool:
        return (self.repetition_penalty != 1.0 or self.frequency_penalty != 0.0
                or self.presence_penalty != 0.0)

    def needs_host_sampling(self) -> bool:
        """Mirostat, typical-p and eta/epsilon cutoffs run on the host sampler; everything
        else (guided decoding too: its constraint is a mask on the logits) is handled by
        the batched sampler."""
        return (self.mirostat_mode > 0 or self.typical_p > 0.0 or self.eta_cutoff > 0.0
                or self.epsilon_cutoff > 0.0 or self.use_beam_search)

    def strategy(self) -> SamplingStrategy:
        if self.use_beam_search:
            return SamplingStrategy.BEAM_SEARCH
        if self.temperature == 0.0:
            return SamplingStrategy.GREEDY
        if self.mirostat_mode > 0:
            return SamplingStrategy.MIROSTAT
        if self.min_p > 0.0:
            return SamplingStrategy.MIN_P
        if self.typical_p > 0.0:
            return SamplingStrategy.TYPICAL_P
        if self.top_k > 0 and self.top_p < 1.0:
            return SamplingStrategy.TOP_K_TOP_P
        if self.top_k > 0:
            return SamplingStrategy.TOP_K
        if self.top_p < 1.0:
            return SamplingStrategy.TOP_P
        return SamplingStrategy.RANDOM

    def clone(self, **overrides) -> "SamplingParams":
        d = asdict(self)
        d["guided_decoding"] = self.guided_decoding
        d.update(overrides)
        return SamplingParams(**d)
