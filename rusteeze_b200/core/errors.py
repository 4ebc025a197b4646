"""Error hierarchy with retry classification and HTTP mapping.

Mirrors the reference's error enum semantics (crates/rusteeze-core/src/error.rs:
`is_retryable` :463, `error_code` :474, `suggested_http_status` :498) as a
Python exception tree.  The API layer turns any `RusteezeError` into an
OpenAI-style error JSON body with `to_openai()`.
"""
from __future__ import annotations

from typing import Optional


class RusteezeError(Exception):
    http_status: int = 500
    error_type: str = "internal_error"
    code: str = "internal_error"
    retryable: bool = False

    def __init__(self, message: str = "", *, param: Optional[str] = None,
                 code: Optional[str] = None) -> None:
        super().__init__(message)
        self.message = message or self.__class__.__name__
        self.param = param
        if code is not None:
            self.code = code

    def is_retryable(self) -> bool:
        return self.retryable

    def to_openai(self) -> dict:
        return {"error": {"message": self.message, "type": self.error_type,
                          "param": self.param, "code": self.code}}


class InvalidRequestError(RusteezeError):
    http_status = 400
    error_type = "invalid_request_error"
    code = "invalid_request"


class ContextLengthExceededError(InvalidRequestError):
    code = "context_length_exceeded"


class PayloadTooLargeError(RusteezeError):
    http_status = 413
    error_type = "invalid_request_error"
    code = "payload_too_large"


class AuthenticationError(RusteezeError):
    http_status = 401
    error_type = "authentication_error"
    code = "invalid_api_key"


class NotFoundError(RusteezeError):
    http_status = 404
    error_type = "not_found_error"
    code = "not_found"


class RateLimitError(RusteezeError):
    http_status = 429
    error_type = "rate_limit_error"
    code = "rate_limit_exceeded"
    retryable = True


class ServiceUnavailableError(RusteezeError):
    http_status = 503
    error_type = "service_unavailable"
    code = "engine_unavailable"
    retryable = True


class OutOfMemoryError(RusteezeError):
    http_status = 503
    error_type = "server_error"
    code = "out_of_memory"
    retryable = True


class RequestTimeoutError(RusteezeError):
    http_status = 504
    error_type = "timeout_error"
    code = "timeout"
    retryable = True


class RequestAbortedError(RusteezeError):
    http_status = 499
    error_type = "aborted"
    code = "aborted"


class ModelLoadError(RusteezeError):
    error_type = "model_error"
    code = "model_load_failed"


class ConfigError(RusteezeError):
    http_status = 400
    error_type = "config_error"
    code = "invalid_config"


class KernelError(RusteezeError):
    """A device kernel reported an error status (e.g. a bounded wait expired)."""
    error_type = "server_error"
    code = "kernel_error"
    retryable = True


class DistributedError(RusteezeError):
    """A peer rank failed, timed out, or left the group."""
    error_type = "server_error"
    code = "distributed_error"
    retryable = True
