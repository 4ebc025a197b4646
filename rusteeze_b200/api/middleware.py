"""HTTP middleware: bearer auth, sliding-window rate limit, request ids, timeouts.

Counterpart of crates/rusteeze-api/src/middleware.rs: bearer-token auth
(:20-45), a sliding-window rate limiter keyed by X-API-Key or
X-Forwarded-For / client address that sets X-RateLimit-* headers
(:48-161), request logging (:164-207) and X-Request-ID propagation
(:215-224), and a request timeout (:227-260).  The reference builds the
rate-limit, request-id and timeout layers but never installs them
(routes.rs:202-233); here they are installed by `create_app`.
"""
from __future__ import annotations

import json

import asyncio
import collections
import hmac
import logging
import math
import time
import uuid
from typing import Deque, Dict, Optional

from starlette.middleware.base import BaseHTTPMiddleware
from starlette.requests import Request
from starlette.responses import JSONResponse

from rusteeze_b200.core.errors import AuthenticationError, RateLimitError, RequestTimeoutError

log = logging.getLogger("rusteeze.api")

OPEN_PATHS = {"/health", "/health/live", "/health/ready", "/metrics", "/version"}


def error_response(err) -> JSONResponse:
    return JSONResponse(err.to_openai(), status_code=err.http_status)


class BodyLimitMiddleware:
    """Refuses request bodies above `max_bytes` (server.max_body_bytes) with 413:
    by the Content-Length header before anything is read, and, for a body sent
    without one (chunked), by reading it here up to the limit -- the read stops
    there, so at most max_body_bytes are ever buffered -- and replaying it to the app."""

    def __init__(self, app, max_bytes: int):
        self.app = app
        self.max_bytes = max_bytes

    async def _reject(self, send) -> None:
        from rusteeze_b200.core.errors import PayloadTooLargeError
        err = PayloadTooLargeError(f"request body exceeds {self.max_bytes} bytes")
        body = json.dumps(err.to_openai()).encode()
        await send({"type": "http.response.start", "status": err.http_status,
                    "headers": [(b"content-type", b"application/json"),
                                (b"content-length", str(len(body)).encode())]})
        await send({"type": "http.response.body", "body": body})

    async def __call__(self, scope, receive, send):
        if scope["type"] != "http" or self.max_bytes <= 0:
            return await self.app(scope, receive, send)
        for k, v in scope.get("headers", []):
            if k == b"content-length":
                try:
                    n = int(v)
                except ValueError:
                    n = self.max_bytes + 1
                if n > self.max_bytes:
                    return await self._reject(send)
        if any(k == b"content-length" for k, _ in scope.get("headers", [])):
            return await self.app(scope, receive, send)
        # no length given (chunked): read up to the limit here, then replay it to the app
        chunks, seen, more = [], 0, True
        while more:
            msg = await receive()
            if msg["type"] != "http.request":
                return                       # the client went away
            chunks.append(msg.get("body", b""))
            seen += len(chunks[-1])
            if seen > self.max_bytes:
                return await self._reject(send)
            more = msg.get("more_body", False)
        replayed = False

        async def replay():
            nonlocal replayed
            if not replayed:
                replayed = True
                return {"type": "http.request", "body": b"".join(chunks), "more_body": False}
            return await receive()
        await self.app(scope, replay, send)


class AuthMiddleware(BaseHTTPMiddleware):
    def __init__(self, app, api_key: Optional[str]):
        super().__init__(app)
        self.api_key = api_key

    async def dispatch(self, request: Request, call_next):
        if self.api_key and request.url.path not in OPEN_PATHS and request.method != "OPTIONS":
            h = request.headers.get("authorization", "")
            tok = h[7:] if h.lower().startswith("bearer ") else request.headers.get("x-api-key", "")
            if not tok or not hmac.compare_digest(tok, self.api_key):
                return error_response(AuthenticationError("invalid or missing API key"))
        return await call_next(request)


class _TokenWindow:
    """(time, tokens) charges of one key inside a window, with their running sum."""
    __slots__ = ("log", "total")

    def __init__(self):
        self.log: Deque = collections.deque()
        self.total = 0

    def expire(self, now: float, span: float) -> None:
        while self.log and now - self.log[0][0] >= span:
            self.total -= self.log.popleft()[1]


class SlidingWindowLimiter:
    """Per-key sliding windows: requests per minute (+ burst) and per day, and, when set,
    tokens per minute and per day.  The server configuration declares all four
    (crates/rusteeze-config/src/server.rs:207-244); the reference's middleware counts
    requests only.  Tokens (prompt + completion) are charged when a generation ends
    (`charge`); a key whose charges inside a window have reached its token limit is
    refused until enough of them age out, so one request may overshoot the limit, never
    a second."""

    def __init__(self, per_minute: int, burst: int = 0, per_day: Optional[int] = None,
                 tokens_per_minute: Optional[int] = None, tokens_per_day: Optional[int] = None):
        self.per_minute = per_minute
        self.burst = burst
        self.per_day = per_day
        self.tokens_per_minute = tokens_per_minute
        self.tokens_per_day = tokens_per_day
        self.hits: Dict[str, Deque[float]] = collections.defaultdict(collections.deque)
        self.day: Dict[str, Deque[float]] = collections.defaultdict(collections.deque)
        self.tok_min: Dict[str, _TokenWindow] = collections.defaultdict(_TokenWindow)
        self.tok_day: Dict[str, _TokenWindow] = collections.defaultdict(_TokenWindow)
        self._checks = 0
        self._sweep_at = 4096          # table size that triggers the next sweep (doubles as it grows)

    def _forget_idle(self, now: float) -> None:
        """Drops keys with no admission inside their windows: keyed by client address, the
        tables would otherwise grow with every client ever seen."""
        for k in [k for k, q in self.hits.items() if not q or now - q[-1] >= 60.0]:
            d = self.day.get(k)
            if d is None or not d or now - d[-1] >= 86400.0:
                self.hits.pop(k, None)
                self.day.pop(k, None)
        for tab, span in ((self.tok_min, 60.0), (self.tok_day, 86400.0)):
            for k in [k for k, w in tab.items() if not w.log or now - w.log[-1][0] >= span]:
                tab.pop(k, None)
        self._sweep_at = max(4096, 2 * len(self.hits))     # amortised O(1) per check

    def charge(self, key: str, tokens: int, now: Optional[float] = None) -> None:
        """Records the tokens a finished (or aborted) generation of `key` used."""
        if tokens <= 0 or (self.tokens_per_minute is None and self.tokens_per_day is None):
            return
        now = time.monotonic() if now is None else now
        for tab in (self.tok_min, self.tok_day):
            w = tab[key]
            w.log.append((now, int(tokens)))
            w.total += int(tokens)

    def tokens_remaining(self, key: str, now: Optional[float] = None) -> Optional[int]:
        """Tokens `key` may still use in the current minute (None: no per-minute token limit)."""
        if self.tokens_per_minute is None:
            return None
        now = time.monotonic() if now is None else now
        w = self.tok_min.get(key)
        if w is None:
            return self.tokens_per_minute
        w.expire(now, 60.0)
        return max(0, self.tokens_per_minute - w.total)

    def _token_block(self, key: str, now: float) -> Optional[float]:
        """Seconds until `key` is under its token limits again, or None when it is now."""
        for tab, limit, span in ((self.tok_min, self.tokens_per_minute, 60.0),
                                 (self.tok_day, self.tokens_per_day, 86400.0)):
            if limit is None:
                continue
            w = tab.get(key)
            if w is None:
                continue
            w.expire(now, span)
            if w.total >= limit:
                # the earliest time the window's sum drops below the limit
                need, t = w.total - limit + 1, span
                for ts, n in w.log:
                    need -= n
                    if need <= 0:
                        t = span - (now - ts)
                        break
                return t
        return None

    def check(self, key: str, now: Optional[float] = None):
        now = time.monotonic() if now is None else now
        self._checks += 1
        if self._checks % 1024 == 0 or len(self.hits) > self._sweep_at:
            self._forget_idle(now)
        q = self.hits[key]
        while q and now - q[0] >= 60.0:
            q.popleft()
        limit = self.per_minute + self.burst
        if len(q) >= limit:
            return False, limit, 0, 60.0 - (now - q[0])
        wait = self._token_block(key, now)
        if wait is not None:
            return False, limit, limit - len(q), wait
        if self.per_day is not None:
            d = self.day[key]
            while d and now - d[0] >= 86400.0:
                d.popleft()
            if len(d) >= self.per_day:
                return False, limit, 0, 86400.0 - (now - d[0])
            d.append(now)
        q.append(now)
        return True, limit, limit - len(q), 60.0 - (now - q[0])


class RateLimitMiddleware(BaseHTTPMiddleware):
    def __init__(self, app, limiter: SlidingWindowLimiter, by: str = "api_key"):
        super().__init__(app)
        self.limiter = limiter
        self.by = by

    def _key(self, request: Request) -> str:
        if self.by == "api_key":
            k = request.headers.get("x-api-key") or request.headers.get("authorization")
            if k:
                return "k:" + k
        fwd = request.headers.get("x-forwarded-for")
        if fwd:
            return "ip:" + fwd.split(",")[0].strip()
        return "ip:" + (request.client.host if request.client else "unknown")

    async def dispatch(self, request: Request, call_next):
        if request.url.path in OPEN_PATHS:
            return await call_next(request)
        key = self._key(request)
        # the handlers charge the tokens of each finished generation to this key
        request.state.rate_key = key
        ok, limit, remaining, reset = self.limiter.check(key)
        if not ok:
            resp = error_response(RateLimitError("rate limit exceeded"))
            resp.headers["Retry-After"] = str(max(1, int(math.ceil(reset))))
        else:
            resp = await call_next(request)
        resp.headers["X-RateLimit-Limit"] = str(limit)
        resp.headers["X-RateLimit-Remaining"] = str(max(0, remaining))
        resp.headers["X-RateLimit-Reset"] = str(max(0, int(reset)))
        toks = self.limiter.tokens_remaining(key)
        if toks is not None:
            resp.headers["X-RateLimit-Limit-Tokens"] = str(self.limiter.tokens_per_minute)
            resp.headers["X-RateLimit-Remaining-Tokens"] = str(toks)
        return resp


class RequestIdMiddleware(BaseHTTPMiddleware):
    def __init__(self, app, log_requests: bool = True):
        super().__init__(app)
        self.log_requests = log_requests

    async def dispatch(self, request: Request, call_next):
        rid = request.headers.get("x-request-id") or uuid.uuid4().hex
        request.state.request_id = rid
        t0 = time.perf_counter()
        resp = await call_next(request)
        resp.headers["X-Request-ID"] = rid
        if self.log_requests:
            log.info("%s %s %d %.1fms", request.method, request.url.path, resp.status_code,
                     (time.perf_counter() - t0) * 1e3, extra={"request_id": rid})
        return resp


class TimeoutMiddleware(BaseHTTPMiddleware):
    """Bounds time-to-response-headers.  Streaming bodies are bounded by the
    engine's per-request deadline instead."""

    def __init__(self, app, timeout_s: float):
        super().__init__(app)
        self.timeout_s = timeout_s

    async def dispatch(self, request: Request, call_next):
        try:
            return await asyncio.wait_for(call_next(request), timeout=self.timeout_s)
        except asyncio.TimeoutError:
            return error_response(RequestTimeoutError(f"request exceeded {self.timeout_s:.0f}s"))
