"""Standalone Prometheus exporter on its own port (`--metrics-port`, default
9090 in the reference: crates/rusteeze-metrics/src/prometheus.rs:34-155,
which hand-rolls an HTTP server with /metrics and /health), and pushes to a
Prometheus push gateway (`metrics.push_gateway`)."""
from __future__ import annotations

import threading
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

from rusteeze_b200.metrics.registry import CONTENT_TYPE


def start_exporter(metrics, port: int, host: str = "0.0.0.0") -> ThreadingHTTPServer:
    class H(BaseHTTPRequestHandler):
        def do_GET(self):  # noqa: N802
            if self.path.startswith("/metrics"):
                body, ctype, code = metrics.export(), CONTENT_TYPE, 200
            elif self.path.startswith("/health"):
                body, ctype, code = b"OK", "text/plain", 200
            else:
                body, ctype, code = b"not found", "text/plain", 404
            self.send_response(code)
            self.send_header("Content-Type", ctype)
            self.send_header("Content-Length", str(len(body)))
            self.end_headers()
            self.wfile.write(body)

        def log_message(self, *a):
            pass

    srv = ThreadingHTTPServer((host, port), H)
    threading.Thread(target=srv.serve_forever, name="metrics-exporter", daemon=True).start()
    return srv


def push_url(url: str, job: str, instance=None) -> str:
    """The Prometheus push gateway's grouping URL for a job (and instance)."""
    from urllib.parse import quote
    u = f"{url.rstrip('/')}/metrics/job/{quote(job, safe='')}"
    if instance:
        u += f"/instance/{quote(instance, safe='')}"
    return u


def push_once(metrics, url: str, job: str, instance=None, timeout_s: float = 10.0) -> None:
    """PUTs the current exposition text to the push gateway (replacing the group's metrics).
    The reference builds the same URL and only logs it
    (crates/rusteeze-metrics/src/prometheus.rs:157-191)."""
    import urllib.request
    req = urllib.request.Request(push_url(url, job, instance), data=metrics.export(), method="PUT",
                                 headers={"Content-Type": CONTENT_TYPE})
    with urllib.request.urlopen(req, timeout=timeout_s) as r:
        if r.status >= 300:
            raise OSError(f"push gateway answered {r.status}")


class PushGatewayPusher:
    """Pushes the metrics every `interval_seconds` from a daemon thread, and once more when
    stopped (so the last values of a short-lived job reach the gateway).  A failed push is
    counted and logged; it never stops the server."""

    def __init__(self, metrics, url: str, job: str, instance=None, interval_seconds: float = 15.0):
        self.metrics, self.url, self.job, self.instance = metrics, url, job, instance
        self.interval = max(0.05, float(interval_seconds))
        self.pushes = 0
        self.failures = 0
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, name="metrics-push", daemon=True)

    def start(self) -> "PushGatewayPusher":
        self._thread.start()
        return self

    def push(self) -> bool:
        try:
            push_once(self.metrics, self.url, self.job, self.instance)
            self.pushes += 1
            return True
        except Exception as e:  # noqa: BLE001 -- network errors of any kind
            self.failures += 1
            import logging
            logging.getLogger("rusteeze.metrics").warning("metrics push to %s failed: %s", self.url, e)
            return False

    def _run(self) -> None:
        while not self._stop.wait(self.interval):
            self.push()

    def stop(self, final_push: bool = True) -> None:
        self._stop.set()
        if self._thread.is_alive():
            self._thread.join(timeout=self.interval + 15.0)
        if final_push:
            self.push()
