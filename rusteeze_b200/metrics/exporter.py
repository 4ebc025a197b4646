"""Standalone Prometheus exporter on its own port (`--metrics-port`, default
9090 in the reference: crates/rusteeze-metrics/src/prometheus.rs:34-155,
which hand-rolls an HTTP server with /metrics and /health)."""
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
