"""Prometheus push gateway: the pusher PUTs the exposition text to the job / instance
grouping URL on its interval and once more when stopped; a gateway that is down is
counted, not raised; the configuration section loads and is validated."""
import threading
import time
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

import pytest

from rusteeze_b200.config.config import Config, PushGatewaySection
from rusteeze_b200.config.loader import ConfigLoader
from rusteeze_b200.config.validation import collect_errors
from rusteeze_b200.metrics.exporter import PushGatewayPusher, push_url
from rusteeze_b200.metrics.registry import EngineMetrics


@pytest.fixture()
def gateway():
    got = []

    class H(BaseHTTPRequestHandler):
        def do_PUT(self):  # noqa: N802
            n = int(self.headers.get("Content-Length", "0"))
            got.append((self.path, self.headers.get("Content-Type"), self.rfile.read(n)))
            self.send_response(200)
            self.send_header("Content-Length", "0")
            self.end_headers()

        def log_message(self, *a):
            pass

    srv = ThreadingHTTPServer(("127.0.0.1", 0), H)
    threading.Thread(target=srv.serve_forever, daemon=True).start()
    yield f"http://127.0.0.1:{srv.server_address[1]}", got
    srv.shutdown()
    srv.server_close()


def test_pusher_puts_the_metrics_on_its_interval_and_at_stop(gateway):
    url, got = gateway
    m = EngineMetrics(model_name="tiny")
    p = PushGatewayPusher(m, url, "serve job", instance="node-1", interval_seconds=0.05).start()
    deadline = time.time() + 10
    while len(got) < 2 and time.time() < deadline:
        time.sleep(0.02)
    n = len(got)
    p.stop()
    assert n >= 2 and len(got) >= n + 1        # at least the final push after stop
    path, ctype, body = got[-1]
    assert path == "/metrics/job/serve%20job/instance/node-1"
    assert ctype.startswith("text/plain")
    assert b"rusteeze" in body
    assert p.failures == 0 and p.pushes == len(got)


def test_a_gateway_that_is_down_is_counted_not_raised():
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()                                  # nothing listens here
    p = PushGatewayPusher(EngineMetrics(model_name="tiny"), f"http://127.0.0.1:{port}", "j")
    assert p.push() is False and p.failures == 1
    p.stop()                                   # never started: only the final push, which fails too
    assert p.failures == 2


def test_push_url_and_config(tmp_path):
    assert push_url("http://gw:9091/", "job") == "http://gw:9091/metrics/job/job"
    f = tmp_path / "c.yaml"
    f.write_text("metrics:\n  push_gateway: {url: 'http://gw:9091', job: rz, instance: a, interval_seconds: 5}\n")
    cfg = ConfigLoader(str(f)).load({})
    assert cfg.metrics.push_gateway == PushGatewaySection(url="http://gw:9091", job="rz", instance="a",
                                                          interval_seconds=5)
    bad = Config()
    bad.metrics.push_gateway = PushGatewaySection(url="gw:9091", job="", interval_seconds=0)
    errs = collect_errors(bad)
    assert sum("push_gateway" in e for e in errs) == 3
