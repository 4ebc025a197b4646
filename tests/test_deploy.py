"""Deployment artefacts (Dockerfile, docker-compose.yml, prometheus.yml, CI workflow)
agree with the code they deploy: the commands, endpoints, ports and environment
variables they name exist."""
import os
import re

import yaml

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _read(p):
    with open(os.path.join(ROOT, p)) as f:
        return f.read()


def test_compose_services_and_health_endpoints():
    from rusteeze_b200.api.server import create_app  # noqa: F401 -- the app the image serves
    d = yaml.safe_load(_read("docker-compose.yml"))
    srv = d["services"]["rusteeze"]
    assert srv["command"][0] == "serve" and srv["ipc"] == "host"
    assert "8000:8000" in srv["ports"]
    hc = " ".join(srv["healthcheck"]["test"])
    paths = re.findall(r"localhost:\d+(/[\w/]+)", hc)
    server_src = _read("rusteeze_b200/api/server.py")
    for p in paths:
        assert f'"{p}"' in server_src, p
    for svc in ("prometheus", "grafana", "dcgm-exporter"):
        assert d["services"][svc]["profiles"] == ["monitoring"]
    env = dict(e.split("=", 1) for e in srv["environment"])
    from rusteeze_b200.config.loader import ENV_OVERRIDES
    for k in env:
        if k.startswith("RUSTEEZE_") and k != "RUSTEEZE_CONFIG":
            assert k[len("RUSTEEZE_"):] in ENV_OVERRIDES, k


def test_prometheus_scrapes_the_metrics_path():
    d = yaml.safe_load(_read("prometheus.yml"))
    jobs = {j["job_name"]: j for j in d["scrape_configs"]}
    from rusteeze_b200.config.config import Config
    assert jobs["rusteeze"]["metrics_path"] == Config().metrics.path
    assert jobs["rusteeze"]["static_configs"][0]["targets"] == ["rusteeze:8000"]


def test_dockerfile_entrypoint_and_build():
    s = _read("Dockerfile")
    assert 'ENTRYPOINT ["python", "-m", "rusteeze_b200"]' in s
    assert os.path.exists(os.path.join(ROOT, "rusteeze_b200", "__main__.py"))
    assert "setup.py build_ext --inplace" in s
    from rusteeze_b200.cli.main import build_parser
    build_parser().parse_args(["serve"])                     # the image's default command parses
    for line in _read("requirements.txt").splitlines():
        line = line.split("#")[0].strip()
        if line:
            assert re.match(r"^[A-Za-z0-9_.-]+(>=|==)[0-9.]+$", line), line


def test_ci_workflow_runs_the_cpu_suite_and_the_build():
    d = yaml.safe_load(_read(".github/workflows/ci.yml"))
    steps = [s.get("run", "") for s in d["jobs"]["cpu-tests"]["steps"]]
    assert any("e.build()" in r for r in steps)
    assert any('-m "not gpu"' in r for r in steps)
