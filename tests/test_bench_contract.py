"""The benchmark script's contract without a GPU: the reference arm's `unavailable`
line, the clock-sample summary, the synthetic workload, and every arm of the harness
(single engine, data-parallel replicas, one tensor-parallel engine with speculative
decoding over a shared prefix) run on CPU with a tiny model (`--device cpu`)."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_reference_arm_prints_unavailable_and_exits_zero():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--gpus", "2", "--steps", "3",
                        "--warmup", "3"], cwd=ROOT, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unavailable"] and d["n_gpus"] == 2


def test_clock_summary_median_and_reasons():
    lines = [
        "1800, 1965, 900.1, 0x4, Not Active, Not Active, Not Active, Active",
        "1850, 1965, 950.0, 0x4, Not Active, Not Active, Not Active, Active",
        "1900, 1965, 990.0, 0x0, Not Active, Not Active, Not Active, Not Active",
        "garbage line",
        "[N/A], 1965, 1.0, 0x0, Not Active, Not Active, Not Active, Not Active",
    ]
    c = bench.summarize_clocks(lines)
    assert c["sm_mhz"] == 1850 and c["sm_max_mhz"] == 1965 and c["samples"] == 3
    assert c["reasons"] == ["sw_power_cap"]
    hot = bench.summarize_clocks(["1200, 1965, 700, 0x40, Not Active, Active, Not Active, Not Active"])
    assert hot["reasons"] == ["hw_thermal_slowdown"]


def test_workload_shape_and_determinism():
    p1, o1, a1 = bench.build_workload(64, 1000, 128256, 200.0)
    p2, o2, a2 = bench.build_workload(64, 1000, 128256, 200.0)
    assert p1 == p2 and o1 == o2 and a1 == a2               # every data-parallel rank serves this stream
    assert all(128 <= len(p) <= 2048 for p in p1) and all(64 <= o <= 512 for o in o1)
    assert all(0 <= t < 128256 for p in p1 for t in p)
    assert all(b >= a for a, b in zip(a1, a1[1:]))           # Poisson arrivals are increasing


_TINY = ["--device", "cpu", "--model", "tiny-llama", "--dtype", "bf16", "--max-seqs", "4",
         "--max-batched-tokens", "256"]
_POISSON = _TINY + ["--requests", "12", "--steps", "3", "--warmup", "3", "--prompt-len", "16,48",
                    "--output-len", "8,24", "--e2e-requests", "4"]


def _json_lines(out):
    return [json.loads(ln) for ln in out.splitlines() if ln.startswith("{")]


def _torchrun(n, port, args):
    return [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", str(n),
            "--master-addr", "127.0.0.1", "--master-port", str(port), "bench.py", "--gpus", str(n)] + args


def _free_port():
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_bench_line_contract_on_cpu_harness():
    """One Poisson run of the harness on CPU: the JSON line carries every contract key."""
    r = subprocess.run([sys.executable, "bench.py"] + _POISSON, cwd=ROOT, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    (d,) = _json_lines(r.stdout)
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "dtype", "data", "config", "clocks", "gpu_launches", "e2e"):
        assert k in d, k
    assert d["n_gpus"] == 1 and d["steps"] == 3 and d["warmup"] == 3 and d["value"] > 0
    assert d["e2e"]["value"] > 0 and d["e2e"]["h2d_bytes_per_step"] > 0
    assert d["config"]["seq_len"] == "prompt U[16,48] + output U[8,24]"


@pytest.mark.timeout(900)
def test_bench_data_parallel_and_tensor_parallel_runs_on_gloo():
    """The multi-rank arms of the harness under torchrun with gloo ranks: data-parallel
    replicas (MAX / SUM over ranks), and one tensor-parallel engine with speculative
    decoding over a shared prefix (rank 0 drives, the worker follows the plan ring)."""
    r = subprocess.run(_torchrun(2, _free_port(), _POISSON + ["--parallel", "dp"]), cwd=ROOT, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    (d,) = _json_lines(r.stdout)
    assert d["n_gpus"] == 2 and d["config"]["parallelism"] == "dp2" and d["e2e"]["requests"] == 8
    # the default at N > 1: one tensor-parallel engine, weak scaling (N x requests and running sequences)
    r = subprocess.run(_torchrun(2, _free_port(), _POISSON + ["--comm", "nccl"]), cwd=ROOT, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    (d,) = _json_lines(r.stdout)
    assert d["n_gpus"] == 2 and d["config"]["parallelism"].startswith("tp2") and d["scaling"] == "weak"
    assert d["config"]["global_batch"] == 8 and d["e2e"]["requests"] == 8 and d["value"] > 0
    tp = _TINY + ["--parallel", "tp", "--comm", "nccl", "--workload", "shared-prefix", "--shared-prefix", "48",
                  "--draft", "self", "--spec-k", "3", "--batches", "4", "--static-prompt", "24",
                  "--static-output", "6"]
    r = subprocess.run(_torchrun(2, _free_port(), tp), cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    (d,) = _json_lines(r.stdout)
    assert d["n_gpus"] == 2 and d["config"]["parallelism"].startswith("tp2")
    assert d["speculative"]["acceptance"] == 1.0 and d["speculative"]["rounds"] > 0


@pytest.mark.timeout(900)
def test_bench_moe_static_batches_one_process_and_tp2_on_gloo():
    """The shape of the Mixtral configuration on the CPU harness: static batches through a
    MoE model, in one process and as one TP2 engine with the experts split over the ranks."""
    moe = ["--device", "cpu", "--model", "tiny-mixtral", "--dtype", "bf16", "--max-seqs", "4",
           "--max-batched-tokens", "256", "--workload", "static", "--batches", "4", "--static-prompt", "24",
           "--static-output", "6"]
    r = subprocess.run([sys.executable, "bench.py"] + moe, cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    lines = _json_lines(r.stdout)
    assert lines and all(d["value"] > 0 for d in lines)
    r = subprocess.run(_torchrun(2, _free_port(), moe + ["--parallel", "tp", "--comm", "nccl"]), cwd=ROOT,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    lines = _json_lines(r.stdout)
    assert lines and lines[-1]["n_gpus"] == 2 and lines[-1]["value"] > 0


@pytest.mark.timeout(900)
def test_bench_e2e_over_http_serves_the_whole_stream():
    """`--e2e-http`: the end-to-end stream goes through the OpenAI-compatible server as
    streamed /v1/completions calls; every request completes and the line says so."""
    r = subprocess.run([sys.executable, "bench.py"] + _POISSON + ["--e2e-http"], cwd=ROOT, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    d = _json_lines(r.stdout)[-1]
    e = d["e2e"]
    assert e["via"] == "http" and e["value"] > 0 and e["completed"] == e["requests"] == 4, e
    assert e["h2d_bytes_per_step"] > 0 and e["d2h_bytes_per_step"] >= 0
