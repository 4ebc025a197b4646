"""Race detection for the host runtime: the plan ring's publish/consume protocol
under ThreadSanitizer (a standalone build of csrc/host/shm_ring.h with one producer
and several reader threads on one mapping, randomised pauses).  A data race makes
the sanitizer print a report and fail the run."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "rusteeze_b200", "csrc", "host", "tests", "shm_ring_stress.cpp")


def _tsan_available() -> bool:
    if shutil.which("g++") is None:
        return False
    r = subprocess.run(["g++", "-print-file-name=libtsan.so"], capture_output=True, text=True)
    return r.returncode == 0 and os.path.isabs(r.stdout.strip())


@pytest.mark.skipif(not _tsan_available(), reason="g++ with libtsan needed")
@pytest.mark.timeout(600)
def test_plan_ring_has_no_data_race(tmp_path):
    exe = str(tmp_path / "ring_tsan")
    b = subprocess.run(["g++", "-std=c++17", "-O1", "-g", "-fsanitize=thread", "-pthread", SRC, "-o", exe, "-lrt"],
                       capture_output=True, text=True, timeout=300)
    assert b.returncode == 0, b.stderr[-3000:]
    env = dict(os.environ, TSAN_OPTIONS="halt_on_error=1 exitcode=66")
    for messages, readers in ((20000, 3), (5000, 7)):
        r = subprocess.run([exe, str(messages), str(readers)], capture_output=True, text=True, timeout=240, env=env)
        assert "ThreadSanitizer" not in r.stderr, r.stderr[-4000:]
        assert r.returncode == 0 and "RING_STRESS_OK" in r.stdout, (r.returncode, r.stderr[-2000:])
