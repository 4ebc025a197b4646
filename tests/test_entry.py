"""The driver entry point: build() compiles in-tree (incremental here) and imports
the package and both native extensions in a fresh interpreter."""
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_build_imports_extensions_in_fresh_process():
    code = "import __graft_entry__ as g; g.build(); print('BUILD_OK')"
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=1800)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "BUILD_OK" in r.stdout
