import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs 2+ CUDA GPUs")
    config.addinivalue_line("markers", "slow: long-running test")
    # the host extension is tiny; build it in-tree if a fresh checkout lacks it
    try:
        import rusteeze_b200._host  # noqa: F401
    except ImportError:
        env = dict(os.environ, RUSTEEZE_SKIP_CUDA="1")
        subprocess.run([sys.executable, "setup.py", "build_ext", "--inplace"], cwd=ROOT, env=env,
                       check=True, stdout=subprocess.DEVNULL)


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        have_gpu = torch.cuda.is_available()
        ngpu = torch.cuda.device_count() if have_gpu else 0
    except Exception:
        have_gpu, ngpu = False, 0
    skip_gpu = pytest.mark.skip(reason="no CUDA GPU")
    skip_multi = pytest.mark.skip(reason="needs 2+ GPUs")
    for it in items:
        if "gpu" in it.keywords and not have_gpu:
            it.add_marker(skip_gpu)
        if "multigpu" in it.keywords and ngpu < 2:
            it.add_marker(skip_multi)
