"""Shared pytest configuration.

Tests marked ``gpu`` need a B200 (sm_100) and the built library; everything
else runs on a CPU-only machine.
"""

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT / "tests") not in sys.path:
    sys.path.insert(0, str(ROOT / "tests"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built CUDA library")


@pytest.fixture(scope="session")
def ct_checkpoint_dir(tmp_path_factory):
    """A small compressed-tensors MXFP4 checkpoint written by compressed-tensors
    itself (``tests/golden/make_ct_checkpoint.py``)."""
    import os
    import subprocess

    out = tmp_path_factory.mktemp("ct_checkpoint")
    env = dict(os.environ, TORCHDYNAMO_DISABLE="1")
    subprocess.run([sys.executable, str(ROOT / "tests" / "golden" / "make_ct_checkpoint.py"), str(out)],
                   check=True, env=env, timeout=900)
    return out
