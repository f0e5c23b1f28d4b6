"""The reference's own operator test module, run unmodified against the drop-in.

``tests/test_moe_mxfp4_soft.py`` of the reference loads the operator module by
file path from ``MXFP4_SOFT_MODULE`` (test:10-19).  Pointing that variable at
``mxfp4-gfx936_b200/moe_op_mxfp4_soft.py`` and running the module's cases that
need no GPU checks the drop-in's module-level contract with the reference's
own assertions: ``_backend`` (test:63-70), ``_require_triton_compiler`` with
``_has_compatible_triton_compiler`` patched (test:73-78) and
``_is_validated_triton_linear_shape`` (test:136-141).  The GPU cases of that
module are restated in ``tests/test_reference_contract.py``, which runs on the
GPU box where the reference checkout does not exist.

The reference checkout is read at test time only on the machine that has it;
elsewhere this test is skipped.
"""

import os
import subprocess
import sys
from pathlib import Path

import pytest

from _paths import PKG

REFERENCE_TEST = Path("/root/reference/tests/test_moe_mxfp4_soft.py")
CPU_CASES = "backend or compiler or shape_guard"


@pytest.mark.skipif(not REFERENCE_TEST.is_file(), reason="reference checkout not present on this machine")
def test_reference_module_cpu_cases_pass_on_the_drop_in(tmp_path):
    env = dict(os.environ)
    env["MXFP4_SOFT_MODULE"] = str(PKG / "moe_op_mxfp4_soft.py")
    env["PYTHONDONTWRITEBYTECODE"] = "1"
    env.pop("MXFP4_GFX936_BACKEND", None)
    cmd = [sys.executable, "-m", "pytest", str(REFERENCE_TEST), "-q", "-k", CPU_CASES,
           "-p", "no:cacheprovider", "--rootdir", str(tmp_path)]
    res = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=tmp_path, timeout=600)
    out = res.stdout + res.stderr
    assert res.returncode == 0, out
    # test:63-78 (3 cases) and test:136-141 (3 parametrised cases)
    assert "6 passed" in out, out
