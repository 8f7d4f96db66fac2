# SPDX-License-Identifier: MIT
"""The drop-in claim, with beamgrad 2.3.0's own Python front end: its package (installed
unchanged, without CUDA operators, by oracle/Makefile ``frontend``) runs on this engine's
``_C_cuda`` and must give on CUDA tensors what its CPU kernels give on CPU tensors.

Two files run in a fresh interpreter with the ``_frontend_hook`` plugin (which points
``beamgrad._C_cuda`` at this engine's module): the reference's own CUDA test file
(python/tests/test_cuda.py: decode and final_scores with gradients over its cases, variable
steps, half precision, streams, debug synchronization, errors) and tests/_frontend_extra.py
(backtrack, search, beam_search). A subprocess keeps beamgrad's operator schemas out of this
test process, where beamgrad_b200.ops defines them.
"""

from __future__ import annotations

import os
import re
import subprocess
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
FRONTEND = ROOT / "oracle" / "_ref" / "frontend" / "beamgrad" / "_torch.py"
REF_TESTS = ROOT / "oracle" / "_ref" / "frontend_tests" / "test_cuda.py"

pytestmark = pytest.mark.gpu


def _run(target: Path, report: Path) -> tuple[int, str]:
    env = dict(os.environ, PYTHONPATH=os.pathsep.join([str(ROOT / "tests"), str(ROOT)]),
               BEAMGRAD_FRONTEND_REPORT=str(report))
    proc = subprocess.run([sys.executable, "-m", "pytest", "-p", "_frontend_hook", "-q", "-p", "no:cacheprovider",
                           "--rootdir", str(target.parent), str(target)],
                          capture_output=True, text=True, env=env, cwd=str(target.parent), timeout=900)
    return proc.returncode, proc.stdout + proc.stderr


@pytest.mark.skipif(not FRONTEND.exists(), reason="the reference Python package was not installed (oracle/Makefile)")
@pytest.mark.parametrize("target", [REF_TESTS, ROOT / "tests" / "_frontend_extra.py"], ids=["reference_test_cuda", "extra"])
def test_reference_frontend_on_this_engine(target, tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    report = tmp_path / "operators"
    rc, out = _run(target, report)
    assert rc == 0, out[-3000:]
    # beamgrad's CUDA operators were this engine's module.
    assert report.exists() and "beamgrad_b200" in report.read_text(), out[-3000:]
    passed = re.search(r"(\d+) passed", out)
    assert passed and int(passed.group(1)) > 0, out[-3000:]
