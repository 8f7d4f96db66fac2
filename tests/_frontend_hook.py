# SPDX-License-Identifier: MIT
"""Pytest plugin (``-p _frontend_hook``): beamgrad 2.3.0's own Python package, unchanged,
on this repository's CUDA operator module.

beamgrad's ``_torch.py`` imports ``beamgrad._C`` (its operator schemas and CPU kernels) and
then, if ``importlib.util.find_spec("beamgrad._C_cuda")`` finds one, ``beamgrad._C_cuda``
(the CUDA kernels of the same operators). The package here was installed without CUDA
operators (oracle/Makefile ``frontend``); this plugin puts it on ``sys.path`` and answers
that find_spec with ``beamgrad_b200/_C_cuda*.so``, so every CUDA tensor beamgrad's API
sees runs on this engine. Used only by tests/test_reference_frontend.py, in a subprocess.
"""

from __future__ import annotations

import importlib.abc
import importlib.machinery
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
FRONTEND = ROOT / "oracle" / "_ref" / "frontend"
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(FRONTEND))

from beamgrad_b200 import _abi  # noqa: E402
from beamgrad_b200 import build as _build  # noqa: E402

_abi.load()  # the engine library, by its soname, before the operator module links to it
_SO = _build.torch_ext_path()


class _EngineOperators(importlib.abc.MetaPathFinder):
    """Resolves ``beamgrad._C_cuda`` to this engine's operator module."""

    def find_spec(self, name, path=None, target=None):
        if name != "beamgrad._C_cuda":
            return None
        loader = importlib.machinery.ExtensionFileLoader(name, str(_SO))
        return importlib.machinery.ModuleSpec(name, loader, origin=str(_SO))


sys.meta_path.insert(0, _EngineOperators())


def pytest_sessionfinish(session, exitstatus):
    """Records which module served beamgrad's CUDA operators ($BEAMGRAD_FRONTEND_REPORT)."""
    report = os.environ.get("BEAMGRAD_FRONTEND_REPORT")
    mod = sys.modules.get("beamgrad._C_cuda")
    if report:
        Path(report).write_text(str(getattr(mod, "__file__", None)))
