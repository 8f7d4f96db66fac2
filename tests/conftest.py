# SPDX-License-Identifier: MIT
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session", autouse=True)
def _built_oracle():
    """The CPU checkers are compiled before any test uses them (no-op when up to date)."""
    from oracle import oracle

    try:
        oracle.build()
    except Exception as exc:  # pragma: no cover - missing toolchain on a GPU box: prebuilt files are used
        if not oracle.ORACLE_LIB.exists():
            raise RuntimeError(f"oracle library unavailable: {exc}") from exc
