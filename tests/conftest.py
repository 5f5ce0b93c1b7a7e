"""Shared test configuration.

* Registers the ``gpu`` marker: tests that need a CUDA device (a B200) carry it; everything
  else runs on the CPU.
* Runs ``async def`` tests with ``asyncio.run`` (tokenserve's own suite uses pytest-asyncio,
  which is not available here).
* Puts the repository root on ``sys.path`` so ``tokenserve_b200`` and ``oracle`` import, and
  ``baseline/_ref`` (tokenserve itself) when it has been installed there.
"""

from __future__ import annotations

import asyncio
import inspect
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
# tokenserve itself, installed unmodified by baseline/install_reference.py (when present).
REF = ROOT / "baseline" / "_ref"
if (REF / "tokenserve").is_dir() and str(REF) not in sys.path:
    sys.path.append(str(REF))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs on the B200 box)")


@pytest.hookimpl(tryfirst=True)
def pytest_pyfunc_call(pyfuncitem: pytest.Function) -> bool | None:
    if inspect.iscoroutinefunction(pyfuncitem.obj):
        args = {a: pyfuncitem.funcargs[a] for a in pyfuncitem._fixtureinfo.argnames}
        asyncio.run(pyfuncitem.obj(**args))
        return True
    return None


@pytest.fixture(scope="session")
def cuda_device():  # type: ignore[no-untyped-def]
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA (run with -m 'not gpu')")
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    return torch.device("cuda", 0)
