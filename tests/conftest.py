"""Pytest configuration: the ``gpu`` marker and import paths.

Tests marked ``gpu`` need a CUDA device (a B200); everything else runs on the
CPU. The product package lives in the directory ``loop-sglang_b200/`` and is
imported as ``loop_sglang_b200`` through ``__graft_entry__.load_package``.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (str(ROOT), str(ROOT / "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def reference_python() -> str | None:
    """The ``python/`` directory of a Loop-SGLang checkout, for the CPU tests that drive
    this package through the reference's own plugin seams: ``$LOOPSGL_REFERENCE_PYTHON``,
    else a checkout named ``reference`` beside this repository. None when neither has
    ``loopsgl`` (those tests then skip; the GPU tests never need it)."""
    import os

    for cand in (os.environ.get("LOOPSGL_REFERENCE_PYTHON"),
                 str(ROOT.parent / "reference" / "python")):
        if cand and (Path(cand) / "loopsgl" / "__init__.py").exists():
            return cand
    return None


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_collection_modifyitems(config: pytest.Config, items: list[pytest.Item]) -> None:
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
