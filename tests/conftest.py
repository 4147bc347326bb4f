"""Test configuration: the ``gpu`` marker, import paths and shared fixtures.

Tests marked ``gpu`` need a B200 and the built libplm_native.so; everything else runs on CPU.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PACKAGE = ROOT / "plm-anon_b200"
for path in (str(PACKAGE), str(ROOT)):
    if path not in sys.path:
        sys.path.insert(0, path)

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100a GPU and the built libplm_native.so")


def cli_bench():
    """The CLI package plm-anon_b200/bench as (generate, harness). The name ``bench`` also belongs to the benchmark
    script at the repository root, which wins on sys.path when pytest runs from there."""
    import importlib

    cached = sys.modules.get("bench")
    if cached is None or not hasattr(cached, "__path__"):
        sys.modules.pop("bench", None)
        sys.path.insert(0, str(PACKAGE))
        try:
            importlib.import_module("bench")
        finally:
            sys.path.remove(str(PACKAGE))
    return importlib.import_module("bench.generate"), importlib.import_module("bench.harness")


@pytest.fixture(scope="session")
def ctx():
    import torch

    from plm import native

    if not torch.cuda.is_available():
        pytest.fail("gpu test collected without a GPU")
    context = native.Context()
    yield context
    context.close()
