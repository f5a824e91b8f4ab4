"""Shared pytest setup: the `gpu` marker, package import, oracle and device fixtures."""
from __future__ import annotations

import importlib
import json
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))
if str(REPO / "tests") not in sys.path:
    sys.path.insert(0, str(REPO / "tests"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU and the built CUDA library")


def load_pkg():
    """The product package (directory name is not an identifier)."""
    return importlib.import_module("llmtoy-zig_b200")


@pytest.fixture(scope="session")
def pkg():
    return load_pkg()


@pytest.fixture(scope="session")
def golden():
    return json.loads((REPO / "tests" / "golden" / "golden.json").read_text())


@pytest.fixture(scope="session")
def oracle():
    import oracle_lib
    oracle_lib.lib()
    return oracle_lib


@pytest.fixture(scope="session")
def pool(oracle):
    import os
    p = oracle.Pool(min(8, os.cpu_count() or 1))
    yield p
    p.close()


@pytest.fixture(scope="session")
def ctx(pkg):
    """A device context on cuda:0.  GPU tests fail (not skip) if the library or
    device is missing: there is no CPU fallback to hide behind."""
    import torch
    assert torch.cuda.is_available(), "gpu test needs a CUDA device"
    torch.cuda.init()
    c = pkg.Context(0)
    c.set_stream(None)  # own stream: inputs are copied synchronously, results read after a device sync
    yield c
    c.close()
