"""Shared pytest set-up: the ``gpu`` marker and import paths.

The product package lives in the hyphenated folder ``mirror-sd_b200``; it is
imported with ``importlib.import_module("mirror-sd_b200")`` and also exposed
as ``mirror_sd_b200``.
"""
import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_pkg():
    pkg = importlib.import_module("mirror-sd_b200")
    sys.modules.setdefault("mirror_sd_b200", pkg)
    return pkg


@pytest.fixture(scope="session")
def pkg():
    return load_pkg()


@pytest.fixture(scope="session")
def golden_dir():
    return os.path.join(ROOT, "tests", "golden")
