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


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    """Print the parity table of the labelled cases (tests/helpers.PARITY):
    hidden-state cosine and max-abs against the oracle, draft-id rows
    compared, rows whose id differs and the largest oracle-logit gap among
    them.  Also written to $DFLASH_PARITY_JSON when that is set."""
    try:
        import helpers
    except ImportError:
        return
    if not helpers.PARITY:
        return
    tr = terminalreporter
    tr.section("draft parity against the oracle")
    tr.write_line(f"{'case':44s} {'cosine':>10s} {'max-abs':>9s} {'rows':>6s} {'differ':>6s} "
                  f"{'max gap':>9s} {'tol':>7s} {'min margin':>10s}")
    fmt = lambda v, f: (f % v) if v is not None else "-"
    for k, v in helpers.PARITY.items():
        tr.write_line(f"{k:44s} {fmt(v.get('cosine'), '%.7f'):>10s} {fmt(v.get('max_abs'), '%.3g'):>9s} "
                      f"{fmt(v.get('rows'), '%d'):>6s} {fmt(v.get('ids_differ'), '%d'):>6s} "
                      f"{fmt(v.get('max_gap'), '%.2g'):>9s} {fmt(v.get('tol'), '%.0e'):>7s} "
                      f"{fmt(v.get('min_margin'), '%.2g'):>10s}")
    out = os.environ.get("DFLASH_PARITY_JSON")
    if out:
        import json
        os.makedirs(os.path.dirname(os.path.abspath(out)), exist_ok=True)
        with open(out, "w") as f:
            json.dump(helpers.PARITY, f, indent=1)


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
