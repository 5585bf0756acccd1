"""Shared pytest configuration: the `gpu` marker and the repository root on sys.path."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def pytest_terminal_summary(terminalreporter):
    """Both parity metrics of every comparison made through helpers.rel_err: the asserted
    max-normalised error and the element-wise max relative error (floor 1e-2 of max|ref|),
    worst comparison per test.  SP_PARITY_REPORT=<path> also writes them as JSON lines."""
    try:
        from helpers import PARITY_LOG
    except Exception:  # pragma: no cover
        return
    if not PARITY_LOG:
        return
    worst = {}
    for test, e, m in PARITY_LOG:
        a, b = worst.get(test, (0.0, 0.0))
        worst[test] = (max(a, e), max(b, m))
    tr = terminalreporter
    tr.write_sep("-", "parity: max-normalised error | element-wise max relative error")
    for test, (e, m) in sorted(worst.items()):
        tr.write_line(f"{e:10.3e} {m:10.3e}  {test}")
    path = os.environ.get("SP_PARITY_REPORT")
    if path:
        import json
        with open(path, "w") as fh:
            for test, (e, m) in sorted(worst.items()):
                fh.write(json.dumps({"test": test, "rel_err": e, "max_rel_err": m}) + "\n")
