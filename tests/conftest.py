import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_cuda = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_cuda = False
    if has_cuda:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def pytest_sessionfinish(session, exitstatus):
    """Under the bounds-checked build (RO_CHECKED=1), write the failed-check
    words of the session's kernels to RO_CHECKED_REPORT (JSON)."""
    report = os.environ.get("RO_CHECKED_REPORT")
    if os.environ.get("RO_CHECKED") != "1" or not report:
        return
    import json

    from rational_optimizer_b200 import _ext
    C = _ext.ext()
    with open(report, "w") as fh:
        json.dump({"module": C.__file__, "checked": bool(C.bounds_checked), "faults": C.bounds_faults(),
                   "exitstatus": int(exitstatus)}, fh)
