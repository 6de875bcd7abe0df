import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")

# A checkout of the reference (NanoSLG), for the CPU tests that import its own Python:
# NANOSLG_REFERENCE, else a "reference" checkout beside this repository, else None.
REFERENCE = os.environ.get("NANOSLG_REFERENCE") or (
    os.path.join(os.path.dirname(ROOT), "reference")
    if os.path.isdir(os.path.join(os.path.dirname(ROOT), "reference", "nanoslg")) else None)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built library")


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)
