import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")
# The reference's agillm41.py: $AGILLM41_REFERENCE, else a checkout named
# "reference" beside this repository. Tests that import it skip without it.
REFERENCE_PY = os.environ.get("AGILLM41_REFERENCE") or os.path.join(os.path.dirname(ROOT), "reference",
                                                                     "agillm41.py")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running case")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
