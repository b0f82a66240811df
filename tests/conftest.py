import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")

# Tolerance stated by the north star, against an fp32 SDPA oracle on the
# dequantised inputs: cosine >= 0.9995 and max-abs error <= 2e-2, taken
# relative to max(1, max|oracle|) (outlier channels make an absolute 2e-2
# unreachable even for bf16 rounding of the output alone); see
# oracle.fp8_attention_ref.within_tolerance.
COS_MIN = 0.9995
MAXABS = 2e-2


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100) device")
    config.addinivalue_line("markers", "slow: long-running")


def _has_gpu():
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
