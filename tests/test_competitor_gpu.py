"""Accuracy against the reference's own GPU path on the same inputs.

The reference's ``fp8_attention`` (its Triton kernels, run from the
unmodified copy that baseline/install_reference.py places in baseline/_ref)
and this package's drop-in ``fp8_attention`` get the same bf16 q, k, v with
outlier channels; each is compared with exact float64 softmax attention of
those bf16 inputs.  This package's error must not exceed the reference's.
Skipped when baseline/_ref holds no reference copy.
"""
import math
import os
import sys

import pytest
import torch

from conftest import ROOT
from oracle import fp8_attention_ref as OA

pytestmark = pytest.mark.gpu
DEV = "cuda"
REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def _reference_fp8_attention():
    if not os.path.isfile(os.path.join(REF_DIR, "kernels", "fp8_attention.py")):
        pytest.skip("baseline/_ref holds no reference copy (baseline/install_reference.py)")
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import importlib

    return importlib.import_module("kernels.fp8_attention").fp8_attention


@pytest.mark.parametrize("S,seed", [(2048, 0), (4096, 1)])
def test_error_not_above_the_reference_kernels(S, seed, record_margin):
    ref_fp8_attention = _reference_fp8_attention()
    from minimaxh3_b200.kernels.fp8_attention import fp8_attention

    g = torch.Generator().manual_seed(seed)
    B, H, D = 1, 2, 128
    xs = []
    for _ in range(3):
        x = torch.randn(B, H, S, D, generator=g)
        x[..., int(torch.randperm(D, generator=g)[0])] *= 8.0
        xs.append(x.to(torch.bfloat16))
    q, k, v = xs
    exact = OA.sdpa_dequant_oracle(q.double(), k.double(), v.double(), 1.0 / math.sqrt(D))
    ours = fp8_attention(q.to(DEV), k.to(DEV), v.to(DEV)).float().cpu()
    theirs = ref_fp8_attention(q.to(DEV), k.to(DEV), v.to(DEV)).float().cpu()
    r_ours, r_ref = OA.compare(ours, exact), OA.compare(theirs, exact)
    record_margin(r_ours, "mh3 vs exact")
    record_margin(r_ref, "reference vs exact")
    assert r_ours["cos"] >= r_ref["cos"], (r_ours, r_ref)
    assert r_ours["max_abs"] <= r_ref["max_abs"], (r_ours, r_ref)
