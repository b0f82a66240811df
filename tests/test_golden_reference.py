"""The CPU oracle against golden vectors produced by the reference itself.

The fixtures in tests/golden/ were made by tests/golden/make_golden.py, which
runs viragadel6/minimaxh3's own Triton kernels (unmodified) under Triton's
CPU interpreter.  These tests pin the oracle that every GPU parity test uses.
"""
import glob
import json
import os

import pytest
import torch

from conftest import GOLDEN
from oracle import fp8_attention_ref as OA
from oracle import fp8_linear_ref as OL
from oracle.router_ref import cpu_sdpa_fallback

ATTN_FIXTURES = sorted(glob.glob(os.path.join(GOLDEN, "attn_*.pt")))


def _load(path):
    return torch.load(path, weights_only=False)


def test_fixtures_present():
    assert len(ATTN_FIXTURES) >= 6
    for name in ("linear_quant_lora.pt", "router_cases.pt", "cpu_fallback.pt", "conversion_policy.json"):
        assert os.path.exists(os.path.join(GOLDEN, name)), name


@pytest.mark.parametrize("path", ATTN_FIXTURES, ids=lambda p: os.path.basename(p)[5:-3])
def test_attention_quantisation_bit_exact(path):
    g = _load(path)
    D = g["q"].shape[-1]
    c = (g["scale"] if g["scale"] is not None else D ** -0.5) * OA.LOG2E
    q8, sq = OA.quantize_q(g["q"], c)
    assert torch.equal(q8.view(torch.uint8), g["q8"])
    assert torch.equal(sq, g["scale_q"])
    km = OA.k_channel_mean(g["k"])
    assert torch.equal(km, g["k_mean"])
    k8, sk = OA.quantize_k(g["k"], km)
    assert torch.equal(k8.view(torch.uint8), g["k8"])
    assert torch.equal(sk, g["scale_k"])
    v8, sv = OA.quantize_v(g["v"])
    assert torch.equal(v8.transpose(2, 3).contiguous().view(torch.uint8), g["v8t"])
    assert torch.equal(sv, g["scale_v"])


@pytest.mark.parametrize("path", ATTN_FIXTURES, ids=lambda p: os.path.basename(p)[5:-3])
def test_attention_output_matches_reference(path):
    g = _load(path)
    out = OA.fp8_attention_ref(g["q"], g["k"], g["v"], g["scale"], g["key_mask"], g["key_bias"],
                               g["repair_tau"], g["block_n"])
    if g["repair_tau"] < 0:
        # Without repair every step is exact arithmetic or correctly rounded.
        assert torch.equal(out, g["out"])
    else:
        # Repair adds exp2 (interpreter: numpy) and a bf16 dot: 1-ulp differences.
        r = OA.compare(out, g["out"])
        assert r["cos"] > 0.99999 and r["max_abs_rel"] < 1e-3, r
        assert (out != g["out"]).float().mean() < 1e-3


def test_block_n_changes_reference_output():
    """The reference's result depends on its autotuned KV tile (64 vs 128)."""
    a = _load(os.path.join(GOLDEN, "attn_base_bn64.pt"))["out"]
    b = _load(os.path.join(GOLDEN, "attn_base_bn128.pt"))["out"]
    assert not torch.equal(a, b)
    # The two autotune outcomes agree only to cos ~0.995 on this input.
    assert 0.99 < OA.compare(a, b)["cos"] < 0.9999


def test_linear_quantisation_and_lora():
    g = _load(os.path.join(GOLDEN, "linear_quant_lora.pt"))
    for nm in ("x", "w"):
        t8, ts = OL.quantize_rows(g[nm])
        assert torch.equal(t8.view(torch.uint8), g[nm + "8"])
        assert torch.equal(ts, g[nm + "_scale"])
    out = OL.apply_lora_adapters(g["x"], g["out_in"], g["adapters"])
    assert torch.equal(out, g["lora_out"])


def test_cpu_fallback_path():
    g = _load(os.path.join(GOLDEN, "cpu_fallback.pt"))
    assert torch.equal(cpu_sdpa_fallback(g["q"], g["k"], g["v"]), g["out"])


def test_conversion_policy_matches_reference():
    """minimaxh3_b200.kernels.fp8_linear converts exactly the reference's Linears."""
    import torch.nn as nn

    from minimaxh3_b200.kernels import fp8_linear as L

    with open(os.path.join(GOLDEN, "conversion_policy.json")) as f:
        cases = json.load(f)

    class Block(nn.Module):
        def __init__(self, odd=False):
            super().__init__()
            self.attn = nn.ModuleDict(dict(to_q=nn.Linear(32, 32), to_k=nn.Linear(32, 32),
                                           to_out=nn.Linear(32, 48 if not odd else 40)))
            self.norm_proj = nn.Linear(32, 32)
            self.ff = nn.Sequential(nn.Linear(32, 64), nn.GELU(), nn.Linear(64, 30))
            self.time_embed = nn.Linear(32, 32)

    class Model(nn.Module):
        def __init__(self):
            super().__init__()
            self.embed = nn.Linear(16, 32)
            self.blocks = nn.ModuleList([Block(odd=(i == 3)) for i in range(7)])
            self.heads = nn.ModuleList([nn.Linear(32, 32), nn.Linear(32, 16)])
            self.proj_out = nn.Linear(32, 16)

    class Dummy(nn.Module):
        pass

    orig = L.FP8Linear.from_linear
    L.FP8Linear.from_linear = classmethod(lambda cls, linear: Dummy())
    try:
        for case in cases:
            m = Model()
            n = L.convert_transformer_to_fp8(m, case["patterns"], case["keep"])
            converted = sorted(name for name, mod in m.named_modules() if isinstance(mod, Dummy))
            assert n == case["count"], case
            assert converted == case["converted"], case
            assert L.find_primary_block_list(m)[0] == case["primary"]
    finally:
        L.FP8Linear.from_linear = orig
