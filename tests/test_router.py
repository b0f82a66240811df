"""routed_sdpa gating and per-key mask extraction vs the reference's decisions.

tests/golden/router_cases.pt records, for a table of calls, whether the
reference's ``routed_sdpa`` took the FP8 branch and with which keyword
arguments (``is_supported`` / ``fp8_attention`` replaced by recorders), or
what its SDPA fallback returned.  The same table is replayed through
``minimaxh3_b200.kernels.attention_router``.
"""
import contextlib
import os
import threading

import torch

from conftest import GOLDEN
from minimaxh3_b200.kernels import attention_router as A


def _replay(case, calls):
    var = case["variant"]
    cfg = dict(scope=True, enabled=True, min_seq=32, dropout_p=0.0, is_causal=False, enable_gqa=False,
               scale=None)
    cfg.update({k: v for k, v in var.items() if k in cfg})
    A.configure(enabled=cfg["enabled"], repair_tau=0.25, min_seq=cfg["min_seq"])
    scope = A.denoiser_scope() if cfg["scope"] else contextlib.nullcontext()
    q = case["q"]
    if var.get("supported") is False:
        q = q.clone()
        q._fake_supported = False
    with scope:
        try:
            out = A.routed_sdpa(q, case["k"], case["v"], attn_mask=case["mask"], dropout_p=cfg["dropout_p"],
                                is_causal=cfg["is_causal"], scale=cfg["scale"], enable_gqa=cfg["enable_gqa"])
            err = None
        except Exception as e:
            out, err = None, type(e).__name__
    return out, err


def test_router_matches_reference_decisions(monkeypatch):
    cases = torch.load(os.path.join(GOLDEN, "router_cases.pt"), weights_only=False)
    calls = []

    def fake_fp8(q, k, v, scale=None, key_mask=None, key_bias=None, repair_tau=-1.0):
        calls.append(dict(scale=scale, key_mask=key_mask, key_bias=key_bias, repair_tau=repair_tau))
        return torch.full_like(q, 7.0)

    monkeypatch.setattr(A, "is_supported", lambda q, k, v: bool(getattr(q, "_fake_supported", True)))
    monkeypatch.setattr(A, "fp8_attention", fake_fp8)
    try:
        for case in cases:
            calls.clear()
            out, err = _replay(case, calls)
            assert bool(calls) == case["routed"], case["variant"]
            assert err == case["error"], case["variant"]
            if case["routed"]:
                got, ref = calls[0], case["fp8_kwargs"]
                assert got["scale"] == ref["scale"] and got["repair_tau"] == ref["repair_tau"]
                for key in ("key_mask", "key_bias"):
                    if ref[key] is None:
                        assert got[key] is None, (case["variant"], key)
                    else:
                        assert got[key].dtype == ref[key].dtype and torch.equal(got[key], ref[key])
            elif case["out"] is not None:
                if case["variant"].get("dropout_p", 0.0) > 0.0:
                    assert out.shape == case["out"].shape  # dropout draws fresh randoms
                else:
                    assert torch.equal(out, case["out"]), case["variant"]
    finally:
        A.configure(enabled=True, repair_tau=-1.0, min_seq=4096)


def test_configure_and_scope_are_thread_local():
    A.configure(enabled=False, repair_tau=0.5, min_seq=10)
    assert (A.enabled, A.repair_tau, A.min_seq) == (False, 0.5, 10)
    A.configure(enabled=True, repair_tau=-1.0, min_seq=4096)
    seen = {}
    with A.denoiser_scope():
        with A.denoiser_scope():
            assert A._get_depth() == 2
            t = threading.Thread(target=lambda: seen.setdefault("d", A._get_depth()))
            t.start()
            t.join()
    assert seen["d"] == 0 and A._get_depth() == 0


def test_instrument_transformer_wraps_once():
    class T(torch.nn.Module):
        def forward(self, x):
            return A._get_depth()

    t = T()
    A.instrument_transformer(t)
    A.instrument_transformer(t)
    assert t(0) == 1 and A._get_depth() == 0


def test_install_patches_sdpa(monkeypatch):
    import torch.nn.functional as F

    monkeypatch.setattr(F, "scaled_dot_product_attention", F.scaled_dot_product_attention)
    monkeypatch.setattr(torch._C._nn, "scaled_dot_product_attention", torch._C._nn.scaled_dot_product_attention)
    monkeypatch.setattr(A, "_installed", False)
    A.install()
    assert F.scaled_dot_product_attention is A.routed_sdpa
    A.install()  # idempotent
    q = torch.randn(1, 2, 8, 16)
    ref = A._orig_sdpa(q, q, q)
    assert torch.equal(F.scaled_dot_product_attention(q, q, q), ref)
