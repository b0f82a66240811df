"""The drop-in modules on the GPU: fp8_attention, routed_sdpa, torch.compile."""
import math
import os

import pytest
import torch

from conftest import GOLDEN
from oracle import fp8_attention_ref as OA

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _golden(name):
    return torch.load(os.path.join(GOLDEN, f"attn_{name}.pt"), weights_only=False)


@pytest.mark.parametrize("name", ["base_bn128", "mask_cross", "bias_cross", "d64_fp16", "repair_bn128"])
def test_fp8_attention_on_reference_golden_inputs(name, record_margin):
    """Same inputs the reference's own kernels were run on (tests/golden).

    The oracle is exact softmax attention on the operands the kernel really
    multiplies: the reference's e4m3 Q and K bytes with their block scales
    (this package's quantisation reproduces them bit for bit, see
    test_quant_gpu) and, for the default f16 PV product, V as f16(v / scale_v)
    times scale_v.  The north-star tolerance is asserted in its relative
    reading (max-abs <= 2e-2 x max|oracle|), and the kernel must be at least
    as accurate as the reference kernel's own output on the same inputs.
    """
    from minimaxh3_b200.kernels.fp8_attention import fp8_attention

    g = _golden(name)
    q, k, v = (g[t].to(DEV) for t in ("q", "k", "v"))
    km = g["key_mask"].to(DEV) if g["key_mask"] is not None else None
    kb = g["key_bias"].to(DEV) if g["key_bias"] is not None else None
    out = fp8_attention(q, k, v, scale=g["scale"], key_mask=km, key_bias=kb, repair_tau=g["repair_tau"])
    assert out.dtype == q.dtype and out.shape == q.shape
    out = out.float().cpu()
    q8 = g["q8"].view(torch.float8_e4m3fn)
    k8 = g["k8"].view(torch.float8_e4m3fn)
    sv = g["scale_v"].float()
    v16 = (g["v"].float() / sv[:, :, None, :]).to(torch.float16)  # the f16 PV operand
    ref = OA.sdpa_dequant_oracle(OA.dequant_blocks(q8, g["scale_q"]), OA.dequant_blocks(k8, g["scale_k"]),
                                 v16.double() * sv.double()[:, :, None, :], 1.0,
                                 key_mask=g["key_mask"], key_bias=g["key_bias"], base2=True)
    r = OA.compare(out, ref)
    r_ref = OA.compare(g["out"].float(), ref)  # the reference kernel's own error against the same oracle
    record_margin(r)
    assert OA.within_tolerance(r), (r, r_ref)
    assert r["cos"] >= r_ref["cos"] and r["max_abs"] <= r_ref["max_abs"], (r, r_ref)


def test_routed_sdpa_takes_fp8_branch():
    from minimaxh3_b200.kernels import attention_router as A

    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(1, 2, 4096, 128, generator=g).to(torch.bfloat16).to(DEV) for _ in range(3))
    A.configure(enabled=True, repair_tau=-1.0, min_seq=4096)
    with A.denoiser_scope():
        out = A.routed_sdpa(q, k, v)
    ref = A._orig_sdpa(q.float(), k.float(), v.float())
    r = OA.compare(out.float().cpu(), ref.cpu())
    # Against the unquantised inputs the e4m3 input rounding is included.
    assert r["cos"] > 0.995, r
    assert not torch.equal(out, A._orig_sdpa(q, k, v))
    # Outside the scope the original SDPA runs.
    out2 = A.routed_sdpa(q, k, v)
    assert torch.equal(out2, A._orig_sdpa(q, k, v))


def test_fp8_attention_is_compile_friendly():
    from minimaxh3_b200.kernels.fp8_attention import fp8_attention

    def block(q, k, v):
        return fp8_attention(q * 1.0, k, v).float().sum(dim=-1)

    g = torch.Generator().manual_seed(1)
    q, k, v = (torch.randn(1, 2, 512, 128, generator=g).to(torch.bfloat16).to(DEV) for _ in range(3))
    import torch._dynamo as dynamo

    dynamo.reset()
    explanation = dynamo.explain(block)(q, k, v)
    assert explanation.graph_break_count == 0
    compiled = torch.compile(block, backend="eager", fullgraph=True)
    assert torch.allclose(compiled(q, k, v), block(q, k, v))


def test_is_supported_rules():
    from minimaxh3_b200.kernels.fp8_attention import is_supported

    t = torch.zeros(1, 2, 8, 128, dtype=torch.bfloat16, device=DEV)
    assert is_supported(t, t, t)
    assert not is_supported(t.float(), t.float(), t.float())
    assert not is_supported(t.cpu(), t.cpu(), t.cpu())
    assert not is_supported(t[..., :96], t[..., :96], t[..., :96])
    assert not is_supported(t, t[:, :, :0], t[:, :, :0])
    with pytest.raises(ValueError):
        from minimaxh3_b200.kernels.fp8_attention import fp8_attention

        fp8_attention(t.float(), t, t)
