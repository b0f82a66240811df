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


@pytest.mark.parametrize("lens_q,lens_k,D,dtype", [
    ([300, 0, 77, 513], None, 128, torch.bfloat16),      # an empty sequence, tails
    ([200, 129], [640, 1], 128, torch.bfloat16),        # query and key packings differ; one key
    ([1, 255, 384], None, 64, torch.float16),
])
def test_fp8_attention_varlen(lens_q, lens_k, D, dtype, record_margin):
    """Packed sequences: per-(sequence, head) absmax/448 quantisation (V as f16 V/scale), attention
    inside each sequence; every row against exact attention of those operands."""
    from minimaxh3_b200.kernels.fp8_attention import fp8_attention_varlen

    lens_k = lens_k or lens_q
    H = 4
    cu_q = torch.tensor([0] + list(torch.tensor(lens_q).cumsum(0)), dtype=torch.int32)
    cu_k = torch.tensor([0] + list(torch.tensor(lens_k).cumsum(0)), dtype=torch.int32)
    g = torch.Generator().manual_seed(sum(lens_q) + D)

    def packed(T):
        x = torch.randn(T, H, D, generator=g)
        x[..., 9] *= 8.0
        return x.to(dtype)

    q, k, v = packed(int(cu_q[-1])), packed(int(cu_k[-1])), packed(int(cu_k[-1]))
    out = fp8_attention_varlen(q.to(DEV), k.to(DEV), v.to(DEV), cu_q.to(DEV), cu_k.to(DEV), max(lens_q))
    assert out.shape == q.shape and out.dtype == dtype
    out = out.float().cpu()
    ls2 = OA.LOG2E / math.sqrt(D)

    def operand(x, dt):
        s = (torch.clamp(x.float().abs().amax(dim=(0, 2)), min=1e-12).double() / 448.0).float()     # [H]
        y = x.float() / s[None, :, None]
        y = (torch.clamp(y, -448, 448) if dt == torch.float8_e4m3fn else y).to(dt)
        return (y.double() * s.double()[None, :, None]).permute(1, 0, 2)[None]  # [1, H, L, D]

    for z in range(len(lens_q)):
        (a, b), (c, d) = (int(cu_q[z]), int(cu_q[z + 1])), (int(cu_k[z]), int(cu_k[z + 1]))
        if b == a:
            continue
        ref = OA.sdpa_dequant_oracle(operand(q[a:b], torch.float8_e4m3fn), operand(k[c:d], torch.float8_e4m3fn),
                                     operand(v[c:d], torch.float16), ls2, base2=True)[0].permute(1, 0, 2)
        r = OA.compare(out[a:b], ref)
        record_margin(r, f"varlen seq{z}")
        assert OA.within_tolerance(r), (z, r)


def test_fp8_attention_varlen_rejects_bad_arguments():
    from minimaxh3_b200.kernels.fp8_attention import fp8_attention_varlen

    x = torch.zeros(64, 2, 128, dtype=torch.bfloat16, device=DEV)
    cu = torch.tensor([0, 64], dtype=torch.int32, device=DEV)
    with pytest.raises(ValueError):
        fp8_attention_varlen(x[None], x, x, cu, cu, 64)                 # not packed
    with pytest.raises(ValueError):
        fp8_attention_varlen(x, x, x, cu.long(), cu, 64)                # int32 offsets
    with pytest.raises(ValueError):
        fp8_attention_varlen(x, x, x, cu, torch.tensor([0, 32, 64], dtype=torch.int32, device=DEV), 64)
    with pytest.raises(ValueError):
        fp8_attention_varlen(x, x, x, cu, cu, 0)
