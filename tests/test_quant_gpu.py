"""GPU parity of the quantisation kernels (through the C ABI) vs the oracle.

Bytes and scales must match the CPU restatement of the reference exactly;
the K channel mean is summed in a different order than torch's CPU mean, so
it is compared to float32 rounding and the K bytes are checked with the
kernel's own mean fed to the oracle.
"""
import pytest
import torch

from oracle import fp8_attention_ref as OA
from oracle import fp8_linear_ref as OL

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _x(seed, shape, dtype=torch.bfloat16, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*shape, generator=g) * scale
    x[..., 3] *= 8.0
    return x.to(dtype)


@pytest.mark.parametrize("B,H,Sq,Sk,D,dtype", [
    (1, 2, 300, 300, 128, torch.bfloat16),
    (2, 3, 129, 1000, 128, torch.bfloat16),
    (1, 3, 257, 257, 64, torch.float16),
    (1, 1, 1, 5, 128, torch.bfloat16),
])
def test_quantize_qkv_matches_oracle(B, H, Sq, Sk, D, dtype):
    from minimaxh3_b200 import ops

    q = _x(1, (B, H, Sq, D), dtype)
    k = _x(2, (B, H, Sk, D), dtype) + 0.7  # a channel mean worth removing
    v = _x(3, (B, H, Sk, D), dtype)
    c = OA.LOG2E / D ** 0.5
    q8, k8, v8, sq, sk, sv, km = (t.cpu() for t in ops.quantize_qkv(q.to(DEV), k.to(DEV), v.to(DEV), c))
    rq8, rsq = OA.quantize_q(q, c)
    assert torch.equal(q8.view(torch.uint8), rq8.view(torch.uint8))
    assert torch.equal(sq, rsq)
    rkm = OA.k_channel_mean(k)[:, :, 0]
    assert torch.allclose(km, rkm, rtol=0, atol=4e-6 * (1 + rkm.abs().max().item()))
    rk8, rsk = OA.quantize_k(k, km[:, :, None])
    assert torch.equal(k8.view(torch.uint8), rk8.view(torch.uint8))
    assert torch.equal(sk, rsk)
    rv8, rsv = OA.quantize_v(v)
    assert torch.equal(v8.view(torch.uint8), rv8.view(torch.uint8))
    assert torch.equal(sv, rsv)


def test_quantize_qkv_strided_inputs():
    from minimaxh3_b200 import ops

    B, S, H, D = 1, 200, 4, 128
    base = [_x(10 + i, (B, S, H, D)).to(DEV) for i in range(3)]
    q, k, v = (t.permute(0, 2, 1, 3) for t in base)  # [B,H,S,D] views
    a = ops.quantize_qkv(q, k, v, 0.1)
    b = ops.quantize_qkv(q.contiguous(), k.contiguous(), v.contiguous(), 0.1)
    for x, y in zip(a, b):
        assert torch.equal(x.view(torch.uint8) if x.dtype == torch.float8_e4m3fn else x,
                           y.view(torch.uint8) if y.dtype == torch.float8_e4m3fn else y)


@pytest.mark.parametrize("M,K,dtype", [(37, 160, torch.bfloat16), (1000, 5120, torch.bfloat16),
                                       (3, 13824, torch.float16), (1, 8, torch.bfloat16),
                                       (5, 9216, torch.bfloat16), (4, 16392, torch.bfloat16),
                                       (2, 20000, torch.float16)])
def test_quantize_rows_matches_oracle(M, K, dtype):
    """Row-in-registers kernel (K <= 16384: 1-16 chunks of 1024, odd counts rounded up) and the
    two-pass kernel (longer rows) give the oracle's bytes and scales."""
    from minimaxh3_b200 import ops

    x = _x(4, (M, K), dtype)
    x8, s = ops.quantize_rows(x.to(DEV))
    r8, rs = OL.quantize_rows(x)
    assert torch.equal(x8.cpu().view(torch.uint8), r8.view(torch.uint8))
    assert torch.equal(s.cpu(), rs)


def test_quantize_rows_golden():
    import os

    from conftest import GOLDEN
    from minimaxh3_b200 import ops

    g = torch.load(os.path.join(GOLDEN, "linear_quant_lora.pt"), weights_only=False)
    for nm in ("x", "w"):
        t8, ts = ops.quantize_rows(g[nm].to(DEV))
        assert torch.equal(t8.cpu().view(torch.uint8), g[nm + "8"])
        assert torch.equal(ts.cpu(), g[nm + "_scale"])


def _wide(seed, shape, dtype=torch.bfloat16):
    """N(0,1) scaled by 2^u with u uniform in [-24, 24): values across ~48 binades, so that the
    quotients x/s fall on every mantissa pattern, with many near rounding midpoints of e4m3/f16."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*shape, generator=g) * torch.exp2(torch.randint(-24, 24, shape, generator=g).float())
    return x.to(dtype)


def test_quotients_are_correctly_rounded_on_wide_ranges():
    """The kernels divide by a scale through a reciprocal and one correction step; the bytes must
    equal the restatement's IEEE division on data spanning many binades: e4m3 rows, the f16 V
    operand (11-bit mantissa: sensitive to any misrounded quotient) and e4m3 Q/K blocks."""
    from minimaxh3_b200 import ops

    x = _wide(21, (2048, 4096))
    x8, s = ops.quantize_rows(x.to(DEV))
    r8, rs = OL.quantize_rows(x)
    assert torch.equal(s.cpu(), rs)
    assert torch.equal(x8.cpu().view(torch.uint8), r8.view(torch.uint8))
    B, H, S, D = 1, 4, 8192, 128
    q, k, v = (_wide(22 + i, (B, H, S, D)) for i in range(3))
    q8, k8, v16, sq, sk, sv, km = (t.cpu() for t in ops.quantize_qkv(q.to(DEV), k.to(DEV), v.to(DEV), 0.1275,
                                                                     v_dtype=torch.float16))
    rsv = torch.clamp(v.float().abs().amax(dim=2), min=1e-12) / 448.0
    assert torch.equal(sv, rsv)
    rv16 = torch.clamp(v.float() / rsv[:, :, None, :], -448, 448).to(torch.float16)
    assert torch.equal(v16.view(torch.int16), rv16.view(torch.int16))
    rq8, rsq = OA.quantize_q(q, 0.1275)
    assert torch.equal(sq, rsq) and torch.equal(q8.view(torch.uint8), rq8.view(torch.uint8))
    rk8, rsk = OA.quantize_k(k, km[:, :, None])
    assert torch.equal(sk, rsk) and torch.equal(k8.view(torch.uint8), rk8.view(torch.uint8))
