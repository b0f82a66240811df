"""GPU parity of the scaled GEMM and the drop-in FP8Linear (through the C ABI).

The e4m3 GEMM must reproduce ``torch._scaled_mm``'s row-wise semantics as
restated in oracle/fp8_linear_ref.py: the e4m3 products are exact and summed
in fp32, so results may differ from the float64-summed restatement by the
final bf16 rounding only.  The fused LoRA epilogue is checked against the
float64 value of ``main + sum_i scale_i (x A_i^T) B_i^T``.
"""
import pytest
import torch
import torch.nn as nn

from oracle import fp8_attention_ref as OA
from oracle import fp8_linear_ref as OL

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rand(seed, *shape, scale=1.0, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dtype)


def _bf16_close(got, ref):
    """At most one bf16 rounding step apart (fp32 sum order differs)."""
    got, ref = got.float(), ref.float()
    tol = ref.abs() * 2.0 ** -7 + 1e-6
    bad = (got - ref).abs() > tol
    return int(bad.sum()), float((got - ref).abs().max())


@pytest.mark.parametrize("M,N,K", [(37, 48, 160), (300, 512, 1024), (129, 96, 256), (2181, 2560, 384),
                                   (1000, 5120, 5120)])
def test_e4m3_gemm_matches_scaled_mm_semantics(M, N, K):
    from minimaxh3_b200 import ops

    x = _rand(1, M, K)
    w = _rand(2, N, K, scale=0.02)
    bias = _rand(3, N, scale=0.01)
    x8, sa = OL.quantize_rows(x)
    w8, sb = OL.quantize_rows(w)
    ref = OL.scaled_mm_rowwise(x8, w8, sa, sb.reshape(1, -1), bias)
    out = ops.scaled_gemm(x8.to(DEV), w8.to(DEV), row_scale=sa.to(DEV), col_scale=sb.to(DEV),
                          bias=bias.to(DEV)).cpu()
    nbad, err = _bf16_close(out, ref)
    assert nbad == 0, (nbad, err)


@pytest.mark.parametrize("M,N,K,R,bf16", [(1000, 1544, 640, 32, False), (4097, 5120, 512, 0, False),
                                          (257, 264, 384, 16, False), (700, 768, 256, 0, True)])
def test_cta_pair_kernel_matches_single_cta_kernel(monkeypatch, M, N, K, R, bf16):
    """The 256x256 CTA-pair kernel and the 128x256 single-CTA kernel (MH3_GEMM_CTA_PAIR=0) agree to
    one bf16 rounding (the same fp32 products per K step); row and column tails, LoRA K-steps and
    bf16 operands included.  Both also meet the float64 restatement."""
    from minimaxh3_b200 import ops

    dt = torch.bfloat16 if bf16 else torch.float8_e4m3fn
    x = _rand(11, M, K)
    w = _rand(12, N, K, scale=0.02)
    if bf16:
        a, b, sa, sb = x, w, torch.rand(M) + 0.5, torch.rand(N) + 0.5
    else:
        a, sa = OL.quantize_rows(x)
        b, sb = OL.quantize_rows(w)
    bias = _rand(13, N, scale=0.01)
    a2 = _rand(14, M, R, scale=0.1) if R else None
    b2 = _rand(15, N, R, scale=0.1) if R else None
    args = dict(row_scale=sa.reshape(-1).to(DEV), col_scale=sb.reshape(-1).to(DEV), bias=bias.to(DEV),
                a2=None if a2 is None else a2.to(DEV), b2=None if b2 is None else b2.to(DEV))
    pair = ops.scaled_gemm(a.to(dt).to(DEV), b.to(dt).to(DEV), **args).cpu()
    monkeypatch.setenv("MH3_GEMM_CTA_PAIR", "0")
    single = ops.scaled_gemm(a.to(dt).to(DEV), b.to(dt).to(DEV), **args).cpu()
    nbad, err = _bf16_close(pair, single)
    assert nbad == 0, (nbad, err)
    acc = a.to(dt).double() @ b.to(dt).double().t()
    if R:
        acc = acc + a2.double() @ b2.double().t()
    ref = acc * sa.reshape(-1, 1).double() * sb.reshape(1, -1).double() + bias.double()
    r = OA.compare(pair.float(), ref)
    assert r["cos"] > 0.99999 and r["max_abs"] <= 1e-2 * r["ref_absmax"], r


def test_bf16_gemm_with_inverse_row_scale():
    from minimaxh3_b200 import ops

    M, N, K = 333, 64, 640
    x = _rand(4, M, K)
    A = _rand(5, N, K, scale=0.05)
    rs = torch.rand(M) + 0.5
    out = ops.scaled_gemm(x.to(DEV), A.to(DEV), row_scale=rs.to(DEV), row_scale_inv=True).float().cpu()
    ref = (x.double() @ A.double().t()) / rs.double()[:, None]
    r = OA.compare(out, ref)
    assert r["cos"] > 0.99999 and r["max_abs"] <= 1e-2 * r["ref_absmax"], r


def _linear(seed, K, N, bias=True):
    lin = nn.Linear(K, N, bias=bias)
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(N, K, generator=g) * 0.02)
        if bias:
            lin.bias.copy_(torch.randn(N, generator=g) * 0.01)
    return lin.to(torch.bfloat16)


@pytest.mark.parametrize("M,K,N,n_adapters", [(37, 160, 48, 0), (300, 1024, 512, 1), (1000, 5120, 1536, 2)])
def test_fp8_linear_forward(M, K, N, n_adapters):
    from minimaxh3_b200.kernels.fp8_linear import FP8Linear

    lin = _linear(7, K, N)
    w_ref = lin.weight.detach().clone()
    b_ref = lin.bias.detach().clone()
    mod = FP8Linear.from_linear(lin.to(DEV))
    adapters = []
    for i in range(n_adapters):
        r = 32 if i == 0 else 8
        A = _rand(20 + i, r, K, scale=0.01)
        B = _rand(30 + i, N, r, scale=0.01)
        adapters.append((A, B, 1.0 if i == 0 else 0.5))
    mod.adapters = [(A.to(DEV), B.to(DEV), s) for A, B, s in adapters]
    x = _rand(8, 2, M // 2 if M % 2 == 0 else M, K) if M % 2 == 0 else _rand(8, M, K)
    out = mod(x.to(DEV)).cpu()
    assert out.shape == (*x.shape[:-1], N) and out.dtype == x.dtype
    # quantised weights identical to the reference's quantize_rows
    w8_ref, ws_ref = OL.quantize_rows(w_ref)
    assert torch.equal(mod.w8.cpu().view(torch.uint8), w8_ref.view(torch.uint8))
    assert torch.equal(mod.w_scale.cpu(), ws_ref.view(1, -1))
    exact = OL.fp8_linear_fused_oracle(x, w8_ref, ws_ref.view(1, -1), b_ref, adapters).reshape(out.shape)
    r = OA.compare(out.float(), exact)
    assert r["cos"] > 0.99999 and r["max_abs"] <= 1e-2 * max(r["ref_absmax"], 1e-3), r
    # and the reference restatement (bf16 rounding after every step) agrees
    ref = OL.fp8_linear_forward(x, w8_ref, ws_ref.view(1, -1), b_ref, adapters, N)
    r2 = OA.compare(out.float(), ref.float())
    assert r2["cos"] > 0.9999, r2


@pytest.mark.parametrize("M,K,N,n_adapters", [(37, 160, 48, 1), (300, 1024, 512, 2), (1000, 5120, 1536, 1),
                                              (129, 256, 264, 0)])
def test_unquantised_linear_lora_fused(M, K, N, n_adapters):
    """runtime/lora.py's nn.Linear + LoRA forward as one bf16 GEMM: against the float64 value of
    x W^T + b + sum_i s_i (x A_i^T) B_i^T, and against the reference's two-step bf16 form."""
    from minimaxh3_b200 import ops
    from minimaxh3_b200.kernels.fp8_linear import apply_lora_adapters
    from minimaxh3_b200.kernels.lora import attach_lora_registry

    lin = _linear(9, K, N).to(DEV)
    w, b = lin.weight.detach().cpu(), lin.bias.detach().cpu()
    adapters = [(_rand(40 + i, 16 * (i + 1), K, scale=0.05), _rand(50 + i, N, 16 * (i + 1), scale=0.05), 0.5 + i)
                for i in range(n_adapters)]
    x = _rand(10, M, K)
    exact = x.double() @ w.double().t() + b.double()
    for A, B, s in adapters:
        exact = exact + s * ((x.double() @ A.double().t()) @ B.double().t())
    dev_adapters = [(A.to(DEV), B.to(DEV), s) for A, B, s in adapters]
    got = ops.linear_lora(x.to(DEV), lin.weight, lin.bias, dev_adapters).float().cpu()
    r = OA.compare(got, exact)
    assert r["cos"] > 0.99999 and r["max_abs"] <= 1e-2 * max(r["ref_absmax"], 1e-3), r
    attach_lora_registry(nn.Sequential(lin))
    lin.adapters = dev_adapters
    wrapped = lin(x.to(DEV)).float().cpu()                      # the wrapped forward takes the fused path
    assert torch.equal(wrapped, got) or n_adapters == 0
    two_step = apply_lora_adapters(x.to(DEV), torch.nn.functional.linear(x.to(DEV), lin.weight, lin.bias),
                                   dev_adapters).float().cpu()
    r2 = OA.compare(got, two_step)
    assert r2["cos"] > 0.9999, r2


def test_fp8_linear_compiles_without_graph_breaks():
    import torch._dynamo as dynamo

    from minimaxh3_b200.kernels.fp8_linear import FP8Linear

    mod = FP8Linear.from_linear(_linear(9, 256, 128).to(DEV))
    mod.adapters = [(_rand(1, 16, 256, scale=0.01).to(DEV), _rand(2, 128, 16, scale=0.01).to(DEV), 1.0)]
    x = _rand(3, 4, 64, 256).to(DEV)
    dynamo.reset()
    assert dynamo.explain(lambda t: mod(t) * 2)(x).graph_break_count == 0
    compiled = torch.compile(lambda t: mod(t) * 2, backend="eager", fullgraph=True)
    assert torch.equal(compiled(x), mod(x) * 2)


def test_convert_transformer_and_forward():
    from minimaxh3_b200.kernels.fp8_linear import FP8Linear, convert_transformer_to_fp8

    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.to_q = nn.Linear(128, 128)
            self.norm_out = nn.Linear(128, 128)

        def forward(self, x):
            return self.norm_out(self.to_q(x))

    class T(nn.Module):
        def __init__(self):
            super().__init__()
            self.blocks = nn.ModuleList([Block() for _ in range(4)])

        def forward(self, x):
            for b in self.blocks:
                x = b(x)
            return x

    t = T().to(torch.bfloat16).to(DEV)
    n = convert_transformer_to_fp8(t, "norm", 1)
    assert n == 2
    assert isinstance(t.blocks[1].to_q, FP8Linear) and not isinstance(t.blocks[1].norm_out, FP8Linear)
    y = t(_rand(4, 8, 128).to(DEV))
    assert torch.isfinite(y.float()).all()
