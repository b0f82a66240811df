"""GPU parity at the benchmark configurations' own sizes (through the C ABI).

* Config 3: packed joint video+audio attention, cu_seqlens [0, 33784, 50676]
  (32760+1024 and 16380+512 tokens), H=40, D=128, per-(sequence, head)
  e4m3 scales, f16 PV product.  Checked on sampled query rows of both
  sequences against exact softmax attention over that sequence's keys only.
  The same lengths through the drop-in ``fp8_attention_varlen`` (bf16 in,
  its own per-(sequence, head) quantisation).
* Config 4: the FP8 scaled GEMM at M=32760, K=5120, N in {5120, 15360,
  13824} and the MLP-down shape (K=13824, N=5120): bit-equal to
  ``torch._scaled_mm`` with row-wise scales and bias (the reference's call,
  kernels/fp8_linear.py:95-102), and ``FP8Linear.forward`` with a rank-32
  LoRA adapter against the float64 value of the fused epilogue on sampled
  rows.
* fp32 input to ``quantize_rows`` / ``FP8Linear.from_linear``, which the
  reference's kernel accepts (kernels/fp8_linear.py:19,27-42).
"""
import math

import pytest
import torch

from oracle import fp8_attention_ref as OA
from oracle import fp8_linear_ref as OL

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _outlier_randn(gen, shape, D, gen_cpu):
    x = torch.randn(*shape, generator=gen, device=DEV)
    ch = int(torch.randperm(D, generator=gen_cpu)[0])
    x[..., ch] *= 8.0
    return x.to(torch.bfloat16).float()


def test_config3_packed_varlen_attention(record_margin):
    from minimaxh3_b200 import ops

    H, D = 40, 128
    lens = [33784, 16892]
    cu = torch.tensor([0, lens[0], lens[0] + lens[1]], dtype=torch.int32)
    T = int(cu[-1])
    g = torch.Generator(device=DEV).manual_seed(3)
    gc = torch.Generator().manual_seed(3)
    xs = [_outlier_randn(g, (T, H, D), D, gc) for _ in range(3)]
    # per-(sequence, head) absmax scales, e4m3 (benchmark configuration 3)
    q8s, scales = [], []
    for x in xs:
        s = torch.empty(len(lens), H, 1, device=DEV)
        x8 = torch.empty(T, H, D, dtype=torch.float8_e4m3fn, device=DEV)
        for b in range(len(lens)):
            seg = x[int(cu[b]):int(cu[b + 1])]
            s[b, :, 0] = torch.clamp(seg.abs().amax(dim=(0, 2)), min=1e-12) / 448.0
            x8[int(cu[b]):int(cu[b + 1])] = torch.clamp(seg / s[b, :, 0][None, :, None], -448, 448).to(x8.dtype)
        q8s.append(x8)
        scales.append(s)
    del xs
    (q8, k8, v8), (sq, sk, sv) = q8s, scales
    ls2 = OA.LOG2E / math.sqrt(D)
    v16 = v8.to(torch.float16)  # exact: the f16 PV product's operand
    out = ops.attention_e4m3(q8, k8, v16, sq, sk, sv, logit_scale_log2=ls2, cu_seqlens_q=cu.to(DEV),
                             cu_seqlens_k=cu.to(DEV), max_seqlen_q=max(lens))
    torch.cuda.synchronize()
    gs = torch.Generator().manual_seed(33)
    heads = [0, 17, 39]
    for b in range(len(lens)):
        lo, hi = int(cu[b]), int(cu[b + 1])
        rows = torch.cat([torch.tensor([0, hi - lo - 1]), torch.randint(1, hi - lo - 1, (30,), generator=gs)])
        for h in heads:
            qd = q8[lo:hi, h][rows].double().cpu() * float(sq[b, h, 0])
            kd = k8[lo:hi, h].double().cpu() * float(sk[b, h, 0])
            vd = v8[lo:hi, h].double().cpu() * float(sv[b, h, 0])
            ref = OA.sdpa_dequant_oracle(qd[None, None], kd[None, None], vd[None, None], ls2, base2=True)[0, 0]
            got = out[lo:hi, h][rows.to(DEV)].float().cpu()
            r = OA.compare(got, ref)
            record_margin(r, f"seq{b} head{h}")
            assert OA.within_tolerance(r), (b, h, r)


def test_config3_through_the_varlen_dropin(record_margin):
    """``fp8_attention_varlen`` on bf16 packed q/k/v at config 3's lengths: its per-(sequence, head)
    quantisation gives the kernel exactly the operands of a torch restatement (outputs bit-equal),
    and sampled rows are within tolerance of exact attention on those operands."""
    from minimaxh3_b200 import ops
    from minimaxh3_b200.kernels.fp8_attention import fp8_attention_varlen

    H, D = 40, 128
    lens = [33784, 16892]
    cu = torch.tensor([0, lens[0], lens[0] + lens[1]], dtype=torch.int32, device=DEV)
    T = lens[0] + lens[1]
    g = torch.Generator(device=DEV).manual_seed(31)
    gc = torch.Generator().manual_seed(31)
    q, k, v = (_outlier_randn(g, (T, H, D), D, gc).to(torch.bfloat16) for _ in range(3))
    out = fp8_attention_varlen(q, k, v, cu, cu, max(lens))
    ops_in, scales = [], []
    for x, dt in ((q, torch.float8_e4m3fn), (k, torch.float8_e4m3fn), (v, torch.float16)):
        s = torch.empty(len(lens), H, 1, device=DEV)
        y = torch.empty(T, H, D, dtype=dt, device=DEV)
        for b in range(len(lens)):
            lo, hi = int(cu[b]), int(cu[b + 1])
            # the correctly rounded quotient (float64, rounded once), as the drop-in computes it
            s[b, :, 0] = (torch.clamp(x[lo:hi].float().abs().amax(dim=(0, 2)), min=1e-12).double() / 448.0).float()
            t = x[lo:hi].float() / s[b, :, 0][None, :, None]
            y[lo:hi] = (torch.clamp(t, -448, 448) if dt == torch.float8_e4m3fn else t).to(dt)
        ops_in.append(y)
        scales.append(s)
    del q, k, v
    ls2 = OA.LOG2E / math.sqrt(D)
    ref_kernel = ops.attention_e4m3(*ops_in, *scales, logit_scale_log2=ls2, cu_seqlens_q=cu, cu_seqlens_k=cu,
                                    max_seqlen_q=max(lens))
    assert torch.equal(out, ref_kernel)
    (q8, k8, v16), (sq, sk, sv) = ops_in, scales
    gs = torch.Generator().manual_seed(34)
    for b in range(len(lens)):
        lo, hi = int(cu[b]), int(cu[b + 1])
        rows = torch.cat([torch.tensor([0, hi - lo - 1]), torch.randint(1, hi - lo - 1, (16,), generator=gs)])
        for h in (3, 38):
            qd = q8[lo:hi, h][rows].double().cpu() * float(sq[b, h, 0])
            kd = k8[lo:hi, h].double().cpu() * float(sk[b, h, 0])
            vd = v16[lo:hi, h].double().cpu() * float(sv[b, h, 0])
            ref = OA.sdpa_dequant_oracle(qd[None, None], kd[None, None], vd[None, None], ls2, base2=True)[0, 0]
            r = OA.compare(out[lo:hi, h][rows.to(DEV)].float().cpu(), ref)
            record_margin(r, f"drop-in seq{b} head{h}")
            assert OA.within_tolerance(r), (b, h, r)


CONFIG4 = [(32760, 5120, 5120), (32760, 5120, 15360), (32760, 5120, 13824), (32760, 13824, 5120)]


@pytest.mark.parametrize("M,K,N", CONFIG4)
def test_config4_gemm_bit_equal_to_scaled_mm(M, K, N):
    from minimaxh3_b200 import ops

    g = torch.Generator(device=DEV).manual_seed(4)
    x = torch.randn(M, K, generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    bias = (torch.randn(N, generator=g, device=DEV) * 0.01).to(torch.bfloat16)
    x8, sa = ops.quantize_rows(x)
    w8, sb = ops.quantize_rows(w)
    del x, w
    ours = ops.scaled_gemm(x8, w8, row_scale=sa, col_scale=sb, bias=bias)
    ref = torch._scaled_mm(x8, w8.t(), scale_a=sa, scale_b=sb.reshape(1, -1), bias=bias, out_dtype=torch.bfloat16)
    ndiff = int((ours != ref).sum())
    assert ndiff == 0, (ndiff, float((ours.float() - ref.float()).abs().max()))


@pytest.mark.parametrize("M,K,N", CONFIG4)
def test_config4_fp8_linear_with_lora(M, K, N, record_margin):
    from minimaxh3_b200.kernels.fp8_linear import FP8Linear

    g = torch.Generator(device=DEV).manual_seed(44)
    lin = torch.nn.Linear(K, N).to(device=DEV, dtype=torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(N, K, generator=g, device=DEV) * 0.02)
        lin.bias.copy_(torch.randn(N, generator=g, device=DEV) * 0.01)
    x = torch.randn(M, K, generator=g, device=DEV).to(torch.bfloat16)
    A = (torch.randn(32, K, generator=g, device=DEV) * 0.01).to(torch.bfloat16)
    Bm = (torch.randn(N, 32, generator=g, device=DEV) * 0.01).to(torch.bfloat16)
    mod = FP8Linear.from_linear(lin)
    mod.adapters = [(A, Bm, 1.0)]
    y = mod(x)
    rows = torch.cat([torch.tensor([0, M - 1]), torch.randint(1, M - 1, (46,), generator=torch.Generator().manual_seed(5))])
    xs = x[rows.to(DEV)].cpu()
    ref = OL.fp8_linear_fused_oracle(xs, mod.w8.cpu(), mod.w_scale.cpu(), mod.bias.cpu(), [(A.cpu(), Bm.cpu(), 1.0)])
    got = y[rows.to(DEV)].float().cpu()
    r = OA.compare(got, ref)
    record_margin(r)
    assert r["cos"] > 0.99999, r
    # one bf16 rounding of the fp32 result
    assert bool(((got - ref).abs() <= ref.abs() * 2.0 ** -7 + 1e-3).all()), r


def test_fp32_rows_and_linear_match_reference_bytes():
    from minimaxh3_b200.kernels.fp8_linear import FP8Linear, quantize_rows

    g = torch.Generator().manual_seed(6)
    x = torch.randn(77, 320, generator=g) * 3.0
    x8, xs = quantize_rows(x.to(DEV))
    r8, rs = OL.quantize_rows(x)
    assert torch.equal(x8.cpu().view(torch.uint8), r8.view(torch.uint8)) and torch.equal(xs.cpu(), rs)
    # an fp32 nn.Linear converts as the reference's does: fp32 weight rows quantised directly
    lin = torch.nn.Linear(320, 96)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(96, 320, generator=g) * 0.02)
    w_ref = lin.weight.detach().clone()
    mod = FP8Linear.from_linear(lin.to(DEV))
    w8r, wsr = OL.quantize_rows(w_ref)
    assert torch.equal(mod.w8.cpu().view(torch.uint8), w8r.view(torch.uint8))
    assert torch.equal(mod.w_scale.cpu().reshape(-1), wsr.reshape(-1))
    y = mod(x.to(DEV))
    assert y.dtype == torch.float32 and y.shape == (77, 96)
    ref = OL.fp8_linear_fused_oracle(x, w8r, wsr.view(1, -1), mod.bias.cpu(), [])
    r = OA.compare(y.cpu(), ref)
    assert r["cos"] > 0.99999, r
