"""GPU parity of the sm_100a FP8 attention kernel (through the C ABI).

Checks against the CPU oracle (oracle/fp8_attention_ref.py):
* the fp32/float64 SDPA oracle on the dequantised inputs - the north-star
  tolerance (cos >= 0.9995, max-abs <= 2e-2 * max(1, max|oracle|));
* the exact-exp2 emulation of the kernel's own block algorithm (tight);
* the reference algorithm's output, which the kernel must beat in accuracy.
"""
import math

import pytest
import torch

from conftest import COS_MIN
from oracle import fp8_attention_ref as OA

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _inputs(seed, B, H, Sq, Sk, D, dtype=torch.bfloat16, outliers=True):
    g = torch.Generator().manual_seed(seed)
    out = []
    for S in (Sq, Sk, Sk):
        x = torch.randn(B, H, S, D, generator=g)
        if outliers:
            ch = torch.randperm(D, generator=g)[: max(1, round(0.01 * D))]
            x[..., ch] *= 8.0
        out.append(x.to(dtype))
    return out


def _per_bh(x):
    xf = x.float()
    s = torch.clamp(xf.abs().amax(dim=(2, 3)), min=1e-12) / 448.0
    return torch.clamp(xf / s[..., None, None], -448, 448).to(torch.float8_e4m3fn), s


def _run_e4m3(q8, k8, v8, sq, sk, sv, ls2, pv="e4m3", **kw):
    """Run the kernel; pv="f16" widens the e4m3 V exactly to f16 (16-bit PV)."""
    from minimaxh3_b200 import ops

    vd = v8.to(DEV)
    if pv == "f16":
        vd = ops.widen_e4m3_to_f16(vd.contiguous())
    return ops.attention_e4m3(q8.to(DEV), k8.to(DEV), vd, sq.to(DEV), sk.to(DEV), sv.to(DEV),
                              logit_scale_log2=ls2, **kw)


def _check(r, pv):
    """f16 PV: the north-star tolerance; e4m3 PV: cosine, and max-abs within 4e-2."""
    if pv == "f16":
        assert OA.within_tolerance(r), r
    else:
        assert r["cos"] >= COS_MIN, r
        assert r["max_abs"] <= 4e-2 * max(1.0, r["ref_absmax"]), r


CASES = [
    # B, H, Sq, Sk, D
    (1, 2, 256, 256, 128),
    (1, 2, 300, 300, 128),     # ragged tails
    (2, 3, 129, 1000, 128),    # cross-attention shape, odd Q tile count
    (1, 1, 1, 77, 128),        # single query, short keys
    (1, 2, 640, 4096, 128),
    (1, 2, 384, 520, 64),
]


@pytest.mark.parametrize("pv", ["f16", "e4m3"])
@pytest.mark.parametrize("B,H,Sq,Sk,D", CASES)
def test_attention_per_bh_scales_vs_oracles(B, H, Sq, Sk, D, pv):
    q, k, v = _inputs(Sq + Sk + D, B, H, Sq, Sk, D)
    (q8, sq), (k8, sk), (v8, sv) = _per_bh(q), _per_bh(k), _per_bh(v)
    ls2 = OA.LOG2E / math.sqrt(D)
    out = _run_e4m3(q8, k8, v8, sq[..., None], sk[..., None], sv[..., None], ls2, pv=pv).float().cpu()
    assert torch.isfinite(out).all()
    ref = OA.sdpa_dequant_oracle(q8.double() * sq[..., None, None], k8.double() * sk[..., None, None],
                                 v8.double() * sv[..., None, None], ls2, base2=True)
    _check(OA.compare(out, ref), pv)
    emu = OA.exp2_attention_emulation(q8, k8, v8, sq[..., None], sk[..., None], sv[..., None].expand(B, H, D),
                                      logit_scale_log2=ls2,
                                      p_dtype=torch.float16 if pv == "f16" else torch.float8_e4m3fn)
    re = OA.compare(out, emu)
    assert re["cos"] > 0.9999, re


@pytest.mark.parametrize("pv", ["f16", "e4m3"])
def test_attention_block_scales_and_fp16_out(pv):
    B, H, S, D = 1, 2, 700, 128
    q, k, v = _inputs(3, B, H, S, S, D)
    c = OA.LOG2E / math.sqrt(D)
    q8, sq = OA.quantize_q(q, c)
    k8, sk = OA.quantize_k(k, OA.k_channel_mean(k))
    v8, sv = OA.quantize_v(v)
    out = _run_e4m3(q8, k8, v8, sq, sk, sv, 1.0, pv=pv, out_dtype=torch.float16).float().cpu()
    ref = OA.sdpa_dequant_oracle(OA.dequant_blocks(q8, sq), OA.dequant_blocks(k8, sk),
                                 v8.double() * sv.double()[:, :, None, :], 1.0, base2=True)
    r = OA.compare(out, ref)
    _check(r, pv)
    # Far closer to the oracle than the reference's own algorithm on the same bytes.
    r_ref = OA.compare(OA.attention_kernel_ref(q8, k8, v8, sq, sk, sv), ref)
    assert r["cos"] > r_ref["cos"] and r["max_abs"] < r_ref["max_abs"], (r, r_ref)


@pytest.mark.parametrize("pv", ["f16", "e4m3"])
def test_attention_key_bias_and_mask(pv):
    from minimaxh3_b200 import ops

    B, H, Sq, Sk, D = 2, 2, 200, 333, 128
    q, k, v = _inputs(4, B, H, Sq, Sk, D)
    (q8, sq), (k8, sk), (v8, sv) = _per_bh(q), _per_bh(k), _per_bh(v)
    g = torch.Generator().manual_seed(9)
    key_bias = torch.randn(B, Sk, generator=g)
    key_bias[:, ::5] = -1.0e9
    key_mask = torch.rand(B, Sk, generator=g) > 0.2
    key_mask[1, :] = False  # a batch with every key masked -> zeros
    ls2 = OA.LOG2E / math.sqrt(D)
    bias2, _ = ops.key_bias_inputs(key_mask.to(DEV), key_bias.to(DEV), B, Sk, DEV)
    out = _run_e4m3(q8, k8, v8, sq[..., None], sk[..., None], sv[..., None], ls2, pv=pv,
                    key_bias2=bias2).float().cpu()
    ref = OA.sdpa_dequant_oracle(q8.double() * sq[..., None, None], k8.double() * sk[..., None, None],
                                 v8.double() * sv[..., None, None], ls2, key_mask=key_mask, key_bias=key_bias,
                                 base2=True)
    assert torch.equal(out[1], torch.zeros_like(out[1]))
    _check(OA.compare(out[0], ref[0]), pv)


@pytest.mark.parametrize("pv", ["f16", "e4m3"])
def test_attention_varlen_matches_per_sequence(pv):
    """cu_seqlens packing == one dense call per sequence (config 3 layout, small)."""
    from minimaxh3_b200 import ops

    H, D = 2, 128
    lens = [300, 77, 513]
    total = sum(lens)
    g = torch.Generator().manual_seed(5)
    x = [torch.randn(total, H, D, generator=g).to(torch.bfloat16) for _ in range(3)]
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    q8s, k8s, v8s, sqs, sks, svs = [], [], [], [], [], []
    for i, L in enumerate(lens):
        sl = slice(int(cu[i]), int(cu[i + 1]))
        for t, dst, sdst in ((x[0], q8s, sqs), (x[1], k8s, sks), (x[2], v8s, svs)):
            seg = t[sl].permute(1, 0, 2)[None]  # [1,H,L,D]
            t8, s = _per_bh(seg)
            dst.append(t8[0].permute(1, 0, 2))
            sdst.append(s[0])
    q8 = torch.cat(q8s).contiguous()
    k8 = torch.cat(k8s).contiguous()
    v8 = torch.cat(v8s).contiguous()
    sq = torch.stack(sqs)[..., None]
    sk = torch.stack(sks)[..., None]
    sv = torch.stack(svs)[..., None]
    ls2 = OA.LOG2E / math.sqrt(D)
    vd = v8.to(DEV)
    if pv == "f16":
        vd = ops.widen_e4m3_to_f16(vd)
    out = ops.attention_e4m3(q8.to(DEV), k8.to(DEV), vd, sq.to(DEV), sk.to(DEV), sv.to(DEV),
                             logit_scale_log2=ls2, cu_seqlens_q=cu.to(DEV), cu_seqlens_k=cu.to(DEV),
                             max_seqlen_q=max(lens)).float().cpu()
    for i, L in enumerate(lens):
        sl = slice(int(cu[i]), int(cu[i + 1]))
        qi, ki, vi = (t[sl].permute(1, 0, 2)[None] for t in (q8, k8, v8))
        ref = OA.sdpa_dequant_oracle(qi.double() * sq[i][None, :, :, None], ki.double() * sk[i][None, :, :, None],
                                     vi.double() * sv[i][None, :, :, None], ls2, base2=True)
        _check(OA.compare(out[sl].permute(1, 0, 2)[None], ref), pv)


@pytest.mark.parametrize("pv", ["f16", "e4m3"])
def test_attention_strided_views(pv):
    """[B,S,H,D] storage seen as [B,H,S,D] (what diffusers passes) for every operand."""
    from minimaxh3_b200 import ops

    B, H, S, D = 1, 4, 384, 128
    q, k, v = _inputs(6, B, H, S, S, D)
    (q8, sq), (k8, sk), (v8, sv) = _per_bh(q), _per_bh(k), _per_bh(v)
    vv = v8.to(DEV)
    if pv == "f16":
        vv = ops.widen_e4m3_to_f16(vv)
    views = [t.to(DEV).permute(0, 2, 1, 3).contiguous().permute(0, 2, 1, 3) for t in (q8, k8, vv)]
    ls2 = OA.LOG2E / math.sqrt(D)
    out_store = torch.empty(B, S, H, D, dtype=torch.bfloat16, device=DEV)
    s3 = [x[..., None].to(DEV) for x in (sq, sk, sv)]
    out = ops.attention_e4m3(*views, *s3, logit_scale_log2=ls2, out=out_store.permute(0, 2, 1, 3))
    ref = ops.attention_e4m3(q8.to(DEV), k8.to(DEV), vv, *s3, logit_scale_log2=ls2)
    assert torch.equal(out, ref)


@pytest.mark.parametrize("pv", ["f16", "e4m3"])
@pytest.mark.parametrize("use_bias", [False, True])
def test_attention_rising_row_max(pv, use_bias):
    """Logits that grow along the keys raise the running max in most tiles.

    The kernel computes P with the old max while it takes the tile max and
    redoes the tile when a row has to raise it; this drives that path (and
    the O rescale) on nearly every tile, through the scale and bias forms.
    """
    from minimaxh3_b200 import ops

    B, H, Sq, Sk, D = 1, 2, 256, 2000, 128
    g = torch.Generator().manual_seed(21)
    u = torch.randn(D, generator=g)
    u = u / u.norm()
    ramp = torch.linspace(0.0, 1.0, Sk)
    q = 3.0 * u + 0.5 * torch.randn(B, H, Sq, D, generator=g)
    if use_bias:
        k = torch.randn(B, H, Sk, D, generator=g)
        key_bias = (80.0 * ramp)[None].expand(B, Sk).contiguous()
    else:
        k = (300.0 * ramp)[:, None] * u + 0.5 * torch.randn(B, H, Sk, D, generator=g)
        key_bias = None
    v = torch.randn(B, H, Sk, D, generator=g)
    (q8, sq), (k8, sk), (v8, sv) = (_per_bh(t.to(torch.bfloat16)) for t in (q, k, v))
    ls2 = OA.LOG2E / math.sqrt(D)
    kw = {}
    if use_bias:
        kw["key_bias2"], _ = ops.key_bias_inputs(None, key_bias.to(DEV), B, Sk, DEV)
    out = _run_e4m3(q8, k8, v8, sq[..., None], sk[..., None], sv[..., None], ls2, pv=pv, **kw).float().cpu()
    assert torch.isfinite(out).all()
    ref = OA.sdpa_dequant_oracle(q8.double() * sq[..., None, None], k8.double() * sk[..., None, None],
                                 v8.double() * sv[..., None, None], ls2, key_bias=key_bias, base2=True)
    _check(OA.compare(out, ref), pv)


@pytest.mark.parametrize("pv", ["f16", "e4m3"])
def test_attention_large_head_subset_property(pv):
    """Config-2 sequence length: finite, and sampled rows match the oracle."""
    B, H, S, D = 1, 2, 32760, 128
    q, k, v = _inputs(0, B, H, S, S, D)
    (q8, sq), (k8, sk), (v8, sv) = _per_bh(q), _per_bh(k), _per_bh(v)
    ls2 = OA.LOG2E / math.sqrt(D)
    out = _run_e4m3(q8, k8, v8, sq[..., None], sk[..., None], sv[..., None], ls2, pv=pv).float().cpu()
    assert torch.isfinite(out).all()
    rows = torch.cat([torch.tensor([0, 1, 127, 128, 4097, 16383, 32639, 32640, 32759]),
                      torch.randperm(S, generator=torch.Generator().manual_seed(1))[:247]])
    ref = OA.sdpa_dequant_oracle(q8[:, :, rows].double() * sq[..., None, None], k8.double() * sk[..., None, None],
                                 v8.double() * sv[..., None, None], ls2, base2=True)
    _check(OA.compare(out[:, :, rows], ref), pv)


def test_attention_rejects_bad_arguments():
    from minimaxh3_b200 import ops

    q8 = torch.zeros(1, 1, 128, 96, dtype=torch.float8_e4m3fn, device=DEV)
    s = torch.ones(1, 1, 1, device=DEV)
    with pytest.raises(ValueError):
        ops.attention_e4m3(q8, q8, q8, s, s, s)


def test_widen_e4m3_to_f16_exact():
    from minimaxh3_b200 import ops

    allbytes = torch.arange(256, dtype=torch.uint8).repeat(64)
    x8 = allbytes.view(torch.float8_e4m3fn)
    got = ops.widen_e4m3_to_f16(x8.to(DEV)).cpu()
    ref = x8.to(torch.float16)
    nan = torch.isnan(ref)
    assert torch.equal(torch.isnan(got), nan)
    assert torch.equal(got[~nan], ref[~nan])


@pytest.mark.parametrize("pv", ["f16", "e4m3"])
def test_padded_batch_kv_len_skips_tiles_exactly(pv):
    """A padded batch (valid keys = a prefix) through fp8_attention: the kernel
    skips the tiles past each batch's last valid key (kv_len), bit-identical
    to computing them masked, and matches the masked oracle."""
    from minimaxh3_b200 import ops
    from minimaxh3_b200.kernels.fp8_attention import fp8_attention

    B, H, Sq, Sk, D = 3, 2, 300, 1000, 128
    q, k, v = _inputs(13, B, H, Sq, Sk, D)
    lens = torch.tensor([700, 1000, 131])
    key_mask = torch.arange(Sk)[None, :] < lens[:, None]
    out = fp8_attention(q.to(DEV), k.to(DEV), v.to(DEV), key_mask=key_mask.to(DEV)).float().cpu()
    assert torch.isfinite(out).all()
    bias2, kv = ops.key_bias_inputs(key_mask.to(DEV), None, B, Sk, DEV)
    assert kv.cpu().tolist() == lens.tolist()
    # same bytes through the kernel with and without the per-batch length
    (q8, sq), (k8, sk), (v8, sv) = _per_bh(q), _per_bh(k), _per_bh(v)
    ls2 = OA.LOG2E / math.sqrt(D)
    args = (q8, k8, v8, sq[..., None], sk[..., None], sv[..., None], ls2)
    full = _run_e4m3(*args, pv=pv, key_bias2=bias2)
    skip = _run_e4m3(*args, pv=pv, key_bias2=bias2, kv_len=kv)
    assert torch.equal(full, skip)
    ref = OA.sdpa_dequant_oracle(q8.double() * sq[..., None, None], k8.double() * sk[..., None, None],
                                 v8.double() * sv[..., None, None], ls2, key_mask=key_mask, base2=True)
    _check(OA.compare(skip.float().cpu(), ref), pv)


@pytest.mark.parametrize("pv", ["f16", "e4m3"])
def test_attention_varlen_empty_and_one_token_sequences(pv):
    """Packed sequences of 0 and 1 tokens, and different query / key packings (cross-attention):
    a sequence with no queries writes nothing, one with no keys gives 0, the rest match the oracle."""
    from minimaxh3_b200 import ops

    H, D = 2, 128
    lq, lk = [5, 0, 130, 1, 64], [0, 7, 300, 1, 129]
    g = torch.Generator().manual_seed(11)
    cq = torch.tensor([0] + list(torch.tensor(lq).cumsum(0)), dtype=torch.int32)
    ck = torch.tensor([0] + list(torch.tensor(lk).cumsum(0)), dtype=torch.int32)
    q = torch.randn(int(cq[-1]), H, D, generator=g).to(torch.bfloat16)
    k = torch.randn(int(ck[-1]), H, D, generator=g).to(torch.bfloat16)
    v = torch.randn(int(ck[-1]), H, D, generator=g).to(torch.bfloat16)

    def quant(t, cu):
        t8 = torch.empty(t.shape, dtype=torch.float8_e4m3fn)
        sc = torch.ones(len(cu) - 1, H, 1)
        for i in range(len(cu) - 1):
            sl = slice(int(cu[i]), int(cu[i + 1]))
            if sl.stop > sl.start:
                s = torch.clamp(t[sl].float().abs().amax(dim=(0, 2)), min=1e-12) / 448.0
                sc[i, :, 0] = s
                t8[sl] = torch.clamp(t[sl].float() / s[None, :, None], -448, 448).to(torch.float8_e4m3fn)
        return t8, sc

    (q8, sq), (k8, sk), (v8, sv) = quant(q, cq), quant(k, ck), quant(v, ck)
    ls2 = OA.LOG2E / math.sqrt(D)
    vd = v8.to(DEV)
    if pv == "f16":
        vd = ops.widen_e4m3_to_f16(vd)
    out = torch.full((int(cq[-1]), H, D), 7.0, dtype=torch.bfloat16, device=DEV)
    ops.attention_e4m3(q8.to(DEV), k8.to(DEV), vd, sq.to(DEV), sk.to(DEV), sv.to(DEV), logit_scale_log2=ls2,
                       cu_seqlens_q=cq.to(DEV), cu_seqlens_k=ck.to(DEV), max_seqlen_q=max(lq), out=out)
    out = out.float().cpu()
    for i in range(len(lq)):
        qs, ks = slice(int(cq[i]), int(cq[i + 1])), slice(int(ck[i]), int(ck[i + 1]))
        if lq[i] == 0:
            continue
        if lk[i] == 0:
            assert torch.equal(out[qs], torch.zeros_like(out[qs])), i
            continue
        qi, ki, vi = (t.permute(1, 0, 2)[None] for t in (q8[qs], k8[ks], v8[ks]))
        ref = OA.sdpa_dequant_oracle(qi.double() * sq[i][None, :, :, None], ki.double() * sk[i][None, :, :, None],
                                     vi.double() * sv[i][None, :, :, None], ls2, base2=True)
        _check(OA.compare(out[qs].permute(1, 0, 2)[None], ref), pv)
