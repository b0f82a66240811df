"""Per-(batch, head) quantisation kernels (mh3_absmax_bh, mh3_quantize_bh) vs a torch restatement."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _restated(x, scale, P, out_dtype):
    B, S, H, D = x.shape
    y = x.float() / scale[:, None, :, None]
    if out_dtype == torch.float8_e4m3fn:
        y = torch.clamp(y, -448.0, 448.0)
    return y.to(out_dtype).reshape(B, S, P, H // P, D).permute(2, 0, 1, 3, 4).contiguous()


@pytest.mark.parametrize("B,S,H,D,P", [(1, 1000, 8, 128, 2), (2, 517, 6, 64, 3), (1, 37, 4, 128, 1)])
@pytest.mark.parametrize("out_dtype", [torch.float8_e4m3fn, torch.float16])
@pytest.mark.parametrize("in_dtype", [torch.bfloat16, torch.float16])
def test_quantize_bh_bit_exact(B, S, H, D, P, out_dtype, in_dtype):
    from minimaxh3_b200 import ops

    g = torch.Generator(device="cuda").manual_seed(B * 1000 + S)
    x = torch.randn(B, H, S, D, generator=g, device="cuda")
    x[..., 3] *= 8.0
    x = x.to(in_dtype).permute(0, 2, 1, 3)          # [B,S,H,D] view of [B,H,S,D] storage
    amax = ops.absmax_bh(x)
    assert torch.equal(amax, x.float().abs().amax(dim=(1, 3)))
    scale = torch.clamp(amax, min=1e-12) / 448.0
    got = ops.quantize_bh(x, scale, out_dtype=out_dtype, groups=P)
    ref = _restated(x, scale, P, out_dtype)
    assert got.shape == ref.shape
    assert torch.equal(got.view(torch.uint8) if out_dtype != torch.float16 else got.view(torch.int16),
                       ref.view(torch.uint8) if out_dtype != torch.float16 else ref.view(torch.int16))


def test_bh_kernels_reject_bad_arguments():
    from minimaxh3_b200 import ops

    x = torch.zeros(1, 8, 6, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        ops.quantize_bh(x, torch.ones(6, device="cuda"), groups=4)       # 4 does not divide 6
    with pytest.raises(ValueError):
        ops.absmax_bh(torch.zeros(1, 8, 6, 96, dtype=torch.bfloat16, device="cuda"))


@pytest.mark.parametrize("B,S,H,D,P,off,hs", [(1, 1000, 8, 128, 2, 1, 2), (2, 517, 12, 64, 3, 0, 1),
                                              (1, 300, 8, 128, 1, 3, 4), (1, 129, 4, 128, 4, 0, 1)])
@pytest.mark.parametrize("out_dtype", [torch.float8_e4m3fn, torch.float16])
def test_head_selection_bit_exact(B, S, H, D, P, off, hs, out_dtype):
    """absmax_bh / quantize_bh over heads p*(H/P)+off+i equal the full-head kernels restricted to them."""
    from minimaxh3_b200 import ops

    g = torch.Generator(device="cuda").manual_seed(H * 100 + off)
    x = torch.randn(B, H, S, D, generator=g, device="cuda").to(torch.bfloat16).permute(0, 2, 1, 3)
    heads = [p * (H // P) + off + i for p in range(P) for i in range(hs)]
    amax = ops.absmax_bh(x, groups=P, head_off=off, heads_sel=hs)
    assert torch.equal(amax, x.float().abs().amax(dim=(1, 3))[:, heads])
    scale = torch.clamp(amax, min=1e-12) / 448.0
    got = ops.quantize_bh(x, scale, out_dtype=out_dtype, groups=P, head_off=off, heads_sel=hs)
    ref = _restated(x[:, :, heads], scale, P, out_dtype)
    assert got.shape == (P, B, S, hs, D)
    bits = torch.uint8 if out_dtype != torch.float16 else torch.int16
    assert torch.equal(got.view(bits), ref.view(bits))


def test_head_selection_rejects_bad_ranges():
    from minimaxh3_b200 import ops

    x = torch.zeros(1, 8, 8, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        ops.absmax_bh(x, groups=2, head_off=3, heads_sel=2)              # 3+2 > 4 heads per group
    with pytest.raises(ValueError):
        ops.quantize_bh(x, torch.ones(1, 4, device="cuda"), groups=2, head_off=0, heads_sel=3)


def _restated_seg(x, seg, scale, P, heads, out_dtype):
    """Rows [seg[z], seg[z+1]) (clamped to [0, S]) / scale[z]; zeros outside every segment."""
    S, H, D = x.shape
    b = [min(max(c, 0), S) for c in seg]
    y = torch.zeros(S, len(heads), D, device=x.device)
    for z, (lo, hi) in enumerate(zip(b, b[1:])):
        if hi > lo:
            y[lo:hi] = x[lo:hi, heads].float() / scale[z][None, :, None]
    if out_dtype == torch.float8_e4m3fn:
        y = torch.clamp(y, -448.0, 448.0)
    return y.to(out_dtype).reshape(1, S, P, len(heads) // P, D).permute(2, 0, 1, 3, 4).contiguous()


@pytest.mark.parametrize("S,H,D,seg,P,off,hs", [
    (1000, 8, 128, [0, 300, 300, 1000], 1, 0, 8),        # an empty segment
    (3000, 6, 64, [17, 1500, 2999], 3, 0, 2),            # rows before the first and after the last
    (2048, 8, 128, [-40, 700, 1900, 5000], 2, 1, 2),     # bounds clamped to [0, S]; head selection
    (129, 4, 128, [0, 129], 4, 0, 1),
])
@pytest.mark.parametrize("out_dtype", [torch.float8_e4m3fn, torch.float16])
@pytest.mark.parametrize("in_dtype", [torch.bfloat16, torch.float16])
def test_segment_kernels_bit_exact(S, H, D, seg, P, off, hs, out_dtype, in_dtype):
    """mh3_absmax_seg / mh3_quantize_seg: per-(segment, head) amax and quantisation of a packed shard."""
    from minimaxh3_b200 import ops

    g = torch.Generator(device="cuda").manual_seed(S + H)
    x = torch.randn(S, H, D, generator=g, device="cuda")
    x[:, :, 5] *= 8.0
    x = x.to(in_dtype)
    heads = [p * (H // P) + off + i for p in range(P) for i in range(hs)]
    segt = torch.tensor(seg, dtype=torch.int32, device="cuda")
    amax = ops.absmax_seg(x, segt, groups=P, head_off=off, heads_sel=hs)
    b = [min(max(c, 0), S) for c in seg]
    ref_amax = torch.stack([x[lo:hi, heads].float().abs().amax(dim=(0, 2)) if hi > lo
                            else torch.zeros(len(heads), device="cuda") for lo, hi in zip(b, b[1:])])
    assert torch.equal(amax, ref_amax)
    scale = torch.clamp(amax, min=1e-12) / 448.0
    got = ops.quantize_seg(x[None], segt, scale, out_dtype=out_dtype, groups=P, head_off=off, heads_sel=hs)
    ref = _restated_seg(x, seg, scale, P, heads, out_dtype)
    assert got.shape == (P, 1, S, hs, D)
    bits = torch.uint8 if out_dtype != torch.float16 else torch.int16
    assert torch.equal(got.view(bits), ref.view(bits))


def test_segment_kernels_reject_bad_arguments():
    from minimaxh3_b200 import ops

    x = torch.zeros(64, 4, 128, dtype=torch.bfloat16, device="cuda")
    seg = torch.tensor([0, 64], dtype=torch.int32, device="cuda")
    with pytest.raises(ValueError):
        ops.absmax_seg(x, seg.long())                                     # int32 offsets only
    with pytest.raises(ValueError):
        ops.absmax_seg(x, seg[:1])                                        # no segment
    with pytest.raises(ValueError):
        ops.quantize_seg(x, seg, torch.ones(2, 4, device="cuda"))        # one scale row per segment
    with pytest.raises(ValueError):
        ops.absmax_seg(torch.zeros(2, 64, 4, 128, dtype=torch.bfloat16, device="cuda"), seg)   # batch 2


def test_scale_from_absmax_on_the_device_is_correctly_rounded():
    """The scale helper the varlen and Ulysses paths use gives the IEEE float32 quotient on CUDA
    tensors too (the same bits as the quantisation kernels' own division)."""
    import numpy as np

    from minimaxh3_b200 import ops

    g = torch.Generator().manual_seed(1)
    amax = torch.cat([torch.rand(200000, generator=g) * 40, torch.exp(torch.randn(200000, generator=g) * 20)]).float()
    got = ops.scale_from_absmax(amax.cuda()).cpu()
    ref = np.maximum(amax.numpy(), np.float32(1e-12)) / np.float32(448.0)
    assert np.array_equal(got.numpy(), ref)
