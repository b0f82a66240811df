"""Host-resident attention (minimaxh3_b200.streaming) equals one device call."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("heads_per_chunk", [None, 4])
def test_fp8_attention_host_matches_device_call(heads_per_chunk):
    from minimaxh3_b200.kernels.fp8_attention import fp8_attention
    from minimaxh3_b200.streaming import fp8_attention_host

    B, H, Sq, Sk, D = 2, 6, 300, 520, 128
    g = torch.Generator().manual_seed(11)
    q, k, v = (torch.randn(B, H, S, D, generator=g).to(torch.bfloat16).pin_memory() for S in (Sq, Sk, Sk))
    key_mask = torch.rand(B, Sk, generator=g) > 0.1
    out = fp8_attention_host(q, k, v, key_mask=key_mask, heads_per_chunk=heads_per_chunk)
    torch.cuda.synchronize()
    ref = fp8_attention(q.cuda(), k.cuda(), v.cuda(), key_mask=key_mask.cuda()).cpu()
    assert out.device.type == "cpu" and out.shape == ref.shape
    assert torch.equal(out, ref)


def test_fp8_attention_host_rejects_device_tensors():
    from minimaxh3_b200.streaming import fp8_attention_host

    x = torch.zeros(1, 1, 8, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        fp8_attention_host(x, x, x)
