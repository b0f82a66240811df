"""Host-side argument logic that needs no GPU: strided-copy bounds, head selection, head groups."""
import pytest
import torch

from minimaxh3_b200 import ops
from minimaxh3_b200.ulysses import _check_heads, default_head_groups


def test_copy_rows_rejects_copies_outside_either_tensor():
    src = torch.zeros(4 * 64, dtype=torch.uint8)
    dst = torch.zeros(4 * 32, dtype=torch.uint8)
    # 4 rows of 32 bytes at a 64-byte pitch fit src; 4 rows at a 40-byte pitch overrun dst
    with pytest.raises(ValueError, match="past the end of dst"):
        ops.copy_rows(dst, 0, 40, src, 0, 64, 32, 4)
    with pytest.raises(ValueError, match="past the end of src"):
        ops.copy_rows(dst, 0, 32, src, 40, 64, 32, 4)
    with pytest.raises(ValueError, match="bad offsets"):
        ops.copy_rows(dst, 0, 16, src, 0, 64, 32, 4)           # pitch below the row length
    with pytest.raises(ValueError, match="contiguous"):
        ops.copy_rows(dst, 0, 32, torch.zeros(8, 64, dtype=torch.uint8).t(), 0, 64, 32, 4)
    with pytest.raises(ValueError, match="CUDA"):
        ops.copy_rows(dst, 0, 32, src, 0, 64, 32, 4)           # in bounds, but neither side is on a GPU


def test_head_selection_arithmetic():
    assert ops._head_sel(40, 2, 0, None) == (20, 0, 20)
    assert ops._head_sel(40, 2, 5, 5) == (20, 5, 5)
    for args in ((40, 3, 0, None), (40, 2, 18, 5), (40, 2, -1, 2), (40, 2, 0, 0)):
        with pytest.raises(ValueError):
            ops._head_sel(*args)


def test_head_groups_defaults_and_checks():
    assert [default_head_groups(h) for h in (40, 20, 10, 5, 1)] == [20, 10, 5, 5, 1]
    _check_heads(40, 2, 10)
    with pytest.raises(ValueError):
        _check_heads(40, 3, 1)
    with pytest.raises(ValueError):
        _check_heads(40, 2, 3)


def test_scale_from_absmax_is_the_correctly_rounded_quotient():
    """max(amax, 1e-12) / 448 in float32, rounded once - the IEEE quotient the quantisation
    kernels compute, whatever the device's scalar-division shortcut."""
    import numpy as np
    import torch

    from minimaxh3_b200 import ops

    g = torch.Generator().manual_seed(0)
    amax = torch.cat([torch.rand(100000, generator=g) * 40, torch.exp(torch.randn(100000, generator=g) * 20),
                      torch.tensor([0.0, 1e-13, 448.0, 3.4e38, 1.0])]).float()
    got = ops.scale_from_absmax(amax)
    ref = np.maximum(amax.numpy(), np.float32(1e-12)) / np.float32(448.0)   # numpy float32: IEEE division
    assert got.dtype == torch.float32
    assert np.array_equal(got.numpy(), ref)


def test_ulysses_exchange_argument_is_checked_before_any_collective():
    from minimaxh3_b200.ulysses import ulysses_attention

    x = torch.zeros(1, 8, 4, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        ulysses_attention(x, x, x, exchange="shared")
    with pytest.raises(ValueError):
        ulysses_attention(x, x, x, exchange="peer", head_groups=2)
    with pytest.raises(ValueError):
        ulysses_attention(x, x, x, exchange="peer", cu_seqlens=[0, 8], cross_kv=(x, x))


def test_nvtx_range_decorator_is_transparent(monkeypatch):
    """ops.nvtx pushes one range per call and pops it on return and on error."""
    from minimaxh3_b200 import ops

    calls = []
    monkeypatch.setattr(torch.cuda.nvtx, "range_push", lambda name: calls.append(("push", name)))
    monkeypatch.setattr(torch.cuda.nvtx, "range_pop", lambda: calls.append(("pop",)))

    @ops.nvtx("mh3.test")
    def f(x, y=1):
        """doc"""
        if x < 0:
            raise ValueError("negative")
        return x + y

    assert f(2, y=3) == 5 and f.__name__ == "f" and f.__doc__ == "doc"
    with pytest.raises(ValueError):
        f(-1)
    assert calls == [("push", "mh3.test"), ("pop",)] * 2
