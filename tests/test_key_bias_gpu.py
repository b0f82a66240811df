"""``mh3_key_bias``: the drop-in path's per-key mask / bias in the kernel's form.

The CPU test pins the oracle's restatement of the reference rule
(kernels/fp8_attention.py:256-262) on a hand-checked case; the GPU tests
require the kernel's ``bias2`` and ``kv_len`` to equal the oracle's bit for
bit over masks, biases, broadcast rows, fully masked rows and ragged tails.
"""
import math

import pytest
import torch

from oracle import fp8_attention_ref as OA

DEV = "cuda"


def test_oracle_key_bias_rule_known_answer():
    mask = torch.tensor([[True, False, True, True, False]])
    bias = torch.tensor([[0.5, 2.0, -2.0e8, -1.0, 3.0]])
    bias2, kv_len = OA.key_bias2_ref(mask, bias, 2, 5, tile=8)
    l2e = torch.tensor(OA.LOG2E, dtype=torch.float32)
    inf = -math.inf
    want = torch.tensor([float(0.5 * l2e), inf, inf, float(-1.0 * l2e), inf, inf, inf, inf])
    assert torch.equal(bias2, want[None].expand(2, 8))
    assert kv_len.tolist() == [4, 4]
    _, kv_none = OA.key_bias2_ref(torch.zeros(1, 5, dtype=torch.bool), None, 1, 5)
    assert kv_none.tolist() == [0]
    b_only, kv_b = OA.key_bias2_ref(None, None, 1, 3, tile=4)
    assert b_only.tolist() == [[0.0, 0.0, 0.0, inf]] and kv_b.tolist() == [3]


def _case(seed, B, Sk, mask_rows, bias_rows):
    g = torch.Generator().manual_seed(seed)
    mask = bias = None
    if mask_rows:
        mask = torch.rand(mask_rows, Sk, generator=g) > 0.3
        if mask_rows == B and B > 1:
            mask[-1] = False                 # a batch with every key masked
            mask[0, Sk // 2:] = False        # a padded batch: valid keys are a prefix
    if bias_rows:
        bias = 4.0 * torch.randn(bias_rows, Sk, generator=g)
        bias[:, ::7] = -1.0e9                # masked through the bias
        bias[:, 3::11] = -1.0e8              # exactly the threshold: masked (not > -1e8)
    return mask, bias


@pytest.mark.gpu
@pytest.mark.parametrize("B,Sk,mask_rows,bias_rows", [
    (1, 1, 1, 0), (2, 127, 2, 0), (2, 128, 0, 2), (3, 333, 3, 3), (3, 1000, 1, 3),
    (4, 4096, 4, 1), (2, 75600, 2, 2), (5, 257, 0, 1),
])
def test_key_bias_kernel_equals_oracle(B, Sk, mask_rows, bias_rows):
    from minimaxh3_b200 import ops

    mask, bias = _case(B * 1000 + Sk, B, Sk, mask_rows, bias_rows)
    if mask is not None and mask_rows == 1 and B > 1:
        mask = mask[0]                       # a [Sk] mask broadcast over the batch
    bias2, kv_len = ops.key_bias_inputs(None if mask is None else mask.to(DEV),
                                        None if bias is None else bias.to(DEV), B, Sk, DEV)
    want_b, want_l = OA.key_bias2_ref(mask, bias, B, Sk)
    torch.cuda.synchronize()
    assert bias2.shape == want_b.shape
    assert torch.equal(bias2.cpu().view(torch.int32), want_b.view(torch.int32))
    assert torch.equal(kv_len.cpu(), want_l)


@pytest.mark.gpu
def test_key_bias_kernel_reads_strided_rows_and_other_dtypes():
    """A bf16 bias and a float mask, taken from wider tensors (row stride > Sk)."""
    from minimaxh3_b200 import ops

    B, Sk = 3, 500
    g = torch.Generator().manual_seed(5)
    wide_bias = torch.randn(B, Sk + 40, generator=g).to(torch.bfloat16)
    wide_mask = (torch.rand(B, Sk + 40, generator=g) > 0.5).float()
    bias, mask = wide_bias[:, :Sk], wide_mask[:, 20:20 + Sk]
    bias2, kv_len = ops.key_bias_inputs(mask.to(DEV), bias.to(DEV), B, Sk, DEV)
    want_b, want_l = OA.key_bias2_ref(mask, bias, B, Sk)
    assert torch.equal(bias2.cpu().view(torch.int32), want_b.view(torch.int32))
    assert torch.equal(kv_len.cpu(), want_l)


def test_key_bias_wrapper_rejects_bad_shapes():
    from minimaxh3_b200 import ops

    with pytest.raises(ValueError, match="key_mask"):
        ops.key_bias_inputs(torch.ones(2, 7, dtype=torch.bool), None, 2, 8, "cpu")
    with pytest.raises(ValueError, match="key_bias"):
        ops.key_bias_inputs(None, torch.ones(3, 8), 2, 8, "cpu")
