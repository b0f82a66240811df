"""Failure detection on the GPU without a fault: bounded pipeline waits.

Every mbarrier wait of the attention and GEMM kernels gives up after
``timeout_ns`` and records MH3_DEVERR_WAIT_TIMEOUT in the caller's error
word; the CTA then drains the copies and MMAs already in flight (under a
fixed bound of its own), frees its tensor memory and returns.  The test sets
MH3_TEST_STALL_PRODUCER, which makes each CTA's load warp first wait (with
a 1 ms limit) on a barrier that nothing arrives on, and expects the error
code, a clean return (no CUDA error) and a context that still computes the
same bits on the next, normal launch.  No trap, no bad address; every wait
has its limit.
"""
import math

import pytest
import torch

from minimaxh3_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _attn_inputs():
    g = torch.Generator(device=DEV).manual_seed(9)
    B, H, S, D = 1, 8, 8192, 128
    xs = []
    for _ in range(3):
        x = torch.randn(B, H, S, D, generator=g, device=DEV)
        s = x.abs().amax(dim=(2, 3), keepdim=True) / 448.0
        xs.append(((x / s).to(torch.float8_e4m3fn), s.reshape(B, H, 1).contiguous()))
    return xs, D


def test_attention_wait_timeout_sets_error_and_context_survives():
    from minimaxh3_b200 import ops

    ((q8, sq), (k8, sk), (v8, sv)), D = _attn_inputs()
    v16 = v8.to(torch.float16)
    ls2 = math.log2(math.e) / math.sqrt(D)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    good = ops.attention_e4m3(q8, k8, v16, sq, sk, sv, logit_scale_log2=ls2, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ops.attention_e4m3(q8, k8, v16, sq, sk, sv, logit_scale_log2=ls2, err=err, timeout_ns=1_000_000,
                       test_flags=_lib.MH3_TEST_STALL_PRODUCER)
    torch.cuda.synchronize()  # a clean return: no CUDA error is raised here
    assert int(err.item()) == _lib.MH3_DEVERR_WAIT_TIMEOUT
    err.zero_()
    again = ops.attention_e4m3(q8, k8, v16, sq, sk, sv, logit_scale_log2=ls2, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(again, good)


@pytest.mark.parametrize("M,N,K", [(4096, 5120, 2048), (64, 512, 1024)])  # CTA-pair and single-CTA kernels
def test_gemm_wait_timeout_sets_error_and_context_survives(M, N, K):
    from minimaxh3_b200 import ops

    g = torch.Generator(device=DEV).manual_seed(10)
    x8, sa = ops.quantize_rows(torch.randn(M, K, generator=g, device=DEV).to(torch.bfloat16))
    w8, sb = ops.quantize_rows((torch.randn(N, K, generator=g, device=DEV) * 0.02).to(torch.bfloat16))
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    good = ops.scaled_gemm(x8, w8, row_scale=sa, col_scale=sb, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ops.scaled_gemm(x8, w8, row_scale=sa, col_scale=sb, err=err, timeout_ns=1_000_000,
                    test_flags=_lib.MH3_TEST_STALL_PRODUCER)
    torch.cuda.synchronize()
    assert int(err.item()) == _lib.MH3_DEVERR_WAIT_TIMEOUT
    err.zero_()
    again = ops.scaled_gemm(x8, w8, row_scale=sa, col_scale=sb, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(again, good)
