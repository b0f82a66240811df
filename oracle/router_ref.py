"""The reference's CPU path for the attention hot path (TEST INFRASTRUCTURE).

``kernels/attention_router.py:56-102``: ``routed_sdpa`` only takes the FP8
branch for CUDA tensors (``is_supported`` needs ``q.is_cuda``,
fp8_attention.py:19); on CPU tensors it always falls through to the torch
SDPA captured at import (``_orig_sdpa``, :17, :93-102).  This module restates
that fallback, which ``bench.py --impl reference`` times on the host cores.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

_orig_sdpa = F.scaled_dot_product_attention


def cpu_sdpa_fallback(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False, scale=None):
    """attention_router.py:93-102 on CPU tensors."""
    return _orig_sdpa(query, key, value, attn_mask=attn_mask, dropout_p=dropout_p,
                      is_causal=is_causal, scale=scale)


def fp8_emulated_inputs(q, k, v):
    """Benchmark configuration 1 variant: per-(b,h) absmax/448 e4m3 quantise-dequantise."""
    outs = []
    for x in (q, k, v):
        xf = x.float()
        s = torch.clamp(xf.abs().amax(dim=(2, 3), keepdim=True), min=1e-12) / 448.0
        outs.append(torch.clamp(xf / s, -448.0, 448.0).to(torch.float8_e4m3fn).float() * s)
    return outs
