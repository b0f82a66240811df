"""CPU restatement of the reference FP8 linear path (TEST INFRASTRUCTURE).

Follows ``kernels/fp8_linear.py`` of viragadel6/minimaxh3.  Never imported by
the shipped package.
"""
from __future__ import annotations

import torch

E4M3 = torch.float8_e4m3fn


def quantize_rows(x2d: torch.Tensor):
    """``_quantize_rows_kernel`` / ``quantize_rows`` (fp8_linear.py:8-42).

    Per-row absmax/448 scale (:20-21), clamp and e4m3 cast (:22).  Returns
    (x8 [M,K] e4m3, x_scale [M,1] f32).
    """
    xf = x2d.float()
    amax = xf.abs().amax(dim=1)                                        # :20
    scale = torch.clamp(amax, min=1.0e-12) / torch.tensor(448.0)       # :21
    x8 = torch.clamp(xf / scale[:, None], -448.0, 448.0).to(E4M3)      # :22
    return x8, scale[:, None].contiguous()


def scaled_mm_rowwise(x8, w8, x_scale, w_scale, bias=None, out_dtype=torch.bfloat16):
    """What ``torch._scaled_mm(x8, w8.t(), scale_a, scale_b, bias, bf16)`` computes.

    fp8_linear.py:95-102: ``(x8 @ w8^T) * scale_a[M,1] * scale_b[1,N] + bias``
    in fp32, one rounding to ``out_dtype``.  The e4m3 products are exact; the
    sum is taken in float64 and rounded once.
    """
    acc = torch.matmul(x8.double(), w8.double().t()).float()
    out = acc * x_scale.reshape(-1, 1).float() * w_scale.reshape(1, -1).float()
    if bias is not None:
        out = out + bias.float().reshape(1, -1)
    return out.to(out_dtype)


def apply_lora_adapters(x, out, adapters):
    """``apply_lora_adapters`` (fp8_linear.py:45-55), verbatim semantics."""
    if not adapters:
        return out
    for A, B, scale in adapters:
        branch = (x.to(A.dtype) @ A.t()) @ B.t()                       # :53
        out = out + (branch * scale).to(out.dtype)                     # :54
    return out


def fp8_linear_forward(x, w8, w_scale, bias, adapters, out_features):
    """``FP8Linear.forward`` (fp8_linear.py:87-108) on CPU tensors.

    The reference pads M to a multiple of 16 for ``_scaled_mm`` (:91-93);
    padding rows are zero and are sliced off again, so they do not change
    the result and are not reproduced here.
    """
    orig_shape = x.shape
    x2d = x.reshape(-1, x.shape[-1])
    x8, xs = quantize_rows(x2d)                                        # :94
    out = scaled_mm_rowwise(x8, w8, xs, w_scale, bias)                 # :95-102
    out = out.reshape(*orig_shape[:-1], out_features).to(x.dtype)     # :107
    return apply_lora_adapters(x, out, adapters)                       # :108


def fp8_linear_fused_oracle(x, w8, w_scale, bias, adapters):
    """float64 value of the fused epilogue this package computes.

    ``(x8 w8^T) sa sb + bias + sum_i scale_i (x A_i^T) B_i^T``, with the
    adapter product taken on the unquantised activations as the reference
    does.  Returned in float32 for tolerance checks.
    """
    x2d = x.reshape(-1, x.shape[-1])
    x8, xs = quantize_rows(x2d)
    out = torch.matmul(x8.double(), w8.double().t()) * xs.double() * w_scale.double().reshape(1, -1)
    if bias is not None:
        out = out + bias.double().reshape(1, -1)
    for A, B, scale in adapters or []:
        out = out + (x2d.double() @ A.double().t()) @ B.double().t() * float(scale)
    return out.float()
