"""Drop-in replacement for the reference's ``kernels/fp8_attention.py``.

Same public surface as viragadel6/minimaxh3 ``kernels/fp8_attention.py``:
``LOG2E`` (:9), ``is_supported(q, k, v)`` (:12-36) and
``fp8_attention(q, k, v, scale=None, key_mask=None, key_bias=None,
repair_tau=-1.0)`` (:300-403).  The work runs in libmh3_b200 (sm_100a):

1. ``mh3_quantize_qkv`` - Q scaled by softmax_scale*log2(e) and quantised
   per 128-row block, K centred on its channel mean and quantised per
   128-key block, V quantised per channel (the reference's granularity,
   :39-170, :338), V kept in [key, channel] order;
2. ``mh3_fp8_attention_fwd`` - tcgen05 FP8 flash attention with exact exp2
   softmax (see minimaxh3_b200/csrc/attn_fwd.cu).

The QK^T product is e4m3 x e4m3.  The PV product runs on f16 P and f16
V/scale_v by default (``MH3_PV_DTYPE=f16``): with P rounded to e4m3 (3
mantissa bits) the max-abs error on peaked rows exceeds the 2e-2 tolerance
for the outlier-channel distribution.  ``MH3_PV_DTYPE=e4m3`` selects the
e4m3 PV product (V quantised per channel to e4m3, as the reference does).

``repair_tau`` is accepted for signature compatibility.  The reference's
repair pass (:288-292) corrects its piecewise-linear P toward the exact
exponential; this kernel already computes P from the exact exponential
(rounded once to e4m3), so the argument does not change the result.

The op is registered as ``torch.ops.mh3.fp8_attention`` with a fake
(meta) implementation, so ``torch.compile``d blocks trace through it
without a graph break.

``fp8_attention_varlen`` is this package's route for packed
variable-length batches (video tokens followed by audio tokens per
sample, ``cu_seqlens`` as in flash-attention's varlen interface), which the
reference does not have: per-(sequence, head) absmax/448 scales for Q, K
and V (``mh3_absmax_seg`` + ``mh3_quantize_seg``), then the same kernel
over the packed tensors (op ``torch.ops.mh3.fp8_attention_varlen``).
"""
from __future__ import annotations

import math

import torch

import os

from .. import ops as _ops

LOG2E = 1.4426950408889634


def _pv_dtype() -> torch.dtype:
    mode = os.environ.get("MH3_PV_DTYPE", "f16").strip().lower()
    if mode in ("e4m3", "fp8"):
        return torch.float8_e4m3fn
    if mode in ("f16", "fp16", "half", ""):
        return torch.float16
    raise ValueError(f"MH3_PV_DTYPE must be f16 or e4m3, got {mode!r}")


def _device_is_sm100(device: torch.device) -> bool:
    return torch.cuda.get_device_capability(device) == (10, 0)


def is_supported(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> bool:
    """Whether ``fp8_attention`` accepts these inputs (fp8_attention.py:12-36).

    Same conditions as the reference: CUDA tensors on one device, 4-D,
    bf16/fp16 of one dtype, head dim 64 or 128 on all three, equal batch and
    head counts, Sk == Sv > 0 and Sq > 0.  The device test is sm_100 (the
    library is built for sm_100a only) where the reference asks cc >= 8.9.
    """
    if not (isinstance(q, torch.Tensor) and isinstance(k, torch.Tensor) and isinstance(v, torch.Tensor)):
        return False
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        return False
    if q.device != k.device or q.device != v.device:
        return False
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        return False
    if q.dtype not in (torch.bfloat16, torch.float16):
        return False
    if k.dtype != q.dtype or v.dtype != q.dtype:
        return False
    d = q.shape[-1]
    if d not in (64, 128) or k.shape[-1] != d or v.shape[-1] != d:
        return False
    if q.shape[:2] != k.shape[:2] or q.shape[:2] != v.shape[:2]:
        return False
    if k.shape[2] != v.shape[2] or q.shape[2] == 0 or k.shape[2] == 0:
        return False
    return _device_is_sm100(q.device)


@_ops.nvtx("mh3.fp8_attention")
def _fp8_attention_impl(q, k, v, scale, key_mask, key_bias, repair_tau):
    B, H, Sq, D = q.shape
    Sk = k.shape[2]
    c = (scale if scale is not None else 1.0 / math.sqrt(D)) * LOG2E
    q8, k8, v8, sq, sk, sv, _ = _ops.quantize_qkv(q, k, v, c, v_dtype=_pv_dtype())
    bias2 = kv_len = None
    if key_mask is not None or key_bias is not None:
        # one launch; padded batches: the tiles past each batch's last valid key are skipped
        bias2, kv_len = _ops.key_bias_inputs(key_mask, key_bias, B, Sk, q.device)
    # Same strides as the reference's ``torch.empty_like(q)`` (:379); the
    # kernel writes through the strides, so transposed views stay correct.
    out = torch.empty_like(q)
    if out.stride(-1) != 1 or any(s % 8 for s in out.stride()[:3]):
        out = torch.empty((B, H, Sq, D), dtype=q.dtype, device=q.device)
    return _ops.attention_e4m3(q8, k8, v8, sq, sk, sv, logit_scale_log2=1.0, out_dtype=q.dtype,
                               key_bias2=bias2, out=out, kv_len=kv_len)


@torch.library.custom_op("mh3::fp8_attention", mutates_args=())
def _fp8_attention_op(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                      key_mask: torch.Tensor | None, key_bias: torch.Tensor | None,
                      repair_tau: float) -> torch.Tensor:
    return _fp8_attention_impl(q, k, v, None if math.isnan(scale) else scale, key_mask, key_bias, repair_tau)


@_fp8_attention_op.register_fake
def _(q, k, v, scale, key_mask, key_bias, repair_tau):
    return torch.empty_like(q)


def fp8_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    scale: float | None = None,
    key_mask: torch.Tensor | None = None,
    key_bias: torch.Tensor | None = None,
    repair_tau: float = -1.0,
) -> torch.Tensor:
    """Non-causal FP8 attention, output in q's dtype and shape [B,H,Sq,D]."""
    if not is_supported(q, k, v):
        raise ValueError("Unsupported inputs for fp8_attention")
    return torch.ops.mh3.fp8_attention(q, k, v, math.nan if scale is None else float(scale),
                                       key_mask, key_bias, float(repair_tau))


def _check_varlen(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q):
    for name, t in (("q", q), ("k", k), ("v", v)):
        if not isinstance(t, torch.Tensor) or not t.is_cuda or t.dim() != 3:
            raise ValueError(f"{name} must be a CUDA tensor [tokens, heads, head_dim]")
    if q.dtype not in (torch.bfloat16, torch.float16) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("q, k, v must share one dtype, bf16 or f16")
    if q.device != k.device or q.device != v.device:
        raise ValueError("q, k, v must be on one device")
    D = q.shape[2]
    if D not in (64, 128) or k.shape[1:] != q.shape[1:] or v.shape != k.shape:
        raise ValueError("q [Tq,H,D], k and v [Tk,H,D] with D 64 or 128")
    for name, c in (("cu_seqlens_q", cu_seqlens_q), ("cu_seqlens_k", cu_seqlens_k)):
        if not isinstance(c, torch.Tensor) or c.dtype != torch.int32 or c.dim() != 1 or c.device != q.device:
            raise ValueError(f"{name} must be an int32 tensor [nseq+1] on q's device")
    if cu_seqlens_q.numel() != cu_seqlens_k.numel() or cu_seqlens_q.numel() < 2:
        raise ValueError("cu_seqlens_q and cu_seqlens_k must both hold nseq+1 >= 2 offsets")
    if int(max_seqlen_q) <= 0:
        raise ValueError("max_seqlen_q must be positive")
    if not _device_is_sm100(q.device):
        raise ValueError("fp8_attention_varlen needs an sm_100 device")


def _per_segment_scales(x, cu):
    return _ops.scale_from_absmax(_ops.absmax_seg(x, cu))                  # [nseq, H]


@_ops.nvtx("mh3.fp8_attention_varlen")
def _fp8_attention_varlen_impl(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, scale):
    D = q.shape[2]
    ls2 = (scale if scale is not None else 1.0 / math.sqrt(D)) * LOG2E
    cq, ck = cu_seqlens_q.contiguous(), cu_seqlens_k.contiguous()
    sq, sk, sv = _per_segment_scales(q, cq), _per_segment_scales(k, ck), _per_segment_scales(v, ck)
    q8 = _ops.quantize_seg(q, cq, sq, torch.float8_e4m3fn)[0, 0]
    k8 = _ops.quantize_seg(k, ck, sk, torch.float8_e4m3fn)[0, 0]
    v8 = _ops.quantize_seg(v, ck, sv, _pv_dtype())[0, 0]
    out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    return _ops.attention_e4m3(q8, k8, v8, sq[..., None], sk[..., None], sv[..., None], logit_scale_log2=ls2,
                               out_dtype=q.dtype, cu_seqlens_q=cq, cu_seqlens_k=ck,
                               max_seqlen_q=int(max_seqlen_q), out=out)


@torch.library.custom_op("mh3::fp8_attention_varlen", mutates_args=())
def _fp8_attention_varlen_op(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens_q: torch.Tensor,
                             cu_seqlens_k: torch.Tensor, max_seqlen_q: int, scale: float) -> torch.Tensor:
    return _fp8_attention_varlen_impl(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
                                      None if math.isnan(scale) else scale)


@_fp8_attention_varlen_op.register_fake
def _(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, scale):
    return torch.empty(q.shape, dtype=q.dtype, device=q.device)


def fp8_attention_varlen(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    cu_seqlens_q: torch.Tensor,
    cu_seqlens_k: torch.Tensor,
    max_seqlen_q: int,
    scale: float | None = None,
) -> torch.Tensor:
    """Non-causal FP8 attention over packed sequences.

    q [Tq, H, D], k and v [Tk, H, D] (bf16 or f16, D 64 or 128); sequence i
    is query rows ``[cu_seqlens_q[i], cu_seqlens_q[i+1])`` attending over key
    rows ``[cu_seqlens_k[i], cu_seqlens_k[i+1])`` (int32 offsets on q's
    device, non-decreasing); ``max_seqlen_q`` bounds the query lengths.
    Quantisation is per (sequence, head): absmax/448 for Q, K and V (V as f16
    V/scale for the f16 PV product unless ``MH3_PV_DTYPE=e4m3``).  Returns
    [Tq, H, D] in q's dtype; rows outside every sequence are not written
    (their values are unspecified).  ``scale`` defaults to 1/sqrt(D).
    """
    _check_varlen(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q)
    return torch.ops.mh3.fp8_attention_varlen(q, k, v, cu_seqlens_q, cu_seqlens_k, int(max_seqlen_q),
                                              math.nan if scale is None else float(scale))
