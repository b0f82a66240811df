"""torch-facing wrappers over the C ABI (include/mh3_b200.h).

Tensors are passed to the library as raw device pointers plus element
strides; outputs are allocated here with torch's caching allocator on the
current stream, as the reference's wrappers do (kernels/fp8_attention.py:
321-379, kernels/fp8_linear.py:34-35).  No host synchronisation happens on
these paths.
"""
from __future__ import annotations

import collections
import functools

import torch

from . import _lib

LOG2E = 1.4426950408889634
BLOCK = 128
E4M3 = torch.float8_e4m3fn


def nvtx(name: str):
    """Decorator: an NVTX range named ``name`` around a composite op (its C
    entry points push their own ranges inside), for profilers that filter or
    group by NVTX (ncu --nvtx).  A push/pop costs well under a microsecond
    when no tool is attached."""

    def wrap(fn):
        @functools.wraps(fn)
        def run(*args, **kwargs):
            torch.cuda.nvtx.range_push(name)
            try:
                return fn(*args, **kwargs)
            finally:
                torch.cuda.nvtx.range_pop()

        return run

    return wrap


def _cdiv(a: int, b: int) -> int:
    return (a + b - 1) // b


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _dtype_code(dt: torch.dtype) -> int:
    if dt == torch.bfloat16:
        return _lib.MH3_DTYPE_BF16
    if dt == torch.float16:
        return _lib.MH3_DTYPE_F16
    raise ValueError(f"unsupported dtype {dt} (bf16 or fp16)")


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("expected CUDA tensors")


def _scale_strides(s: torch.Tensor, nblk_full: int):
    """Strides (b, h, blk) of a [B,H,nblk] or [B,H,1] / [B,H] scale tensor."""
    if s.dtype != torch.float32:
        raise ValueError("scales must be float32")
    if s.dim() == 2:
        return s.stride(0), s.stride(1), 0
    if s.dim() != 3:
        raise ValueError("scale tensors must be [B,H] or [B,H,n]")
    if s.shape[2] == 1:
        return s.stride(0), s.stride(1), 0
    if s.shape[2] < nblk_full:
        raise ValueError(f"scale has {s.shape[2]} blocks, need {nblk_full}")
    return s.stride(0), s.stride(1), s.stride(2)


def device_error_word(device=None) -> torch.Tensor:
    """The library's device error word for ``device`` as a 1-element int32 view."""
    lib = _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        addr = lib.mh3_device_error_word()
    if not addr:
        raise _lib.Mh3Error("could not resolve the device error word")
    return _wrap_device_int(addr, dev)


def _wrap_device_int(addr: int, dev: torch.device) -> torch.Tensor:
    # A zero-copy int32 view of library-owned device memory.
    class _Holder:
        __cuda_array_interface__ = {"shape": (1,), "typestr": "<i4", "data": (addr, False), "version": 3}

    with torch.cuda.device(dev):
        return torch.as_tensor(_Holder(), device=dev)


def read_and_clear_device_error(device=None) -> int:
    """Synchronise ``device``, return its error word and reset it to 0 (testing/debug)."""
    w = device_error_word(device)
    torch.cuda.synchronize(w.device)
    val = int(w.item())
    w.zero_()
    return val


# ---------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------


def attention_e4m3(
    q8: torch.Tensor,
    k8: torch.Tensor,
    v8: torch.Tensor,
    scale_q: torch.Tensor,
    scale_k: torch.Tensor,
    scale_v: torch.Tensor,
    logit_scale_log2: float = 1.0,
    out_dtype: torch.dtype = torch.bfloat16,
    key_bias2: torch.Tensor | None = None,
    cu_seqlens_q: torch.Tensor | None = None,
    cu_seqlens_k: torch.Tensor | None = None,
    max_seqlen_q: int = 0,
    out: torch.Tensor | None = None,
    err: torch.Tensor | None = None,
    timeout_ns: int = 0,
    kv_len: torch.Tensor | None = None,
    test_flags: int = 0,
) -> torch.Tensor:
    """Non-causal FP8 attention (``mh3_fp8_attention_fwd``).

    Dense: q8 [B,H,Sq,D], k8/v8 [B,H,Sk,D] e4m3 (channels contiguous, any
    other strides that are multiples of 16).  ``v8`` may instead be float16
    (V already divided by scale_v): the PV product then runs on f16 P and V
    instead of e4m3.  Varlen (``cu_seqlens_*`` int32
    [nseq+1] on the device): q8 [Tq,H,D], k8/v8 [Tk,H,D].  scale_q/scale_k
    [B,H,nblk] per 128-row block, or [B,H,1] / [B,H] per (batch, head);
    scale_v [B,H,D] or [B,H,1].  ``logit_scale_log2`` multiplies q.k (log2
    units: softmax_scale * log2(e) when the scales do not already carry it).
    ``key_bias2`` [B, ceil(Sk/128)*128] f32 additive log2 bias (-inf = masked,
    and for the padding).
    """
    lib = _lib.load()
    _require_cuda(q8, k8, v8, scale_q, scale_k, scale_v, key_bias2)
    for t in (q8, k8):
        if t.dtype != E4M3:
            raise ValueError("q8/k8 must be float8_e4m3fn")
    if v8.dtype not in (E4M3, torch.float16):
        raise ValueError("v8 must be float8_e4m3fn or float16")
    for t in (q8, k8, v8):
        if t.stride(-1) != 1:
            raise ValueError("q8/k8/v8 need a contiguous last dimension")
    varlen = cu_seqlens_q is not None or cu_seqlens_k is not None
    a = _lib.AttnArgs()
    if varlen:
        if cu_seqlens_q is None or cu_seqlens_k is None:
            raise ValueError("varlen needs cu_seqlens_q and cu_seqlens_k")
        if q8.dim() != 3 or k8.dim() != 3 or v8.dim() != 3:
            raise ValueError("varlen q8/k8/v8 are [tokens, H, D]")
        if cu_seqlens_q.dtype != torch.int32 or cu_seqlens_k.dtype != torch.int32:
            raise ValueError("cu_seqlens must be int32")
        Tq, H, D = q8.shape
        Tk = k8.shape[0]
        B = cu_seqlens_q.numel() - 1
        if max_seqlen_q <= 0:
            raise ValueError("varlen needs max_seqlen_q")
        Sq, Sk = int(max_seqlen_q), 0
        a.q_stride_b, a.q_stride_h, a.q_stride_s = 0, q8.stride(1), q8.stride(0)
        a.k_stride_b, a.k_stride_h, a.k_stride_s = 0, k8.stride(1), k8.stride(0)
        a.v_stride_b, a.v_stride_h, a.v_stride_s = 0, v8.stride(1), v8.stride(0)
        a.total_q, a.total_k = Tq, Tk
        a.cu_seqlens_q = cu_seqlens_q.data_ptr()
        a.cu_seqlens_k = cu_seqlens_k.data_ptr()
        a.max_seqlen_q = int(max_seqlen_q)
        if out is None:
            out = torch.empty((Tq, H, D), dtype=out_dtype, device=q8.device)
        a.o_stride_b, a.o_stride_h, a.o_stride_s = 0, out.stride(1), out.stride(0)
        nq_full = nk_full = 1
    else:
        if q8.dim() != 4 or k8.dim() != 4 or v8.dim() != 4:
            raise ValueError("q8/k8/v8 are [B,H,S,D]")
        B, H, Sq, D = q8.shape
        Sk = k8.shape[2]
        if k8.shape[:2] != (B, H) or v8.shape[:3] != k8.shape[:3] or k8.shape[3] != D or v8.shape[3] != D:
            raise ValueError("q8/k8/v8 shapes disagree")
        a.q_stride_b, a.q_stride_h, a.q_stride_s = q8.stride(0), q8.stride(1), q8.stride(2)
        a.k_stride_b, a.k_stride_h, a.k_stride_s = k8.stride(0), k8.stride(1), k8.stride(2)
        a.v_stride_b, a.v_stride_h, a.v_stride_s = v8.stride(0), v8.stride(1), v8.stride(2)
        if out is None:
            out = torch.empty((B, H, Sq, D), dtype=out_dtype, device=q8.device)
        a.o_stride_b, a.o_stride_h, a.o_stride_s = out.stride(0), out.stride(1), out.stride(2)
        nq_full, nk_full = _cdiv(Sq, BLOCK), _cdiv(Sk, BLOCK)
    if out.stride(-1) != 1 or out.dtype != out_dtype:
        raise ValueError("out must have a contiguous last dim and dtype out_dtype")
    a.batch, a.heads, a.seqlen_q, a.seqlen_k, a.head_dim = B, H, Sq, Sk, D
    a.out_dtype = _dtype_code(out_dtype)
    a.v_dtype = _lib.MH3_DTYPE_F16 if v8.dtype == torch.float16 else _lib.MH3_DTYPE_E4M3
    a.q8, a.k8, a.v8, a.out = q8.data_ptr(), k8.data_ptr(), v8.data_ptr(), out.data_ptr()
    a.scale_q = scale_q.data_ptr()
    a.sq_stride_b, a.sq_stride_h, a.sq_stride_blk = _scale_strides(scale_q, nq_full if not varlen else 1)
    a.scale_k = scale_k.data_ptr()
    a.sk_stride_b, a.sk_stride_h, a.sk_stride_blk = _scale_strides(scale_k, nk_full if not varlen else 1)
    if scale_v.dtype != torch.float32 or scale_v.dim() != 3:
        raise ValueError("scale_v must be float32 [B,H,D] or [B,H,1]")
    a.scale_v = scale_v.data_ptr()
    a.sv_stride_b, a.sv_stride_h = scale_v.stride(0), scale_v.stride(1)
    a.sv_stride_d = scale_v.stride(2) if scale_v.shape[2] != 1 else 0
    a.logit_scale_log2 = float(logit_scale_log2)
    if key_bias2 is not None:
        if key_bias2.dtype != torch.float32 or key_bias2.dim() != 2 or key_bias2.stride(1) != 1:
            raise ValueError("key_bias2 must be float32 [B, n*128] with contiguous rows")
        a.key_bias2 = key_bias2.data_ptr()
        a.key_bias2_stride_b = key_bias2.stride(0)
    if err is not None:
        a.err = err.data_ptr()
    a.timeout_ns = int(timeout_ns)
    a.test_flags = int(test_flags)
    if kv_len is not None:
        if kv_len.dtype != torch.int32 or kv_len.numel() < a.batch or not kv_len.is_cuda:
            raise ValueError("kv_len must be a CUDA int32 tensor with one entry per batch")
        kv_len = kv_len.contiguous()
        a.kv_len = kv_len.data_ptr()
    with torch.cuda.device(q8.device):
        rc = lib.mh3_fp8_attention_fwd(a, _stream(q8.device))
    _lib.check(rc, "mh3_fp8_attention_fwd")
    return out


def _per_key_rows(t, B: int, Sk: int, dtype, device, what: str):
    """A per-key input as (tensor with contiguous keys, batch stride): shapes
    [Sk], [1, Sk] (one row for every batch, stride 0) or [B, Sk]."""
    t = t.to(device=device, dtype=dtype)
    if t.dim() == 1:
        t = t.unsqueeze(0)
    if t.dim() != 2 or t.shape[1] != Sk or t.shape[0] not in (1, B):
        raise ValueError(f"{what} must be [B, Sk], [1, Sk] or [Sk] with Sk = {Sk}")
    if t.stride(1) != 1:
        t = t.contiguous()
    return t, (t.stride(0) if t.shape[0] == B and B > 1 else 0)


def key_bias_inputs(key_mask, key_bias, B: int, Sk: int, device):
    """The drop-in path's per-key inputs in the attention kernel's form, one
    launch (``mh3_key_bias``): ``(bias2, kv_len)`` with bias2 an fp32
    ``[B, ceil(Sk/128)*128]`` additive log2 bias (``key_bias * log2(e)`` for a
    valid key, ``-inf`` for a masked one and for the padding; the reference's
    rule, fp8_attention.py:256-264: a key is valid when its mask is true and
    its bias is above -1e8) and kv_len an int32 ``[B]``, one past the last
    valid key, past which the kernel skips whole tiles."""
    lib = _lib.load()
    mask_ptr = bias_ptr = 0
    msb = bsb = 0
    if key_mask is not None:
        m, msb = _per_key_rows(key_mask, B, Sk, torch.bool, device, "key_mask")
        mask_ptr = m.data_ptr()
    if key_bias is not None:
        kb, bsb = _per_key_rows(key_bias, B, Sk, torch.float32, device, "key_bias")
        bias_ptr = kb.data_ptr()
    bias2 = torch.empty((B, _cdiv(Sk, BLOCK) * BLOCK), dtype=torch.float32, device=device)
    kv_len = torch.empty((B,), dtype=torch.int32, device=device)
    with torch.cuda.device(bias2.device):
        rc = lib.mh3_key_bias(mask_ptr or None, msb, bias_ptr or None, bsb, B, Sk, bias2.data_ptr(),
                              bias2.stride(0), kv_len.data_ptr(), _stream(bias2.device))
    _lib.check(rc, "mh3_key_bias")
    return bias2, kv_len


# ---------------------------------------------------------------------------
# quantisation
# ---------------------------------------------------------------------------


def quantize_qkv(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_premul: float,
                 v_dtype: torch.dtype = E4M3):
    """Q/K/V e4m3 quantisation of the drop-in path (``mh3_quantize_qkv``).

    Returns (q8, k8, v8, scale_q, scale_k, scale_v, k_mean): q8 [B,H,Sq,D],
    k8/v8 [B,H,Sk,D] contiguous e4m3; scale_q [B,H,ceil(Sq/128)],
    scale_k [B,H,ceil(Sk/128)], scale_v / k_mean [B,H,D] float32.
    ``v_dtype=torch.float16`` returns v/scale_v in f16 instead of e4m3.
    """
    lib = _lib.load()
    _require_cuda(q, k, v)
    B, H, Sq, D = q.shape
    Sk = k.shape[2]
    dev = q.device
    tensors = []
    for t in (q, k, v):
        if t.stride(-1) != 1 or any(s % 8 for s in t.stride()[:3]) or t.data_ptr() % 16:
            t = t.contiguous()
        tensors.append(t)
    q, k, v = tensors
    q8 = torch.empty((B, H, Sq, D), dtype=E4M3, device=dev)
    k8 = torch.empty((B, H, Sk, D), dtype=E4M3, device=dev)
    if v_dtype not in (E4M3, torch.float16):
        raise ValueError("v_dtype must be float8_e4m3fn or float16")
    v8 = torch.empty((B, H, Sk, D), dtype=v_dtype, device=dev)
    sq = torch.empty((B, H, _cdiv(Sq, BLOCK)), dtype=torch.float32, device=dev)
    sk = torch.empty((B, H, _cdiv(Sk, BLOCK)), dtype=torch.float32, device=dev)
    sv = torch.empty((B, H, D), dtype=torch.float32, device=dev)
    kmean = torch.empty((B, H, D), dtype=torch.float32, device=dev)
    ws_bytes = int(lib.mh3_qkv_workspace_bytes(B, H, Sk, D))
    ws = torch.empty((max(ws_bytes, 16),), dtype=torch.uint8, device=dev)
    a = _lib.QkvQuantArgs()
    a.batch, a.heads, a.seqlen_q, a.seqlen_k, a.head_dim = B, H, Sq, Sk, D
    a.in_dtype = _dtype_code(q.dtype)
    a.q, a.q_stride_b, a.q_stride_h, a.q_stride_s = q.data_ptr(), q.stride(0), q.stride(1), q.stride(2)
    a.k, a.k_stride_b, a.k_stride_h, a.k_stride_s = k.data_ptr(), k.stride(0), k.stride(1), k.stride(2)
    a.v, a.v_stride_b, a.v_stride_h, a.v_stride_s = v.data_ptr(), v.stride(0), v.stride(1), v.stride(2)
    a.q_premul = float(q_premul)
    a.v_out_dtype = _lib.MH3_DTYPE_F16 if v_dtype == torch.float16 else _lib.MH3_DTYPE_E4M3
    a.q8, a.k8, a.v8 = q8.data_ptr(), k8.data_ptr(), v8.data_ptr()
    a.scale_q, a.scale_k, a.scale_v, a.k_mean = sq.data_ptr(), sk.data_ptr(), sv.data_ptr(), kmean.data_ptr()
    a.workspace = ws.data_ptr()
    with torch.cuda.device(dev):
        rc = lib.mh3_quantize_qkv(a, _stream(dev))
    _lib.check(rc, "mh3_quantize_qkv")
    return q8, k8, v8, sq, sk, sv, kmean


def quantize_rows(x2d: torch.Tensor):
    """Per-row e4m3 quantisation (``mh3_quantize_rows``): (x8 [M,K], scale [M,1]).

    x2d: bf16, f16 or f32 [M,K] on the device."""
    lib = _lib.load()
    if x2d.dim() != 2 or not x2d.is_cuda:
        raise ValueError("quantize_rows expects a 2D CUDA tensor")
    if x2d.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        raise ValueError(f"quantize_rows: unsupported dtype {x2d.dtype} (bf16, f16 or f32)")
    if x2d.stride(1) != 1 or x2d.stride(0) % 8 or x2d.data_ptr() % 16:
        x2d = x2d.contiguous()
    M, K = x2d.shape
    x8 = torch.empty((M, K), dtype=E4M3, device=x2d.device)
    scale = torch.empty((M, 1), dtype=torch.float32, device=x2d.device)
    if M > 0 and K > 0:
        with torch.cuda.device(x2d.device):
            code = _lib.MH3_DTYPE_F32 if x2d.dtype == torch.float32 else _dtype_code(x2d.dtype)
            rc = lib.mh3_quantize_rows(x2d.data_ptr(), x2d.stride(0), code, M, K,
                                       x8.data_ptr(), scale.data_ptr(), _stream(x2d.device))
        _lib.check(rc, "mh3_quantize_rows")
    return x8, scale


def widen_e4m3_to_f16(x8: torch.Tensor) -> torch.Tensor:
    """Exact e4m3 -> float16 copy of a contiguous tensor (``mh3_widen_e4m3_to_f16``)."""
    lib = _lib.load()
    if x8.dtype != E4M3 or not x8.is_cuda:
        raise ValueError("expected a CUDA float8_e4m3fn tensor")
    x8 = x8.contiguous()
    out = torch.empty(x8.shape, dtype=torch.float16, device=x8.device)
    n = x8.numel()
    if n % 16:
        raise ValueError("widen_e4m3_to_f16 needs a multiple of 16 elements")
    if x8.data_ptr() % 16:
        x8 = x8.clone()  # fresh allocations are 16-byte aligned
    with torch.cuda.device(x8.device):
        rc = lib.mh3_widen_e4m3_to_f16(x8.data_ptr(), out.data_ptr(), n, _stream(x8.device))
    _lib.check(rc, "mh3_widen_e4m3_to_f16")
    return out


def _bh_args(x: torch.Tensor):
    if not x.is_cuda or x.dim() != 4 or x.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("expected a CUDA bf16/f16 tensor [B, S, H, D]")
    if x.stride(-1) != 1 or x.data_ptr() % 16 or any(st % 8 for st in x.stride()[:3]):
        x = x.contiguous()
    B, S, H, D = x.shape
    return x, (x.data_ptr(), _dtype_code(x.dtype), B, S, H, D, x.stride(0), x.stride(1), x.stride(2))


def _head_sel(H: int, groups: int, head_off: int, heads_sel: int | None):
    if groups <= 0 or H % groups:
        raise ValueError("groups must divide the head count")
    hb = H // groups
    hs = hb - head_off if heads_sel is None else heads_sel
    if head_off < 0 or hs <= 0 or head_off + hs > hb:
        raise ValueError("bad head selection")
    return hb, head_off, hs


def absmax_bh(x: torch.Tensor, groups: int = 1, head_off: int = 0, heads_sel: int | None = None) -> torch.Tensor:
    """max |x[b, :, h, :]| as float32 [B, groups*heads_sel] for x [B, S, H, D] over the selected
    heads h = p*(H/groups) + head_off + i (``mh3_absmax_bh``; default: all heads, [B, H])."""
    lib = _lib.load()
    x, args = _bh_args(x)
    hb, off, hs = _head_sel(x.shape[2], groups, head_off, heads_sel)
    out = torch.empty((x.shape[0], groups * hs), dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        rc = lib.mh3_absmax_bh(*args, hb, off, hs, out.data_ptr(), _stream(x.device))
    _lib.check(rc, "mh3_absmax_bh")
    return out


def quantize_bh(x: torch.Tensor, scale: torch.Tensor, out_dtype: torch.dtype = E4M3, groups: int = 1,
                out: torch.Tensor | None = None, head_off: int = 0, heads_sel: int | None = None) -> torch.Tensor:
    """x [B,S,H,D] / scale[b, j] -> e4m3 (clamped to +-448) or f16, as [groups, B, S, heads_sel, D]
    for the selected heads h = p*(H/groups) + head_off + i, numbered j = p*heads_sel + i
    (``mh3_quantize_bh``; default: all heads, scale [B, H], out [groups, B, S, H/groups, D])."""
    lib = _lib.load()
    x, args = _bh_args(x)
    B, S, H, D = x.shape
    if out_dtype not in (E4M3, torch.float16):
        raise ValueError("out_dtype must be float8_e4m3fn or float16")
    hb, off, hs = _head_sel(H, groups, head_off, heads_sel)
    scale = scale.to(device=x.device, dtype=torch.float32).contiguous()
    if scale.numel() != B * groups * hs:
        raise ValueError("scale must hold one value per (batch, selected head)")
    shape = (groups, B, S, hs, D)
    if out is None:
        out = torch.empty(shape, dtype=out_dtype, device=x.device)
    elif tuple(out.shape) != shape or out.dtype != out_dtype or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous {out_dtype} tensor of shape {shape}")
    code = _lib.MH3_DTYPE_F16 if out_dtype == torch.float16 else _lib.MH3_DTYPE_E4M3
    with torch.cuda.device(x.device):
        rc = lib.mh3_quantize_bh(*args, hb, off, hs, scale.data_ptr(), code, out.data_ptr(), _stream(x.device))
    _lib.check(rc, "mh3_quantize_bh")
    return out


def scale_from_absmax(amax: torch.Tensor) -> torch.Tensor:
    """Per-(batch or sequence, head) e4m3 scale ``max(amax, 1e-12) / 448`` as float32, rounded
    correctly (the IEEE quotient, as the library's own kernels compute it) on any device.

    ``tensor / 448.0`` would not do on CUDA: torch multiplies by the rounded reciprocal of a
    Python-scalar divisor, which misses the quotient by one ulp for some values, and a scale one
    ulp off moves elements across e4m3 rounding boundaries.  The quotient is taken in float64 and
    rounded once to float32; for the divisor 448 = 7 * 2^6 that is always the correctly rounded
    float32 quotient (a float32 divided by 7 is never within a float64 error of a float32
    rounding midpoint)."""
    a = torch.clamp(amax.to(torch.float32), min=1e-12)
    return (a.to(torch.float64) / 448.0).to(torch.float32)


def _seg_args(x: torch.Tensor, seg: torch.Tensor):
    """Packed x [S, H, D] or [1, S, H, D] and int32 segment bounds [nseg+1] on x's device."""
    if x.dim() == 4:
        if x.shape[0] != 1:
            raise ValueError("a packed shard has batch 1: [1, S, H, D] or [S, H, D]")
        x = x[0]
    if not x.is_cuda or x.dim() != 3 or x.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("expected a CUDA bf16/f16 tensor [S, H, D]")
    if x.stride(-1) != 1 or x.data_ptr() % 16 or any(st % 8 for st in x.stride()[:2]):
        x = x.contiguous()
    if not isinstance(seg, torch.Tensor) or seg.dtype != torch.int32 or seg.dim() != 1 or seg.numel() < 2:
        raise ValueError("seg must be an int32 tensor [nseg+1]")
    if seg.device != x.device:
        raise ValueError("seg must be on x's device")
    seg = seg.contiguous()
    S, H, D = x.shape
    return x, seg, (x.data_ptr(), _dtype_code(x.dtype), S, H, D, x.stride(0), x.stride(1))


def absmax_seg(x: torch.Tensor, seg: torch.Tensor, groups: int = 1, head_off: int = 0,
               heads_sel: int | None = None) -> torch.Tensor:
    """max |x[rows of segment z, h, :]| as float32 [nseg, groups*heads_sel] for a packed shard
    x [S, H, D] whose rows [seg[z], seg[z+1]) form segment z (entries clamped to [0, S];
    ``mh3_absmax_seg``); heads selected as in ``absmax_bh``."""
    lib = _lib.load()
    x, seg, args = _seg_args(x, seg)
    hb, off, hs = _head_sel(x.shape[1], groups, head_off, heads_sel)
    nseg = seg.numel() - 1
    out = torch.empty((nseg, groups * hs), dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        rc = lib.mh3_absmax_seg(*args, hb, off, hs, seg.data_ptr(), nseg, out.data_ptr(), _stream(x.device))
    _lib.check(rc, "mh3_absmax_seg")
    return out


def quantize_seg(x: torch.Tensor, seg: torch.Tensor, scale: torch.Tensor, out_dtype: torch.dtype = E4M3,
                 groups: int = 1, out: torch.Tensor | None = None, head_off: int = 0,
                 heads_sel: int | None = None) -> torch.Tensor:
    """Packed x [S, H, D] / scale[z, j] for the rows of segment z -> e4m3 (clamped to +-448) or
    f16, as [groups, 1, S, heads_sel, D] (``mh3_quantize_seg``; rows outside every segment are
    zeros; heads selected and numbered as in ``quantize_bh``)."""
    lib = _lib.load()
    x, seg, args = _seg_args(x, seg)
    S, H, D = x.shape
    if out_dtype not in (E4M3, torch.float16):
        raise ValueError("out_dtype must be float8_e4m3fn or float16")
    hb, off, hs = _head_sel(H, groups, head_off, heads_sel)
    nseg = seg.numel() - 1
    scale = scale.to(device=x.device, dtype=torch.float32).contiguous()
    if scale.numel() != nseg * groups * hs:
        raise ValueError("scale must hold one value per (segment, selected head)")
    shape = (groups, 1, S, hs, D)
    if out is None:
        out = torch.empty(shape, dtype=out_dtype, device=x.device)
    elif tuple(out.shape) != shape or out.dtype != out_dtype or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous {out_dtype} tensor of shape {shape}")
    code = _lib.MH3_DTYPE_F16 if out_dtype == torch.float16 else _lib.MH3_DTYPE_E4M3
    with torch.cuda.device(x.device):
        rc = lib.mh3_quantize_seg(*args, hb, off, hs, seg.data_ptr(), nseg, scale.data_ptr(), code, out.data_ptr(),
                                  _stream(x.device))
    _lib.check(rc, "mh3_quantize_seg")
    return out


# ---------------------------------------------------------------------------
# scaled GEMM / FP8 linear
# ---------------------------------------------------------------------------


def scaled_gemm(a: torch.Tensor, b: torch.Tensor, row_scale=None, col_scale=None, bias=None, a2=None, b2=None,
                row_scale_inv: bool = False, out: torch.Tensor | None = None, err: torch.Tensor | None = None,
                timeout_ns: int = 0, test_flags: int = 0) -> torch.Tensor:
    """``mh3_scaled_gemm``: bf16 (a b^T [+ a2 b2^T]) * rs[m] * cs[n] + bias[n].

    a [M,K], b [N,K]: both float8_e4m3fn or both bfloat16, last dim
    contiguous.  row_scale [M] / [M,1], col_scale [N] / [1,N] float32; bias
    bf16 [N]; a2 [M,R], b2 [N,R] bf16 (optional low-rank term).  ``err``: an
    int32 device word for wait timeouts (default: the library's own);
    ``timeout_ns``: bound on every pipeline wait (0 = the library default);
    ``test_flags``: MH3_TEST_* bits (tests of the bounded waits only).
    """
    lib = _lib.load()
    _require_cuda(a, b)
    if a.dtype != b.dtype or a.dtype not in (E4M3, torch.bfloat16):
        raise ValueError("a and b must both be float8_e4m3fn or both bfloat16")
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[1]:
        raise ValueError("a is [M,K] and b is [N,K]")
    M, K = a.shape
    N = b.shape[0]
    if a.stride(1) != 1 or b.stride(1) != 1:
        raise ValueError("a and b need a contiguous last dimension")
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    g = _lib.GemmArgs()
    g.M, g.N, g.K = M, N, K
    g.ab_dtype = _lib.MH3_DTYPE_BF16 if a.dtype == torch.bfloat16 else _lib.MH3_DTYPE_E4M3
    g.row_scale_inv = 1 if row_scale_inv else 0
    g.a, g.lda, g.b, g.ldb = a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0)
    keep = []
    for name, t, n in (("row_scale", row_scale, M), ("col_scale", col_scale, N)):
        if t is not None:
            t = t.reshape(-1)
            if t.dtype != torch.float32 or t.numel() != n:
                raise ValueError(f"{name} must be float32 with {n} elements")
            t = t.contiguous()
            keep.append(t)
            setattr(g, name, t.data_ptr())
    if bias is not None:
        bias = bias.reshape(-1).to(torch.bfloat16).contiguous()
        if bias.numel() != N:
            raise ValueError("bias must have N elements")
        keep.append(bias)
        g.bias = bias.data_ptr()
    if a2 is not None:
        if b2 is None or a2.dtype != torch.bfloat16 or b2.dtype != torch.bfloat16:
            raise ValueError("a2/b2 must both be bfloat16")
        if a2.shape[0] != M or b2.shape[0] != N or a2.shape[1] != b2.shape[1]:
            raise ValueError("a2 is [M,R] and b2 is [N,R]")
        g.R = a2.shape[1]
        g.a2, g.lda2, g.b2, g.ldb2 = a2.data_ptr(), a2.stride(0), b2.data_ptr(), b2.stride(0)
    g.out, g.ldo = out.data_ptr(), out.stride(0)
    if err is not None:
        if err.dtype != torch.int32 or not err.is_cuda:
            raise ValueError("err must be a CUDA int32 tensor")
        g.err = err.data_ptr()
    g.timeout_ns = int(timeout_ns)
    g.test_flags = int(test_flags)
    with torch.cuda.device(a.device):
        rc = lib.mh3_scaled_gemm(g, _stream(a.device))
    _lib.check(rc, "mh3_scaled_gemm")
    return out


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


# Folded LoRA operands, keyed on the identity and version of the adapter tensors and of the
# column scale: a layer's forward reuses them until an adapter or the weight scale changes
# (runtime/lora.py swaps the ``adapters`` list, an in-place edit bumps a tensor's version).
# Entries hold the source tensors, so a key's ids cannot be reused while it is cached.
_LORA_CACHE: "collections.OrderedDict" = collections.OrderedDict()
_LORA_CACHE_MAX = 1024


def _lora_key(adapters, scale_src):
    parts = []
    for A, B_, s in adapters:
        parts += [id(A), A._version, id(B_), B_._version, float(s)]
    if scale_src is not None:
        parts += [id(scale_src), scale_src._version]
    return tuple(parts)


def _lora_operands(adapters, N: int, K: int, device, col_scale=None, scale_src=None):
    """``_fold_lora`` with a cache over calls (see ``_LORA_CACHE``); ``scale_src`` is the tensor
    ``col_scale`` was derived from (the layer's ``w_scale`` buffer), which keys the cache."""
    scale_src = col_scale if scale_src is None else scale_src
    key = _lora_key(adapters, scale_src)
    hit = _LORA_CACHE.get(key)
    if hit is not None:
        _LORA_CACHE.move_to_end(key)
        return hit[1], hit[2]
    A_cat, B_cat = _fold_lora(adapters, N, K, device, col_scale)
    refs = [t for A, B_, _ in adapters for t in (A, B_)] + ([scale_src] if scale_src is not None else [])
    _LORA_CACHE[key] = (refs, A_cat, B_cat)
    while len(_LORA_CACHE) > _LORA_CACHE_MAX:
        _LORA_CACHE.popitem(last=False)
    return A_cat, B_cat


def _fold_lora(adapters, N: int, K: int, device, col_scale=None):
    """(A_cat [Rp, K] bf16, B_cat [N, Rp] bf16 = (scale*B)_cat / col_scale): the adapters
    concatenated along the rank (padded to a multiple of 16 with zeros)."""
    R = sum(int(A.shape[0]) for A, _, _ in adapters)
    Rp = _round_up(max(R, 1), 16)
    A_cat = torch.zeros((Rp, K), dtype=torch.bfloat16, device=device)
    B_cat = torch.zeros((N, Rp), dtype=torch.float32, device=device)
    r0 = 0
    for A, B_, s in adapters:
        r = int(A.shape[0])
        A_cat[r0:r0 + r] = A.to(torch.bfloat16)
        B_cat[:, r0:r0 + r] = B_.float() * float(s)
        r0 += r
    if col_scale is not None:
        B_cat = B_cat / col_scale[:, None]
    return A_cat, B_cat.to(torch.bfloat16)


@nvtx("mh3.fp8_linear")
def fp8_linear(x2d: torch.Tensor, w8: torch.Tensor, w_scale: torch.Tensor, bias, adapters) -> torch.Tensor:
    """FP8Linear forward: per-token e4m3 activations, one fused GEMM (bf16 out).

    ``adapters``: list of (A [r,K], B [N,r], scale).  Their delta
    ``scale * (x A^T) B^T`` (on the unquantised x, fp8_linear.py:45-55) is
    folded into the GEMM: a2 = (x A_cat^T) / x_scale and
    b2 = (scale*B)_cat / w_scale, both bf16, accumulated with the e4m3
    product before the row/column scales are applied.
    """
    if x2d.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        x2d = x2d.to(torch.float32)  # quantised from fp32 like the reference (fp8_linear.py:19)
    x2d = x2d.contiguous()
    M, K = x2d.shape
    N = w8.shape[0]
    x8, sa = quantize_rows(x2d)
    sb = w_scale.reshape(-1).float()
    a2 = b2 = None
    if adapters:
        xb = x2d if x2d.dtype == torch.bfloat16 else x2d.to(torch.bfloat16)
        A_cat, b2 = _lora_operands(adapters, N, K, x2d.device, col_scale=sb, scale_src=w_scale)
        a2 = scaled_gemm(xb, A_cat, row_scale=sa, row_scale_inv=True)
    return scaled_gemm(x8, w8, row_scale=sa, col_scale=sb, bias=bias, a2=a2, b2=b2)


@nvtx("mh3.linear_lora")
def linear_lora(x2d: torch.Tensor, weight: torch.Tensor, bias, adapters) -> torch.Tensor:
    """bf16 ``x W^T + bias + sum_i scale_i (x A_i^T) B_i^T`` in one GEMM (bf16 out).

    The unquantised ``nn.Linear`` + LoRA forward (runtime/lora.py:206-226
    wraps ``nn.Linear.forward`` with fp8_linear.py:45-55): ``mh3_scaled_gemm``
    on bf16 operands, the adapters' low-rank product accumulated into the same
    TMEM accumulator as extra K-steps (a2 = x A_cat^T in bf16,
    b2 = (scale*B)_cat), bias added in the epilogue, bf16 written once.
    """
    x2d = x2d.to(torch.bfloat16).contiguous()
    M, K = x2d.shape
    N = weight.shape[0]
    w = weight.to(torch.bfloat16).contiguous()
    a2 = b2 = None
    if adapters:
        A_cat, b2 = _lora_operands(adapters, N, K, x2d.device)
        a2 = scaled_gemm(x2d, A_cat)
    return scaled_gemm(x2d, w, bias=bias, a2=a2, b2=b2)


# ---------------------------------------------------------------------------
# strided host <-> device row copies
# ---------------------------------------------------------------------------


def copy_rows(dst: torch.Tensor, dst_offset: int, dst_pitch: int, src: torch.Tensor, src_offset: int,
              src_pitch: int, row_bytes: int, rows: int, stream: torch.cuda.Stream | None = None) -> None:
    """Copy ``rows`` runs of ``row_bytes`` bytes from ``src`` (byte offset ``src_offset``, row pitch
    ``src_pitch``) to ``dst`` (``dst_offset``, ``dst_pitch``), asynchronously on ``stream``
    (``mh3_copy_rows``).  Both tensors contiguous; one on the GPU, the other pinned host memory or
    the GPU.  Every byte touched must lie inside both tensors."""
    for name, t, off, pitch in (("dst", dst, dst_offset, dst_pitch), ("src", src, src_offset, src_pitch)):
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
        if off < 0 or pitch < row_bytes or row_bytes < 0 or rows < 0:
            raise ValueError("bad offsets, pitches or sizes")
        if rows and off + (rows - 1) * pitch + row_bytes > t.numel() * t.element_size():
            raise ValueError(f"copy runs past the end of {name}")
    devs = [t.device for t in (dst, src) if t.device.type == "cuda"]
    if not devs:
        raise ValueError("one of dst / src must be a CUDA tensor")
    if stream is None:
        stream = torch.cuda.current_stream(devs[0])
    lib = _lib.load()
    with torch.cuda.device(devs[0]):
        rc = lib.mh3_copy_rows(dst.data_ptr() + dst_offset, dst_pitch, src.data_ptr() + src_offset, src_pitch,
                               row_bytes, rows, stream.cuda_stream)
    _lib.check(rc, "mh3_copy_rows")


# ---------------------------------------------------------------------------
# step-residual cache reductions
# ---------------------------------------------------------------------------
_STEP_DT = {torch.bfloat16: _lib.MH3_DTYPE_BF16, torch.float16: _lib.MH3_DTYPE_F16, torch.float32: _lib.MH3_DTYPE_F32}


def step_diff(h1: torch.Tensor, prev: torch.Tensor, copy: bool = False) -> torch.Tensor:
    """float64 [2] on the device: (sum |h1 - prev|, sum |prev|) in one pass (``mh3_step_diff``);
    with ``copy`` prev is overwritten with h1 in the same pass.  Same dtype, shape and device,
    contiguous, 16-byte aligned."""
    lib = _lib.load()
    _require_cuda(h1, prev)
    if h1.dtype != prev.dtype or h1.shape != prev.shape or h1.dtype not in _STEP_DT:
        raise ValueError("h1 and prev must share a shape and a dtype in (bf16, f16, f32)")
    if not (h1.is_contiguous() and prev.is_contiguous()):
        raise ValueError("h1 and prev must be contiguous")
    sums = torch.empty(2, dtype=torch.float64, device=h1.device)
    ws = torch.empty(int(lib.mh3_step_diff_workspace_bytes()), dtype=torch.uint8, device=h1.device)
    with torch.cuda.device(h1.device):
        rc = lib.mh3_step_diff(h1.data_ptr(), prev.data_ptr(), _STEP_DT[h1.dtype], h1.numel(), 1 if copy else 0,
                               sums.data_ptr(), ws.data_ptr(), _stream(h1.device))
    _lib.check(rc, "mh3_step_diff")
    return sums
