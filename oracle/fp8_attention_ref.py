"""CPU restatement of the reference FP8 attention path (TEST INFRASTRUCTURE).

Restates ``kernels/fp8_attention.py`` of viragadel6/minimaxh3 as vectorised
torch-on-CPU code.  Every function cites the reference lines it follows.  It
is the checker for the CUDA path in ``minimaxh3_b200`` and is never imported
by the package itself.

Also holds two oracles that are not in the reference:

* :func:`sdpa_dequant_oracle` - float64 softmax attention on the dequantised
  e4m3 inputs.  The north-star tolerance (cosine >= 0.9995, max-abs error
  <= 2e-2 relative to this oracle) is stated against it.
* :func:`exp2_attention_emulation` - the block algorithm of this package's
  CUDA kernel (lazy max with threshold ``T``, P = e4m3(2^(s - m + OFF)),
  per-row sums) with exact exp2, used as a tighter second check.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

LOG2E = 1.4426950408889634  # fp8_attention.py:9
E4M3_MAX = 448.0
E4M3 = torch.float8_e4m3fn


def cdiv(a: int, b: int) -> int:
    return (a + b - 1) // b


def _f32(x: float) -> torch.Tensor:
    return torch.tensor(x, dtype=torch.float32)


def _pad_rows(x: torch.Tensor, rows: int) -> torch.Tensor:
    """Zero-pad dim 2 of a [B,H,S,D] tensor to ``rows`` (masked loads, other=0)."""
    pad = rows - x.shape[2]
    return F.pad(x, (0, 0, 0, pad)) if pad > 0 else x


def quantize_q(q: torch.Tensor, c: float, block: int = 128):
    """``_quantize_q_kernel`` (fp8_attention.py:39-77).

    q: [B,H,S,D] bf16/fp16 (any strides).  Returns (q8 [B,H,S,D] e4m3,
    scale_q [B,H,ceil(S/128)] f32).  ``c`` = softmax scale * log2(e), folded
    into q before quantisation (:69) and therefore into ``scale_q``.
    """
    B, H, S, D = q.shape
    nq = cdiv(S, block)
    qf = q.float() * _f32(c)                                   # :68-69
    blk = _pad_rows(qf, nq * block).reshape(B, H, nq, block, D)
    amax = blk.abs().amax(dim=(3, 4))                          # :70
    scale = torch.clamp(amax, min=1.0e-12) / _f32(448.0)       # :71
    q8 = torch.clamp(blk / scale[..., None, None], -448.0, 448.0).to(E4M3)  # :72-73
    return q8.reshape(B, H, nq * block, D)[:, :, :S].contiguous(), scale


def k_channel_mean(k: torch.Tensor) -> torch.Tensor:
    """``k.float().mean(dim=2, keepdim=True)`` (fp8_attention.py:338)."""
    return k.float().mean(dim=2, keepdim=True).contiguous()


def quantize_k(k: torch.Tensor, k_mean: torch.Tensor, block: int = 128):
    """``_quantize_k_kernel`` (fp8_attention.py:80-119): centre, per-128-key scale."""
    B, H, S, D = k.shape
    nk = cdiv(S, block)
    kf = k.float() - k_mean.reshape(B, H, 1, D).float()        # :109-111
    blk = _pad_rows(kf, nk * block).reshape(B, H, nk, block, D)
    amax = blk.abs().amax(dim=(3, 4))                          # :112
    scale = torch.clamp(amax, min=1.0e-12) / _f32(448.0)       # :113
    k8 = torch.clamp(blk / scale[..., None, None], -448.0, 448.0).to(E4M3)  # :114-115
    return k8.reshape(B, H, nk * block, D)[:, :, :S].contiguous(), scale


def quantize_v(v: torch.Tensor):
    """``_quantize_v_kernel`` (fp8_attention.py:122-170).

    Per-(b,h,channel) absmax over the whole sequence (:140-153), scale
    (:154), cast (:167-168).  Returns (v8 [B,H,S,D] e4m3 in natural
    [key, channel] order, scale_v [B,H,D]).  The reference stores the same
    bytes transposed as ``v8t[B,H,D,S]`` (:168-170); ``v8.transpose(2,3)``
    gives that layout.
    """
    vf = v.float()
    amax = vf.abs().amax(dim=2)                                # :153
    scale = torch.clamp(amax, min=1.0e-12) / _f32(448.0)       # :154
    v8 = torch.clamp(vf / scale[:, :, None, :], -448.0, 448.0).to(E4M3)  # :167-168
    return v8.contiguous(), scale


def bittrick_p(s: torch.Tensor, m: torch.Tensor, valid: torch.Tensor) -> torch.Tensor:
    """The reference's P: a piecewise-linear 2^(s-m) built from e4m3 bits.

    fp8_attention.py:274-279: ``bits = rint(8 s + 56 - 8 m)`` clamped to
    [0, 126], zero where ``8 s + 56 - 8 m < 8`` or the key is invalid, then
    bit-cast to e4m3.  ``torch.round`` rounds half to even like ``rint``.
    """
    cst = _f32(56.0) - _f32(8.0) * m                           # :274
    bits_f = s * _f32(8.0) + cst[..., None]                    # :275
    rounded = torch.round(bits_f)                              # :276
    clamped = torch.clamp(rounded, 0.0, 126.0)                 # :277
    bits = torch.where((bits_f < 8.0) | (~valid), torch.zeros_like(clamped), clamped)
    return bits.to(torch.uint8).view(E4M3)                     # :278-279


def attention_kernel_ref(
    q8: torch.Tensor,
    k8: torch.Tensor,
    v8: torch.Tensor,
    scale_q: torch.Tensor,
    scale_k: torch.Tensor,
    scale_v: torch.Tensor,
    key_mask: torch.Tensor | None = None,
    key_bias: torch.Tensor | None = None,
    repair_tau: float = -1.0,
    block_n: int = 128,
    out_dtype: torch.dtype = torch.bfloat16,
) -> torch.Tensor:
    """``_fp8_attn_kernel`` (fp8_attention.py:190-297), all query blocks at once.

    q8, k8, v8: [B,H,S,D] e4m3 (v8 in [key, channel] order); scale_q
    [B,H,ceil(Sq/128)], scale_k [B,H,ceil(Sk/128)], scale_v [B,H,D];
    key_mask [B,Sk] bool, key_bias [B,Sk] f32.  ``block_n`` is the autotuned
    KV tile (64 or 128, :179); the result depends on it.  Dot products are
    summed in float64 and rounded once to float32 (the tensor core sums the
    exact e4m3 products in fp32).
    """
    B, H, Sq, D = q8.shape
    Sk = k8.shape[2]
    BM = 128
    nq = cdiv(Sq, BM)                                          # :226
    nk = cdiv(Sk, block_n)                                     # :227
    qd = _pad_rows(q8.double(), nq * BM).reshape(B, H, nq, BM, D)
    kd = _pad_rows(k8.double(), nk * block_n).reshape(B, H, nk, block_n, D)
    vd = _pad_rows(v8.double(), nk * block_n).reshape(B, H, nk, block_n, D)
    rows = torch.arange(nq * BM).reshape(nq, BM)
    mask_m = rows < Sq                                         # :221
    # scale_q is loaded per row with other=1.0 for rows >= Sq (:230-234)
    sq_rows = scale_q[:, :, (rows // 128).clamp(max=scale_q.shape[2] - 1)]
    sq_rows = torch.where(mask_m, sq_rows, torch.ones_like(sq_rows))

    m = torch.full((B, H, nq, BM), -1.0e9, dtype=torch.float32)   # :236
    l = torch.zeros((B, H, nq, BM), dtype=torch.float32)           # :237
    acc = torch.zeros((B, H, nq, BM, D), dtype=torch.float32)      # :238
    acc_r = torch.zeros_like(acc)                                  # :239
    j0 = (torch.arange(nq) * nk) // nq                             # :241
    do_repair = float(repair_tau) >= 0.0
    tau = _f32(float(repair_tau))
    for i in range(nk):                                            # :244
        j = (j0 + i) % nk                                          # :245
        offs_n = j[:, None] * block_n + torch.arange(block_n)[None, :]  # :246
        mask_n = offs_n < Sk                                       # :247
        k_t = kd[:, :, j]                                          # [B,H,nq,BN,D]
        v_t = vd[:, :, j]
        sk_j = scale_k[:, :, (j * block_n) // 128]                 # :252
        dot = torch.matmul(qd, k_t.transpose(-1, -2)).float()
        s = dot * sq_rows[..., None] * sk_j[..., None, None]       # :253
        valid = mask_m[:, :, None] & mask_n[:, None, :]            # :255  [nq,BM,BN]
        valid = valid.expand(B, H, nq, BM, block_n)
        gidx = offs_n.clamp(max=Sk - 1)
        if key_bias is not None:                                   # :256-259
            kb = key_bias.float()[:, gidx]                         # [B,nq,BN]
            kb = torch.where(mask_n, kb, torch.zeros_like(kb))[:, None, :, None, :]
            valid = valid & (kb > -1.0e8)
            s = s + kb * _f32(LOG2E)
        if key_mask is not None:                                   # :260-262
            km = key_mask.bool()[:, gidx] & mask_n
            valid = valid & km[:, None, :, None, :]
        s = torch.where(valid, s, _f32(-1.0e9))                    # :264
        rowmax = s.amax(dim=-1)                                    # :266
        m_new = torch.where((rowmax > m + 8.0) | (m == -1.0e9), rowmax, m)  # :267
        alpha = torch.exp2(m - m_new)                              # :268
        acc = acc * alpha[..., None]                               # :269
        acc_r = acc_r * alpha[..., None]                           # :270
        l = l * alpha                                              # :271
        m = m_new                                                  # :272
        p8 = bittrick_p(s, m, valid)                               # :274-279
        p_apx = p8.float()                                         # :284
        l = l + p_apx.sum(dim=-1)                                  # :285
        acc = acc + torch.matmul(p_apx.double(), v_t).float()      # :286
        if do_repair:                                              # :288-292
            p_exact = torch.where(valid, torch.exp2(s - m[..., None]), _f32(0.0))
            delta = torch.where(p_apx >= tau, p_exact - p_apx, _f32(0.0))
            acc_r = acc_r + torch.matmul(
                delta.to(torch.bfloat16).double(), v_t.to(torch.bfloat16).double()
            ).float()
            l = l + delta.sum(dim=-1)
    out = (acc + acc_r) * scale_v[:, :, None, None, :] / torch.clamp(l, min=1.0e-12)[..., None]  # :295
    out = out.reshape(B, H, nq * BM, D)[:, :, :Sq]
    return out.to(out_dtype)                                       # :296-297, :403


def key_bias2_ref(key_mask, key_bias, B: int, Sk: int, tile: int = 128):
    """The reference's per-key validity and bias (fp8_attention.py:256-262) in
    the form the CUDA kernel takes: ``(bias2, kv_len)``.

    A key is valid when ``key_mask`` is true and ``key_bias > -1e8``;
    ``bias2[b, j] = fp32(key_bias * fp32(log2 e))`` for a valid key (0 with no
    bias), ``-inf`` for an invalid key and for the padding up to a whole
    ``tile``; ``kv_len[b]`` is one past the last valid key (0 if none).
    ``key_mask`` / ``key_bias`` broadcast over the batch ([Sk], [1, Sk] or
    [B, Sk]).  CPU tensors in, CPU tensors out.
    """
    valid = torch.ones((B, Sk), dtype=torch.bool)
    val = torch.zeros((B, Sk), dtype=torch.float32)
    if key_bias is not None:
        kb = key_bias.cpu().float().reshape(-1, Sk).expand(B, Sk)
        valid = valid & (kb > -1.0e8)                          # :258
        val = kb * _f32(LOG2E)                                 # :259
    if key_mask is not None:
        valid = valid & key_mask.cpu().bool().reshape(-1, Sk).expand(B, Sk)   # :261-262
    bias2 = torch.full((B, cdiv(Sk, tile) * tile), -math.inf, dtype=torch.float32)
    bias2[:, :Sk] = torch.where(valid, val, torch.full_like(val, -math.inf))
    idx = torch.arange(1, Sk + 1, dtype=torch.int32)
    kv_len = torch.where(valid, idx, torch.zeros_like(idx)).amax(dim=1).to(torch.int32)
    return bias2, kv_len


def fp8_attention_ref(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    scale: float | None = None,
    key_mask: torch.Tensor | None = None,
    key_bias: torch.Tensor | None = None,
    repair_tau: float = -1.0,
    block_n: int = 128,
    return_intermediates: bool = False,
):
    """``fp8_attention`` wrapper (fp8_attention.py:300-403) on CPU tensors."""
    B, H, Sq, D = q.shape
    c = (scale if scale is not None else (1.0 / math.sqrt(D))) * LOG2E   # :315
    q8, sq = quantize_q(q, c)                                  # :321-336
    k_mean = k_channel_mean(k)                                 # :338
    k8, sk = quantize_k(k, k_mean)                             # :339-354
    v8, sv = quantize_v(v)                                     # :356-369
    km = key_mask.to(torch.bool).contiguous() if key_mask is not None else None   # :373
    kb = key_bias.to(torch.float32).contiguous() if key_bias is not None else None  # :374
    out = attention_kernel_ref(q8, k8, v8, sq, sk, sv, km, kb, repair_tau, block_n, q.dtype)
    if return_intermediates:
        return out, dict(q8=q8, scale_q=sq, k_mean=k_mean, k8=k8, scale_k=sk, v8=v8, scale_v=sv)
    return out


# ---------------------------------------------------------------------------
# Oracles that are not in the reference
# ---------------------------------------------------------------------------


def dequant_blocks(x8: torch.Tensor, scale: torch.Tensor, block: int = 128) -> torch.Tensor:
    """x8 [B,H,S,D] e4m3 times a per-``block``-row scale [B,H,nblk] (float64)."""
    B, H, S, D = x8.shape
    idx = torch.arange(S) // block
    return x8.double() * scale.double()[:, :, idx][..., None]


def sdpa_dequant_oracle(
    q_deq: torch.Tensor,
    k_deq: torch.Tensor,
    v_deq: torch.Tensor,
    logit_scale: float,
    key_mask: torch.Tensor | None = None,
    key_bias: torch.Tensor | None = None,
    base2: bool = False,
) -> torch.Tensor:
    """float64 softmax attention on dequantised inputs -> float32.

    ``logits = (q_deq k_deq^T) * logit_scale (+ key_bias)``, softmax over
    keys (base 2 when ``base2``: the drop-in path folds log2(e) into q).
    Keys with ``key_mask`` False or ``key_bias <= -1e8`` are excluded; a row
    with no valid key gives 0, as the reference kernel does (:295 with l=0).
    """
    logits = torch.matmul(q_deq.double(), k_deq.double().transpose(-1, -2)) * logit_scale
    B = q_deq.shape[0]
    Sk = k_deq.shape[2]
    valid = torch.ones((B, 1, 1, Sk), dtype=torch.bool)
    if key_bias is not None:
        kb = key_bias.double().reshape(B, 1, 1, Sk)
        valid = valid & (kb > -1.0e8)
        logits = logits + (kb * LOG2E if base2 else kb)
    if key_mask is not None:
        valid = valid & key_mask.bool().reshape(B, 1, 1, Sk)
    logits = torch.where(valid, logits, torch.tensor(-math.inf, dtype=torch.float64))
    mx = logits.amax(dim=-1, keepdim=True)
    mx = torch.where(torch.isfinite(mx), mx, torch.zeros_like(mx))
    p = torch.exp2(logits - mx) if base2 else torch.exp(logits - mx)
    den = p.sum(dim=-1, keepdim=True)
    out = torch.matmul(p, v_deq.double()) / torch.clamp(den, min=1e-300)
    return out.float()


# Lazy-max threshold and P offset of this package's kernel (log2 units):
# the running max is only raised when a tile's max exceeds it by more than
# LAZY_T, and P = 2^(s - m + P_OFFSET) stays <= 2^(LAZY_T + P_OFFSET) < 448.
LAZY_T = 4.5
P_OFFSET = 4.0
LAZY_T16 = 12.0
P_OFFSET16 = 0.0


def softmax_params(p_dtype: torch.dtype) -> tuple[float, float]:
    """(lazy threshold, P offset) the kernel uses for a P dtype (log2 units).

    e4m3 P: P <= 2^(4 + 4.5) < 448 with the row max at exactly 2^4; 16-bit
    P: a wide threshold (P <= 2^12) so that the running max rises in few tiles.
    """
    if p_dtype == E4M3:
        return LAZY_T, P_OFFSET
    return LAZY_T16, P_OFFSET16


def exp2_attention_emulation(
    q8: torch.Tensor,
    k8: torch.Tensor,
    v8: torch.Tensor,
    scale_q: torch.Tensor,
    scale_k: torch.Tensor,
    scale_v: torch.Tensor,
    logit_scale_log2: float = 1.0,
    key_mask: torch.Tensor | None = None,
    key_bias: torch.Tensor | None = None,
    block_n: int = 128,
    lazy_t: float | None = None,
    p_offset: float | None = None,
    p_dtype: torch.dtype = E4M3,
) -> torch.Tensor:
    """Block algorithm of the CUDA kernel with exact exp2 (float32 result).

    Per 128-key tile: ``t = s * c + bias*log2e``; running max raised only when
    the tile max exceeds it by ``lazy_t``; ``P = e4m3(2^(t - m + p_offset))``
    feeds the PV product (``p_dtype`` = torch.bfloat16 / float16 for the
    kernel's 16-bit-PV variant); the row sum uses the unrounded 2^(...)
    values.  ``lazy_t`` / ``p_offset`` default to the kernel's values for
    ``p_dtype`` (``softmax_params``).
    Scales: scale_q/scale_k per 128-row block [B,H,nblk] (broadcast a
    per-(b,h) scale by passing nblk=1), scale_v per channel [B,H,D] (or
    [B,H,1]).
    """
    d_lazy, d_off = softmax_params(p_dtype)
    lazy_t = d_lazy if lazy_t is None else lazy_t
    p_offset = d_off if p_offset is None else p_offset
    B, H, Sq, D = q8.shape
    Sk = k8.shape[2]
    nk = cdiv(Sk, block_n)
    qblk = torch.arange(Sq) // 128
    qblk = qblk.clamp(max=scale_q.shape[2] - 1)
    qd = q8.double() * scale_q.double()[:, :, qblk][..., None]
    m = torch.full((B, H, Sq), -1.0e30, dtype=torch.float64)
    l = torch.zeros((B, H, Sq), dtype=torch.float64)
    acc = torch.zeros((B, H, Sq, D), dtype=torch.float64)
    for j in range(nk):
        lo, hi = j * block_n, min(Sk, (j + 1) * block_n)
        kblk = min(lo // 128, scale_k.shape[2] - 1)
        kt = k8[:, :, lo:hi].double() * scale_k.double()[:, :, kblk][..., None, None]
        t = torch.matmul(qd, kt.transpose(-1, -2)).float().double() * logit_scale_log2
        valid = torch.ones((B, 1, 1, hi - lo), dtype=torch.bool)
        if key_bias is not None:
            kb = key_bias.double()[:, lo:hi].reshape(B, 1, 1, -1)
            valid = valid & (kb > -1.0e8)
            t = t + kb * LOG2E
        if key_mask is not None:
            valid = valid & key_mask.bool()[:, lo:hi].reshape(B, 1, 1, -1)
        t = torch.where(valid, t, torch.tensor(-math.inf, dtype=torch.float64))
        tmax = t.amax(dim=-1)
        upd = tmax > m + lazy_t
        m_new = torch.where(upd, tmax, m)
        alpha = torch.exp2(m - m_new)
        acc = acc * alpha[..., None]
        l = l * alpha
        m = m_new
        p = torch.exp2(t - m[..., None] + p_offset)
        l = l + p.sum(dim=-1)
        pq = p.float().to(p_dtype).double()
        acc = acc + torch.matmul(pq, v8[:, :, lo:hi].double())
    out = acc * scale_v.double()[:, :, None, :] / torch.clamp(l, min=1e-30)[..., None]
    return out.float()


def compare(out: torch.Tensor, ref: torch.Tensor) -> dict:
    """cosine, max-abs error, max|ref| and max-abs error relative to max|ref|."""
    a = out.double().flatten()
    b = ref.double().flatten()
    cos = float(torch.dot(a, b) / (a.norm() * b.norm()).clamp(min=1e-300))
    err = float((a - b).abs().max()) if a.numel() else 0.0
    scale = float(b.abs().max()) if b.numel() else 1.0
    return {"cos": cos, "max_abs": err, "ref_absmax": scale, "max_abs_rel": err / max(scale, 1e-30)}


def within_tolerance(r: dict, cos_min: float = 0.9995, max_abs_rel: float = 2e-2) -> bool:
    """The north-star tolerance: cos >= 0.9995 and max-abs error <= 2e-2 x max|oracle|.

    The max-abs bound is read relative to the oracle's largest magnitude:
    with the outlier-channel inputs outputs reach ~10, where the bf16
    rounding of the output alone exceeds an absolute 2e-2; for outputs below
    unit scale the relative reading is the stricter one.  ``compare``
    reports the absolute error beside it (``max_abs``).
    """
    return r["cos"] >= cos_min and r["max_abs"] <= max_abs_rel * r["ref_absmax"]
