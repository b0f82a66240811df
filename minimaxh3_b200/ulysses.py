"""Ulysses (head-parallel) sharding of FP8 attention over NCCL.

The reference runs one GPU per container and has no sequence or head
parallelism; the long-sequence workload (S=75600 self-attention) is sharded
here over 2/4/8 GPUs.  Each rank holds a contiguous sequence shard of q, k, v
``[B, S_local, H, D]`` (the layout a sequence-parallel DiT block holds).  Rank
r attends over heads ``[r*H/P, (r+1)*H/P)``.  The heads are processed in
``head_groups`` groups G; group g takes local heads ``[g*Hg, (g+1)*Hg)``,
``Hg = H/(P*G)``, i.e. global heads ``p*H/P + g*Hg + i`` of every rank block
p.  Per group:

1. per-(batch, head) absmax of the local shard's group heads
   (``mh3_absmax_bh`` with a head selection) and one ``all_reduce(MAX)``, so
   every rank quantises with the global per-(b,h) scale (the benchmark
   workloads use per-(b,h) scales);
2. local e4m3 quantisation (V: f16 V/scale for the f16 PV product, or e4m3)
   straight into the send layout ``[P, B, S_local, Hg, D]``
   (``mh3_quantize_bh``, one read of the bf16 group heads, no fp32
   temporaries);
3. one NCCL ``all_to_all_single`` per tensor: rank r receives every rank's
   tokens for its Hg group heads; for B = 1 the receive buffer is already
   ``[S, Hg, D]`` in global token order and the attention kernel reads it in
   place through its strided TMA maps;
4. local FP8 attention over the Hg heads, written (B = 1: by the kernel
   itself, through output strides) into the send buffer
   ``[P, B, S_local, Hg, D]``;
5. one ``all_to_all_single`` back, after which the group's output lands in
   its heads of ``[B, S_local, H, D]``.

Steps 1, 3 and 5 communicate (the e4m3 all-to-all moves half the bytes of a
bf16 one).  The groups form a software pipeline: the collectives run on
NCCL's stream asynchronously, and the host issues group g+2's absmax +
all-reduce, group g+1's quantisation + all-to-all and group g's attention +
all-to-all back before it waits on anything of group g-1, so the exchanges of
neighbouring groups overlap the attention kernel.  Every quantity is per
(batch, head), so the result is the same, bit for bit, for every G.

Packed variable-length batches (``cu_seqlens``: global token offsets of the
sequences packed along S, batch 1) keep the offsets global: rank r's shard
holds tokens ``[r*S_local, (r+1)*S_local)``, the scales are per (sequence,
head) (``mh3_absmax_seg`` over the shard's part of each sequence, then the
same ``all_reduce(MAX)``), the quantisation picks each row's sequence scale
(``mh3_quantize_seg``; rows outside every sequence become zeros), and after
the all-to-all the received ``[S, Hg, D]`` buffer is exactly the packed
layout the varlen kernel reads with the global ``cu_seqlens``.  Output rows
outside every sequence are zeros.  A packed total that is not a multiple of
the world size is padded by the caller with tokens past the last sequence.

``ulysses_attention_host`` runs the same pipeline on shards in pinned host
memory: each group's heads are copied in (one strided copy per tensor) on
one stream and copied back on another, overlapping the other groups'
compute; it optionally computes the block's cross-attention to replicated
text K/V per group as well.  Cross-attention needs no collective (it is
``fp8_attention`` of the local query shard); ``ulysses_attention(...,
cross_kv=)`` issues it right after the first input all-to-all, so NCCL's
exchange runs on a few SMs while the cross-attention takes the rest.

``attn_fn``, ``absmax_fn`` and ``quant_fn`` are injectable so the collective
plumbing can be tested on CPU ``gloo`` ranks with the oracle standing in for
the kernels; the defaults are the CUDA kernels and fail loudly without them.
"""
from __future__ import annotations

import math
import threading

import torch
import torch.distributed as dist

from .ops import nvtx

LOG2E = 1.4426950408889634
E4M3 = torch.float8_e4m3fn


def _world(group):
    return dist.get_world_size(group), dist.get_rank(group)


def _cuda_absmax(x, groups=1, head_off=0, heads_sel=None):
    """[B, groups*heads_sel] per-(b, selected head) absmax: ``mh3_absmax_bh``."""
    from . import ops

    return ops.absmax_bh(x, groups=groups, head_off=head_off, heads_sel=heads_sel)


def _cuda_quant(x, scale, P, out_dtype, head_off=0, heads_sel=None):
    """x [B,S_l,H,D] / scale[B, P*hs] -> [P, B, S_l, hs, D] (e4m3 clamp or f16): ``mh3_quantize_bh``."""
    from . import ops

    return ops.quantize_bh(x, scale, out_dtype=out_dtype, groups=P, head_off=head_off, heads_sel=heads_sel)


def _cuda_absmax_seg(x, groups=1, head_off=0, heads_sel=None, seg=None):
    """[nseq, groups*heads_sel] per-(sequence, selected head) absmax of a packed shard: ``mh3_absmax_seg``."""
    from . import ops

    return ops.absmax_seg(x, seg, groups=groups, head_off=head_off, heads_sel=heads_sel)


def _cuda_quant_seg(x, scale, P, out_dtype, head_off=0, heads_sel=None, seg=None):
    """Packed [1,S_l,H,D] / scale[nseq, P*hs] -> [P, 1, S_l, hs, D], zeros outside every sequence:
    ``mh3_quantize_seg``."""
    from . import ops

    return ops.quantize_seg(x, seg, scale, out_dtype=out_dtype, groups=P, head_off=head_off, heads_sel=heads_sel)


class _Packing:
    """Global ``cu_seqlens`` of a packed batch and this rank's view of them."""

    _cache: dict = {}

    def __init__(self, cu, P, r, S_l, device):
        cu = [int(c) for c in (cu.tolist() if isinstance(cu, torch.Tensor) else cu)]
        T = P * S_l
        if len(cu) < 2 or any(b < a for a, b in zip(cu, cu[1:])) or cu[0] < 0 or cu[-1] > T:
            raise ValueError(f"cu_seqlens must be non-decreasing offsets within [0, {T}] (P * S_local)")
        self.nseq = len(cu) - 1
        self.max_seqlen = max(max(b - a for a, b in zip(cu, cu[1:])), 1)
        self.first, self.last = cu[0], cu[-1]
        key = (tuple(cu), r, S_l, str(device))
        tensors = _Packing._cache.get(key)
        if tensors is None:
            if len(_Packing._cache) >= 16:
                _Packing._cache.pop(next(iter(_Packing._cache)))
            local = [min(max(c - r * S_l, 0), S_l) for c in cu]
            tensors = _Packing._cache[key] = (torch.tensor(cu, dtype=torch.int32, device=device),
                                              torch.tensor(local, dtype=torch.int32, device=device))
        self.cu, self.seg = tensors

    def clear_outside(self, rows):
        """Zero the rows of a [T, ...] tensor (global token order) outside every sequence."""
        if self.first > 0:
            rows[:self.first].zero_()
        if self.last < rows.shape[0]:
            rows[self.last:].zero_()


def _scale_from_absmax(amax):
    from . import ops

    return ops.scale_from_absmax(amax)


def global_absmax(xs, group=None, absmax_fn=None):
    """[len(xs), B, H] float32 absmax over (S, D) of each [B,S_local,H,D], max-reduced over ranks."""
    fn = absmax_fn or _cuda_absmax
    local = torch.stack([fn(x) for x in xs])
    dist.all_reduce(local, op=dist.ReduceOp.MAX, group=group)
    return local


def _exchange_async(send, group):
    """all_to_all_single on the leading (rank) dimension, dtype-agnostic; returns (recv, work)."""
    recv = torch.empty_like(send)
    s8 = send.view(torch.uint8) if send.dtype == E4M3 else send
    r8 = recv.view(torch.uint8) if recv.dtype == E4M3 else recv
    return recv, dist.all_to_all_single(r8, s8, group=group, async_op=True)


def _head_major(recv):
    """[P(src), B, S_l, Hg, D] -> [B, Hg, S, D] view (copy only when B > 1)."""
    P, B, S_l, Hg, D = recv.shape
    if B == 1:
        return recv.view(P * S_l, Hg, D).permute(1, 0, 2).unsqueeze(0)  # strided, no copy
    return recv.permute(1, 3, 0, 2, 4).reshape(B, Hg, P * S_l, D)


def _default_attn(q8, k8, v, sq, sk, sv, logit_scale_log2, out=None, cu_seqlens=None, max_seqlen=0):
    from . import ops

    kw = {} if out is None else {"out": out, "out_dtype": out.dtype}
    if cu_seqlens is not None:
        kw.update(cu_seqlens_q=cu_seqlens, cu_seqlens_k=cu_seqlens, max_seqlen_q=max_seqlen)
    return ops.attention_e4m3(q8, k8, v, sq, sk, sv, logit_scale_log2=logit_scale_log2, **kw)


def default_head_groups(local_heads: int) -> int:
    """Head groups of ``ulysses_attention_host``: groups of 2 heads (1 when the count is odd).

    The host copies are the bound there (about 55 GB/s host->device and 33 GB/s back per
    B200, 25 GB/s each way when both run), so the first group's input copy and the last
    group's output copy, which nothing overlaps, should be small; a 2-head group's attention
    launch still fills every SM several times at S >= 32K.  Device-resident calls default to
    one group: there the all-to-alls cannot overlap the attention kernel, which holds every
    SM, and smaller launches only add collective latency (measured at 2 GPUs, S=75600, H=40:
    step 46.5 ms with 1 group, 50.1 ms with 10)."""
    return local_heads // 2 if local_heads % 2 == 0 else local_heads


def _check_heads(H, P, G):
    if H % P:
        raise ValueError(f"heads ({H}) must be divisible by the world size ({P})")
    if G <= 0 or (H // P) % G:
        raise ValueError(f"head_groups ({G}) must divide the heads per rank ({H // P})")


class _Pipeline:
    """The per-group stages of one Ulysses call and their issue order.

    ``source(g)`` returns the group's tensors ``(q, k, v)`` [B, S_l, H', D] and
    the head offset of the group inside each rank block of H' (the group's
    heads are ``p*H'/P + off + i``, i < Hg); ``sink(g, recv_o, work, send_o)``
    takes the group's output ``[P(src heads), B, S_l, Hg, D]`` once ``work``
    (its all-to-all back, which reads ``send_o``) is waited on.  Tensors an
    exchange touches are only freed after a stream that waited on it: the
    sink records ``recv_o`` / ``send_o`` on its own stream when that is not
    the compute stream.
    """

    def __init__(self, P, r, Hg, shape, out_dtype, group, pv_dtype, ls2, attn_fn, absmax_fn, quant_fn, events,
                 packing=None):
        self.P, self.r, self.Hg = P, r, Hg
        self.B, self.S_l, self.D = shape
        self.out_dtype, self.group, self.pv_dtype, self.ls2 = out_dtype, group, pv_dtype, ls2
        self.attn = attn_fn or _default_attn
        self.direct = attn_fn is None and self.B == 1
        self.packing = packing
        # packed batches: the scale axis is the sequence, the kernels get the shard's segment bounds
        self.seg_kw = {} if packing is None else {"seg": packing.seg}
        self.absmax_fn = absmax_fn or (_cuda_absmax if packing is None else _cuda_absmax_seg)
        self.quant_fn = quant_fn or (_cuda_quant if packing is None else _cuda_quant_seg)
        self.events = events

    def absmax(self, xs, off):
        local = torch.stack([self.absmax_fn(x, groups=self.P, head_off=off, heads_sel=self.Hg, **self.seg_kw)
                             for x in xs])
        work = dist.all_reduce(local, op=dist.ReduceOp.MAX, group=self.group, async_op=True)
        return local, work

    def exchange_in(self, xs, off, amax, work):
        work.wait()
        scales = _scale_from_absmax(amax)                      # [3, B (packed: nseq), P*Hg]
        recvs, works = [], []
        for x, s, dt in zip(xs, scales, (E4M3, E4M3, self.pv_dtype)):
            send = self.quant_fn(x, s, self.P, dt, head_off=off, heads_sel=self.Hg, **self.seg_kw)
            recv, w = _exchange_async(send, self.group)
            recvs.append(recv)
            works.append((w, send))                             # send stays alive until the wait
        return recvs, works, scales

    def attend(self, recvs, works, scales):
        for w, _ in works:
            w.wait()
        P, B, S_l, Hg, D = self.P, self.B, self.S_l, self.Hg, self.D
        mine = slice(self.r * Hg, (self.r + 1) * Hg)
        sq, sk, sv = (s[:, mine].contiguous()[..., None] for s in scales)  # [B or nseq, Hg, 1]
        send_o = torch.empty((P, B, S_l, Hg, D), dtype=self.out_dtype, device=recvs[0].device)
        ev = None
        if self.events is not None:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        if self.packing is not None:
            # B = 1: the received [P, 1, S_l, Hg, D] is the packed [S, Hg, D] in global token order
            pk = self.packing
            hq, hk, hv = (t.view(P * S_l, Hg, D) for t in recvs)
            o_rows = send_o.view(P * S_l, Hg, D)
            kw = {"cu_seqlens": pk.cu, "max_seqlen": pk.max_seqlen}
            if self.direct:
                self.attn(hq, hk, hv, sq, sk, sv, self.ls2, out=o_rows, **kw)
            else:
                o_rows.copy_(self.attn(hq, hk, hv, sq, sk, sv, self.ls2, **kw).to(self.out_dtype))
            pk.clear_outside(o_rows)                           # the kernel writes no row outside a sequence
        else:
            hq, hk, hv = (_head_major(t) for t in recvs)
            if self.direct:
                # token s of group head h sits at s*Hg*D + h*D of the send buffer
                self.attn(hq, hk, hv, sq, sk, sv, self.ls2,
                          out=send_o.view(P * S_l, Hg, D).permute(1, 0, 2).unsqueeze(0))
            else:
                o = self.attn(hq, hk, hv, sq, sk, sv, self.ls2)     # [B, Hg, S, D]
                # chunk p = tokens of rank p -> [P, B, S_l, Hg, D]
                send_o.copy_(o.to(self.out_dtype).permute(2, 0, 1, 3).reshape(P, S_l, B, Hg, D)
                             .permute(0, 2, 1, 3, 4))
        if ev is not None:
            ev[1].record()
            self.events.append(ev)
        recv_o, w = _exchange_async(send_o, self.group)
        return recv_o, (w, send_o)

    def run(self, G, source, sink, on_quantized=None, before_first_attention=None):
        a, b, c = {}, {}, {}

        def stage_a(g):
            xs, off = source(g)
            a[g] = (xs, off) + self.absmax(xs, off)

        def stage_b(g):
            b[g] = self.exchange_in(*a.pop(g))
            if on_quantized is not None:
                on_quantized(g)  # the group's inputs are no longer read

        def stage_c(g):
            c[g] = self.attend(*b.pop(g))

        def stage_d(g):
            recv_o, (w, send_o) = c.pop(g)
            sink(g, recv_o, w, send_o)

        # Every rank issues the same collectives in the same order: all-reduce(g+2),
        # all-to-all(g+1), all-to-all back(g) per iteration.
        stage_a(0)
        if G > 1:
            stage_a(1)
        stage_b(0)
        for g in range(G):
            if g + 2 < G:
                stage_a(g + 2)
            if g + 1 < G:
                stage_b(g + 1)
            if g == 0 and before_first_attention is not None:
                # local work issued here runs while the first exchanges are in flight
                before_first_attention()
            stage_c(g)
            if g >= 1:
                stage_d(g - 1)
        stage_d(G - 1)


def _packing(cu_seqlens, P, r, B, S_l, device):
    if cu_seqlens is None:
        return None
    if B != 1:
        raise ValueError("cu_seqlens needs a packed batch: shards [1, S_local, H, D]")
    return _Packing(cu_seqlens, P, r, S_l, device)


@nvtx("mh3.ulysses_attention")
def ulysses_attention(q, k, v, group=None, scale=None, pv_dtype=torch.float16, attn_fn=None, events=None,
                      absmax_fn=None, quant_fn=None, head_groups=1, out=None, cu_seqlens=None, cross_kv=None,
                      exchange="nccl"):
    """Head-parallel FP8 attention of sequence shards ``[B, S_local, H, D]``.

    Returns the local output shard ``[B, S_local, H, D]`` (q's dtype; written
    into ``out`` when given, contiguous).  H must be divisible by the world
    size P and H/P by ``head_groups``; every rank must hold the same S_local.
    ``cross_kv``: optional (k_text, v_text) CUDA tensors ``[B, H, T, D]``
    replicated on every rank; the block's cross-attention of the local query
    shard (``fp8_attention``, no collective) is then issued right after the
    first input all-to-all, so that exchange runs while it computes, and the
    call returns ``(out, cross)`` with ``cross`` ``[B, S_local, H, D]`` (a
    view of a ``[B, H, S_local, D]``-strided tensor).
    ``exchange``: ``"nccl"`` (NCCL all-to-alls) or ``"peer"`` (copy-engine
    pulls from the peers' buffers mapped through CUDA IPC,
    ``peer_exchange.ulysses_attention_peer``: batch 1, one head group, the
    CUDA kernels, with or without ``cu_seqlens``; same result bit for bit).
    ``cu_seqlens``: global offsets (host ints: a list or a CPU tensor, the same
    on every rank) of sequences packed along S of a batch-1 input; attention
    then stays inside each sequence, with per-(sequence, head) scales.
    ``events``: optional list that receives one (start, end) pair of timing
    CUDA events around each local attention launch.  ``attn_fn`` /
    ``absmax_fn`` / ``quant_fn`` replace the CUDA kernels (for CPU process
    groups in tests; absmax_fn / quant_fn take the head selection of
    ``ops.absmax_bh`` / ``ops.quantize_bh``, plus ``seg=`` (the shard's
    segment bounds) and attn_fn ``cu_seqlens=`` / ``max_seqlen=`` for a packed
    batch).
    """
    if exchange == "peer":
        if head_groups != 1 or attn_fn or absmax_fn or quant_fn:
            raise ValueError("exchange='peer' takes one head group and the CUDA kernels")
        if cu_seqlens is not None and cross_kv is not None:
            raise ValueError("cross_kv is not supported with cu_seqlens")
        from .peer_exchange import ulysses_attention_peer

        P, r = _world(group)
        packing = _packing(cu_seqlens, P, r, q.shape[0], q.shape[1], q.device)
        return ulysses_attention_peer(q, k, v, group=group, scale=scale, pv_dtype=pv_dtype, out=out,
                                      cross_kv=cross_kv, events=events, packing=packing)
    if exchange != "nccl":
        raise ValueError("exchange must be 'nccl' or 'peer'")
    P, r = _world(group)
    B, S_l, H, D = q.shape
    _check_heads(H, P, head_groups)
    packing = _packing(cu_seqlens, P, r, B, S_l, q.device)
    Hl = H // P
    Hg = Hl // head_groups
    if out is None:
        out = torch.empty((B, S_l, H, D), dtype=q.dtype, device=q.device)
    elif tuple(out.shape) != (B, S_l, H, D) or out.dtype != q.dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous tensor shaped and typed like q")
    oview = out.view(B, S_l, P, Hl, D)
    ls2 = (scale if scale is not None else 1.0 / math.sqrt(D)) * LOG2E

    def source(g):
        return (q, k, v), g * Hg

    def sink(g, recv_o, work, send_o):
        work.wait()
        oview[:, :, :, g * Hg:(g + 1) * Hg].copy_(recv_o.permute(1, 2, 0, 3, 4))

    pipe = _Pipeline(P, r, Hg, (B, S_l, D), q.dtype, group, pv_dtype, ls2, attn_fn, absmax_fn, quant_fn, events,
                     packing)
    cross = []

    def cross_attention():
        from .kernels.fp8_attention import fp8_attention

        kt, vt = cross_kv
        cross.append(fp8_attention(q.transpose(1, 2), kt, vt, scale=scale).transpose(1, 2))

    if cross_kv is not None and packing is not None:
        raise ValueError("cross_kv is not supported with cu_seqlens")
    pipe.run(head_groups, source, sink, before_first_attention=cross_attention if cross_kv is not None else None)
    return out if cross_kv is None else (out, cross[0])


class _HostShardBuffers:
    """Device copies of host-resident shards, reused across ``ulysses_attention_host`` calls."""

    _pool: dict = {}
    _lock = threading.Lock()

    @classmethod
    def get(cls, key, make, groups):
        with cls._lock:
            ent = cls._pool.get(key)
            if ent is None:
                if len(cls._pool) >= 4:          # bound the cache: drop the oldest shape
                    cls._pool.pop(next(iter(cls._pool)))
                ent = cls._pool[key] = {"bufs": make(), "free": [None] * groups}
            return ent


def ulysses_attention_host(q, k, v, out=None, group=None, scale=None, pv_dtype=torch.float16, head_groups=None,
                           cross_kv=None, cross_out=None, events=None, cu_seqlens=None):
    """``ulysses_attention`` of host-resident shards, streamed per head group.

    q, k, v: contiguous pinned CPU tensors ``[B, S_local, H, D]`` (bf16 or
    f16); ``out``: pinned CPU tensor like q (allocated when None).  The work
    runs on the current CUDA device's current stream, which is made to wait
    for the last copy back: ``out`` is valid once that stream is
    synchronised.  Group g's heads (``p*H/P + g*Hg + i``) are copied to the
    device as ``[B, S_local, P*Hg, D]`` on an input stream while earlier
    groups compute, and its output is copied back on an output stream.

    ``cross_kv``: optional (k_text, v_text) CUDA tensors ``[B, H, T, D]``
    replicated on every rank; then each group also runs ``fp8_attention`` of
    its query heads against them, written to ``cross_out`` (pinned CPU
    ``[B, S_local, H, D]``, allocated when None).  Returns ``out`` or
    ``(out, cross_out)``.  ``cu_seqlens``: as in ``ulysses_attention`` (not
    with ``cross_kv``: each packed sequence would need its own text K/V).
    """
    from . import ops

    P, r = _world(group)
    for name, t in (("q", q), ("k", k), ("v", v)):
        if t.device.type != "cpu" or t.dim() != 4 or not t.is_contiguous() or t.shape != q.shape or t.dtype != q.dtype:
            raise ValueError(f"{name} must be a contiguous 4-D CPU tensor shaped and typed like q")
    B, S_l, H, D = q.shape
    G = head_groups or default_head_groups(H // P if H % P == 0 else 1)
    _check_heads(H, P, G)
    if cu_seqlens is not None and cross_kv is not None:
        raise ValueError("cross_kv is not supported with cu_seqlens")
    Hl = H // P
    Hg = Hl // G
    es = q.element_size()
    dev = torch.device("cuda", torch.cuda.current_device())
    packing = _packing(cu_seqlens, P, r, B, S_l, dev)

    def host_like(t, name):
        if t is None:
            return torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
        if t.shape != q.shape or t.dtype != q.dtype or t.device.type != "cpu" or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous CPU tensor shaped like q")
        return t

    out = host_like(out, "out")
    if cross_kv is not None:
        cross_out = host_like(cross_out, "cross_out")
        kt, vt = cross_kv
        heads = [torch.tensor([p * Hl + g * Hg + i for p in range(P) for i in range(Hg)], device=dev)
                 for g in range(G)]
    ls2 = (scale if scale is not None else 1.0 / math.sqrt(D)) * LOG2E
    s_cmp = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    # Device copies of the shard, kept across calls (per device, compute stream
    # and shape): group g's buffer is refilled once the previous call's
    # quantisation of group g (its last reader) is done, so a call's first
    # copies overlap the previous call's last groups.
    ent = _HostShardBuffers.get((dev.index, s_cmp.cuda_stream, q.dtype, G, B, S_l, P * Hg, D),
                                lambda: [torch.empty((G, B, S_l, P * Hg, D), dtype=q.dtype, device=dev)
                                         for _ in range(3)], G)
    xs, free = ent["bufs"], ent["free"]
    row = Hg * D * es                       # bytes of one group's heads of one (token, rank block)
    pitch = Hl * D * es                     # one rank block of heads

    def source(g):
        with torch.cuda.stream(s_in):
            if free[g] is not None:
                s_in.wait_event(free[g])
            for x, h in zip(xs, (q, k, v)):
                ops.copy_rows(x[g], 0, row, h, g * row, pitch, row, B * S_l * P, stream=s_in)
            ev = torch.cuda.Event()
            ev.record(s_in)
        s_cmp.wait_event(ev)
        grp = tuple(x[g] for x in xs)
        if cross_kv is not None:
            from .kernels.fp8_attention import fp8_attention

            c = fp8_attention(grp[0].transpose(1, 2), kt.index_select(1, heads[g]), vt.index_select(1, heads[g]),
                              scale=scale)
            ct = c.transpose(1, 2)          # storage is [B, S_l, P*Hg, D] (empty_like of q's view)
            if not ct.is_contiguous():
                ct = ct.contiguous()
            done = torch.cuda.Event()
            done.record(s_cmp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(done)
                ops.copy_rows(cross_out, g * row, pitch, ct, 0, row, row, B * S_l * P, stream=s_out)
            ct.record_stream(s_out)
        return grp, 0

    def sink(g, recv_o, work, send_o):
        with torch.cuda.stream(s_out):
            work.wait()
            for p in range(P):
                ops.copy_rows(out, (p * Hl + g * Hg) * D * es, H * D * es, recv_o[p], 0, row, row, B * S_l,
                              stream=s_out)
        recv_o.record_stream(s_out)
        send_o.record_stream(s_out)

    def quantized(g):
        ev = torch.cuda.Event()
        ev.record(s_cmp)
        free[g] = ev

    pipe = _Pipeline(P, r, Hg, (B, S_l, D), q.dtype, group, pv_dtype, ls2, None, None, None, events, packing)
    pipe.run(G, source, sink, on_quantized=quantized)
    s_cmp.wait_stream(s_out)
    return out if cross_kv is None else (out, cross_out)
