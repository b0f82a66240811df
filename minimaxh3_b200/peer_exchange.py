"""Ulysses exchange over copy engines: CUDA IPC mappings of the peers' send buffers.

``ulysses_attention(..., exchange="peer")`` runs the head-parallel step of
``ulysses.py`` with the two all-to-alls replaced by copy-engine pulls:

1. per-(b,h) absmax of the shard, one NCCL ``all_reduce(MAX)`` (as before);
2. quantisation into this rank's exported send buffers ``[P, B, S_l, Hl, D]``
   (two sets, alternating between calls);
3. barrier A (a one-word NCCL all-reduce on the compute stream): every
   rank's quantisation is done;
4. on one copy stream per source rank, rank r pulls chunk r of every
   rank's send buffers into its receive buffers (``mh3_copy_rows`` on peer
   pointers: copy engines, no SM time), while the compute stream runs the
   block's cross-attention when ``cross_kv`` is given;
5. the attention kernel over the Hl local heads, written into this rank's
   exported output buffer ``[P, B, S_l, Hl, D]``;
6. barrier B: every rank's attention is done;
7. on the copy streams, rank r pulls chunk r of every rank's output buffer
   straight into its heads of ``out [B, S_l, H, D]`` (one pitched copy per
   peer), and the compute stream waits for it.

Why the buffers may be reused: a rank's quantisation of call n+1 writes the
send set the peers pulled in call n-1, whose pulls each peer's compute
stream waited for before its own quantisation of call n, which barrier A of
call n ordered before this rank's call n+1; the output buffer is written
after barrier A of the next call, which every peer passes only after waiting
for its output pulls.  Buffers are allocated once per (process group,
device, shape) with ``mh3_peer_alloc`` and kept for the life of the process
(a peer may still hold a mapping).  Plain peer mappings; no multicast.
"""
from __future__ import annotations

import ctypes
import math

import torch
import torch.distributed as dist

from . import _lib

E4M3 = torch.float8_e4m3fn
LOG2E = 1.4426950408889634


class _Raw:
    """A device allocation seen through ``__cuda_array_interface__`` (bytes)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}


def _check(rc: int, what: str) -> None:
    _lib.check(rc, what)


def _alloc(nbytes: int) -> int:
    lib = _lib.load()
    p = ctypes.c_void_p()
    _check(lib.mh3_peer_alloc(nbytes, ctypes.byref(p)), "mh3_peer_alloc")
    return int(p.value)


def _handle(ptr: int) -> bytes:
    lib = _lib.load()
    buf = ctypes.create_string_buffer(_lib.MH3_PEER_HANDLE_BYTES)
    _check(lib.mh3_peer_handle(ptr, buf), "mh3_peer_handle")
    return buf.raw


def _open(handle: bytes) -> int:
    lib = _lib.load()
    p = ctypes.c_void_p()
    _check(lib.mh3_peer_open(ctypes.create_string_buffer(handle, len(handle)), ctypes.byref(p)), "mh3_peer_open")
    return int(p.value)


def _copy(dst: int, dst_pitch: int, src: int, src_pitch: int, row_bytes: int, rows: int, stream) -> None:
    _check(_lib.load().mh3_copy_rows(dst, dst_pitch, src, src_pitch, row_bytes, rows, stream.cuda_stream),
           "mh3_copy_rows")


class _Buffers:
    """This rank's exported buffers of one shape and the peers' buffers mapped here."""

    _cache: dict = {}

    def __init__(self, group, device, B, S_l, Hl, D, pv_dtype, out_dtype):
        self.P, self.r = dist.get_world_size(group), dist.get_rank(group)
        P = self.P
        n = P * B * S_l * Hl * D
        self.dtypes = (E4M3, E4M3, pv_dtype)
        self.shape = (P, B, S_l, Hl, D)
        self.out_dtype = out_dtype
        roles = {f"in{s}_{i}": n * torch.empty((), dtype=dt).element_size()
                 for s in range(2) for i, dt in enumerate(self.dtypes)}
        roles["out"] = n * torch.empty((), dtype=out_dtype).element_size()
        self.ptr = {role: _alloc(nb) for role, nb in roles.items()}
        self.nbytes = roles
        handles = {role: _handle(p) for role, p in self.ptr.items()}
        gathered = [None] * P
        dist.all_gather_object(gathered, handles, group=group)
        self.peer = {role: [self.ptr[role] if p == self.r else _open(gathered[p][role]) for p in range(P)]
                     for role in roles}
        self.tensor = {role: torch.as_tensor(_Raw(ptr, roles[role]), device=device) for role, ptr in self.ptr.items()}
        self.recv = [torch.empty(self.shape, dtype=dt, device=device) for dt in self.dtypes]
        self.flag = torch.zeros(1, dtype=torch.int32, device=device)
        # one copy stream per source rank, so the copy engines move the chunks concurrently
        self.copy_streams = [torch.cuda.Stream(device) for _ in range(P)]
        self.calls = 0

    def view(self, role: str, dtype) -> torch.Tensor:
        return self.tensor[role].view(dtype).view(self.shape)

    @classmethod
    def get(cls, group, device, B, S_l, Hl, D, pv_dtype, out_dtype):
        ranks = tuple(dist.get_process_group_ranks(group if group is not None else dist.group.WORLD))
        key = (ranks, str(device), B, S_l, Hl, D, pv_dtype, out_dtype)
        ent = cls._cache.get(key)
        if ent is None:
            ent = cls._cache[key] = cls(group, device, B, S_l, Hl, D, pv_dtype, out_dtype)
        return ent


def ulysses_attention_peer(q, k, v, group=None, scale=None, pv_dtype=torch.float16, out=None, cross_kv=None,
                           events=None, packing=None):
    """``ulysses_attention`` with the exchanges done by copy-engine pulls from peer buffers.

    Shards ``[1, S_local, H, D]`` (batch 1), one head group; same arguments
    and result as ``ulysses_attention`` (bit for bit: the same scales, bytes
    and kernel).  ``packing``: the ``ulysses._Packing`` of a packed batch
    (per-(sequence, head) scales, the varlen kernel over the global
    ``cu_seqlens``, rows outside every sequence zero).  Every rank of
    ``group`` must be a process on this node.
    """
    from . import ops

    P, r = dist.get_world_size(group), dist.get_rank(group)
    B, S_l, H, D = q.shape
    if B != 1:
        raise ValueError("the peer exchange takes batch-1 shards [1, S_local, H, D]")
    if H % P:
        raise ValueError(f"heads ({H}) must be divisible by the world size ({P})")
    for name, t in (("k", k), ("v", v)):
        if t.shape != q.shape or t.dtype != q.dtype:
            raise ValueError(f"{name} must be shaped and typed like q")
    Hl = H // P
    dev = q.device
    if out is None:
        out = torch.empty((B, S_l, H, D), dtype=q.dtype, device=dev)
    elif tuple(out.shape) != (B, S_l, H, D) or out.dtype != q.dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous tensor shaped and typed like q")
    bufs = _Buffers.get(group, dev, B, S_l, Hl, D, pv_dtype, q.dtype)
    s = bufs.calls % 2
    bufs.calls += 1
    ls2 = (scale if scale is not None else 1.0 / math.sqrt(D)) * LOG2E
    compute = torch.cuda.current_stream(dev)
    copies = bufs.copy_streams

    # 1-2: global per-(b,h) scales, quantisation into the exported send set s
    xs = (q, k, v)
    if packing is None:
        amax = torch.stack([ops.absmax_bh(x) for x in xs])                  # [3, B, H]
    else:
        amax = torch.stack([ops.absmax_seg(x, packing.seg) for x in xs])   # [3, nseq, H]
    dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=group)
    scales = ops.scale_from_absmax(amax)
    for i, (x, dt) in enumerate(zip(xs, bufs.dtypes)):
        dst = bufs.view(f"in{s}_{i}", dt)
        if packing is None:
            ops.quantize_bh(x, scales[i], out_dtype=dt, groups=P, out=dst)
        else:
            ops.quantize_seg(x, packing.seg, scales[i], out_dtype=dt, groups=P, out=dst)
    # 3: barrier A
    dist.all_reduce(bufs.flag, group=group)
    # 4: pull chunk r of every rank's send set (copy engines, one stream per source rank)
    chunk = B * S_l * Hl * D
    for p, cs in enumerate(copies):
        cs.wait_stream(compute)
        for i, dt in enumerate(bufs.dtypes):
            es = torch.empty((), dtype=dt).element_size()
            src = bufs.peer[f"in{s}_{i}"][p] + r * chunk * es
            _copy(bufs.recv[i].data_ptr() + p * chunk * es, Hl * D * es, src, Hl * D * es, Hl * D * es, B * S_l, cs)
    cross = None
    if cross_kv is not None:
        from .kernels.fp8_attention import fp8_attention

        kt, vt = cross_kv
        cross = fp8_attention(q.transpose(1, 2), kt, vt, scale=scale).transpose(1, 2)
    for cs in copies:
        compute.wait_stream(cs)
    # 5: attention over the local heads, into the exported output buffer
    mine = slice(r * Hl, (r + 1) * Hl)
    sq, sk, sv = (sc[:, mine].contiguous()[..., None] for sc in scales)
    hq, hk, hv = (t.view(P * S_l, Hl, D).permute(1, 0, 2).unsqueeze(0) for t in bufs.recv)
    send_o = bufs.view("out", q.dtype)
    ev = None
    if events is not None:
        ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        ev[0].record(compute)
    if packing is None:
        ops.attention_e4m3(hq, hk, hv, sq, sk, sv, logit_scale_log2=ls2, out_dtype=q.dtype,
                           out=send_o.view(P * S_l, Hl, D).permute(1, 0, 2).unsqueeze(0))
    else:
        # the received buffers are the packed [S, Hl, D] layout in global token order
        o_rows = send_o.view(P * S_l, Hl, D)
        ops.attention_e4m3(*(t.view(P * S_l, Hl, D) for t in bufs.recv), sq, sk, sv, logit_scale_log2=ls2,
                           out_dtype=q.dtype, cu_seqlens_q=packing.cu, cu_seqlens_k=packing.cu,
                           max_seqlen_q=packing.max_seqlen, out=o_rows)
        packing.clear_outside(o_rows)
    if ev is not None:
        ev[1].record(compute)
        events.append(ev)
    # 6: barrier B
    dist.all_reduce(bufs.flag, group=group)
    # 7: pull chunk r of every rank's output straight into this rank's heads of out
    es = q.element_size()
    row = Hl * D * es
    for p, cs in enumerate(copies):
        cs.wait_stream(compute)
        src = bufs.peer["out"][p] + r * chunk * es
        _copy(out.data_ptr() + p * row, H * D * es, src, row, row, B * S_l, cs)
    for cs in copies:
        compute.wait_stream(cs)
    return out if cross_kv is None else (out, cross)
