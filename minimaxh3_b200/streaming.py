"""FP8 attention over host-resident (pinned) tensors, streamed through the GPU.

For callers whose q, k, v live in host memory - activations offloaded
between denoising steps, or a host-side service feeding the model -
``fp8_attention_host`` copies (batch, head-range) chunks to the device, runs
the drop-in ``fp8_attention`` on each chunk and copies the result back.  The
three stages run on three CUDA streams with two device buffers per stage, so
the host->device copy of chunk i+1, the quantisation + attention of chunk i
and the device->host copy of chunk i-1 overlap; a step costs about the
slower of the PCIe transfer and the compute instead of their sum.  The
input buffers persist across calls (per device, compute stream and shape),
so back-to-back calls also overlap at their boundary.

Every quantity of the reference's algorithm is per (batch, head): Q and K
scales per 128-row block of one head, the K channel mean and V's per-channel
scales over one head's keys (kernels/fp8_attention.py:39-170, :338).  The
chunked result therefore equals one ``fp8_attention`` call over the whole
tensors, bit for bit.
"""
from __future__ import annotations

import threading

import torch

from .kernels.fp8_attention import fp8_attention


def _chunks(B: int, H: int, heads_per_chunk: int):
    for b in range(B):
        for h0 in range(0, H, heads_per_chunk):
            yield b, h0, min(H, h0 + heads_per_chunk)


def fp8_attention_host(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    out: torch.Tensor | None = None,
    scale: float | None = None,
    key_mask: torch.Tensor | None = None,
    key_bias: torch.Tensor | None = None,
    heads_per_chunk: int | None = None,
    device: torch.device | int | None = None,
) -> torch.Tensor:
    """``fp8_attention`` of host tensors ``[B, H, S, D]`` into a host tensor.

    q, k, v: contiguous CPU tensors (bf16 or f16; pinned, or the copies are
    synchronous).  ``out``: contiguous CPU tensor shaped like q (allocated
    pinned when None).  key_mask / key_bias: ``[B, Sk]`` (any device).  The
    work is enqueued on ``device``'s current stream, which is made to wait for
    the last copy back: ``out`` is valid once that stream is synchronised.
    """
    for name, t in (("q", q), ("k", k), ("v", v)):
        if t.device.type != "cpu" or t.dim() != 4 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous 4-D CPU tensor")
    if k.shape != v.shape or q.shape[0] != k.shape[0] or q.shape[1] != k.shape[1] or q.shape[3] != k.shape[3]:
        raise ValueError("q, k, v shapes do not match [B, H, S, D]")
    B, H = q.shape[:2]
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
    elif out.shape != q.shape or out.dtype != q.dtype or out.device.type != "cpu" or not out.is_contiguous():
        raise ValueError("out must be a contiguous CPU tensor shaped like q")
    if device is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    else:
        dev = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
    hc = heads_per_chunk or max(1, min(H, -(-B * H // 40)))  # about 40 chunks (measured best)
    with torch.cuda.device(dev):
        _run(q, k, v, out, scale, key_mask, key_bias, hc, dev)
    return out


class _ChunkBuffers:
    """Two device buffer sets (q, k, v chunks) per (device, dtype, shapes), kept across calls,
    each with the event after the last attention that read it.  A call's first input copies
    wait only for those events, so they overlap the previous call's last chunks; buffers that
    came from the caching allocator instead would first have to wait for everything queued on
    the compute stream (memory freed there may still be read)."""

    _pool: dict = {}
    _lock = threading.Lock()

    @classmethod
    def get(cls, key, make):
        with cls._lock:
            ent = cls._pool.get(key)
            if ent is None:
                ent = {"bufs": [make() for _ in range(2)], "free": [None, None]}
                if len(cls._pool) >= 8:          # bound the cache: drop the oldest shape
                    cls._pool.pop(next(iter(cls._pool)))
                cls._pool[key] = ent
            return ent


def _run(q, k, v, out, scale, key_mask, key_bias, hc, dev):
    B, H, Sq, D = q.shape
    Sk = k.shape[2]
    s_cmp = torch.cuda.current_stream(dev)
    s_in = torch.cuda.Stream(dev)
    s_out = torch.cuda.Stream(dev)
    km = key_mask.to(dev, non_blocking=True) if key_mask is not None else None
    kb = key_bias.to(dev, non_blocking=True) if key_bias is not None else None
    key = (dev.index, s_cmp.cuda_stream, q.dtype, hc, Sq, Sk, D)  # one buffer pair per compute stream
    ent = _ChunkBuffers.get(key, lambda: tuple(torch.empty((1, hc, S, D), dtype=q.dtype, device=dev)
                                               for S in (Sq, Sk, Sk)))
    for i, (b, h0, h1) in enumerate(_chunks(B, H, hc)):
        n = h1 - h0
        j = i % 2
        dq, dk, dv = (x[:, :n] for x in ent["bufs"][j])
        with torch.cuda.stream(s_in):
            if ent["free"][j] is not None:
                s_in.wait_event(ent["free"][j])  # the last attention that read this set is done
            dq[0].copy_(q[b, h0:h1], non_blocking=True)
            dk[0].copy_(k[b, h0:h1], non_blocking=True)
            dv[0].copy_(v[b, h0:h1], non_blocking=True)
        s_cmp.wait_stream(s_in)
        o = fp8_attention(dq, dk, dv, scale=scale,
                          key_mask=None if km is None else km[b:b + 1],
                          key_bias=None if kb is None else kb[b:b + 1])
        ev = torch.cuda.Event()
        ev.record(s_cmp)
        ent["free"][j] = ev
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev)
            out[b, h0:h1].copy_(o[0], non_blocking=True)
        o.record_stream(s_out)
    s_cmp.wait_stream(s_out)
