"""Ulysses head-parallel plumbing on CPU gloo ranks (world sizes 2 and 4).

The scale all-reduce, the e4m3/f16 packing, both all-to-alls and the head
interleave run exactly as on NCCL; the attention kernel is replaced by the
float64 oracle on the dequantised operands, so the sharded result must equal
one process computing attention over the whole sequence with the same
global per-(batch, head) scales.
"""
import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import fp8_attention_ref as OA


def _oracle_attn(q8, k8, v, sq, sk, sv, ls2):
    qd = q8.double() * sq.double()[..., None]
    kd = k8.double() * sk.double()[..., None]
    vd = v.double() * sv.double()[..., None]
    return OA.sdpa_dequant_oracle(qd, kd, vd, ls2, base2=True)


def _selected(H, groups, head_off, heads_sel):
    """Heads p*(H/groups) + head_off + i, in the order mh3_absmax_bh / mh3_quantize_bh number them."""
    hb = H // groups
    hs = hb - head_off if heads_sel is None else heads_sel
    return [p * hb + head_off + i for p in range(groups) for i in range(hs)], hs


def _oracle_absmax(x, groups=1, head_off=0, heads_sel=None):
    heads, _ = _selected(x.shape[2], groups, head_off, heads_sel)
    return x.float().abs().amax(dim=(1, 3))[:, heads]


def _oracle_quant(x, scale, P, out_dtype, head_off=0, heads_sel=None):
    """Restatement of mh3_quantize_bh: x [B,S_l,H,D] selected heads / scale[B, P*hs] -> [P, B, S_l, hs, D]."""
    B, S_l, H, D = x.shape
    heads, hs = _selected(H, P, head_off, heads_sel)
    y = x[:, :, heads].float() / scale[:, None, :, None]
    if out_dtype == torch.float8_e4m3fn:
        y = torch.clamp(y, -448.0, 448.0)
    y = y.to(out_dtype)
    return y.reshape(B, S_l, P, hs, D).permute(2, 0, 1, 3, 4).contiguous()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(B, S, H, D):
    g = torch.Generator().manual_seed(0)
    return [torch.randn(B, S, H, D, generator=g).to(torch.bfloat16) for _ in range(3)]


def _worker(rank, world, port, B, S, H, D, pv, out_dir, head_groups=1):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from minimaxh3_b200.ulysses import ulysses_attention

        q, k, v = _inputs(B, S, H, D)
        Sl = S // world
        sl = slice(rank * Sl, (rank + 1) * Sl)
        out = ulysses_attention(q[:, sl], k[:, sl], v[:, sl], pv_dtype=pv, attn_fn=_oracle_attn,
                                absmax_fn=_oracle_absmax, quant_fn=_oracle_quant, head_groups=head_groups)
        torch.save(out, os.path.join(out_dir, f"out{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _reference(B, S, H, D, pv):
    """Whole-sequence attention with the same per-(b,h) quantisation."""
    q, k, v = _inputs(B, S, H, D)
    outs = []
    scales = []
    for x, dt in ((q, torch.float8_e4m3fn), (k, torch.float8_e4m3fn), (v, pv)):
        s = (torch.clamp(x.float().abs().amax(dim=(1, 3)), min=1e-12).double() / 448.0).float()   # [B,H]
        y = x.float() / s[:, None, :, None]
        if dt == torch.float8_e4m3fn:
            y = torch.clamp(y, -448, 448)
        outs.append(y.to(dt).permute(0, 2, 1, 3))                                # [B,H,S,D]
        scales.append(s[..., None])
    o = _oracle_attn(*outs, *scales, OA.LOG2E / math.sqrt(D))
    return o.to(torch.bfloat16).permute(0, 2, 1, 3)


@pytest.mark.parametrize("world,pv,head_groups,B", [(2, torch.float16, 1, 1), (4, torch.float8_e4m3fn, 1, 1),
                                                    (2, torch.float16, 4, 1), (2, torch.float16, 2, 2),
                                                    (4, torch.float8_e4m3fn, 2, 1)])
def test_ulysses_matches_single_process(tmp_path, world, pv, head_groups, B):
    """Any head grouping of the pipeline gives the single-process result (every quantity is per head)."""
    S, H, D = 64 * world, 8, 64
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, B, S, H, D, pv, str(tmp_path), head_groups))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0
    got = torch.cat([torch.load(tmp_path / f"out{r}.pt") for r in range(world)], dim=1)
    ref = _reference(B, S, H, D, pv)
    assert got.shape == ref.shape
    r = OA.compare(got.float(), ref.float())
    assert r["cos"] > 0.99999 and r["max_abs"] < 1e-2, r


def test_ulysses_rejects_indivisible_heads(tmp_path):
    port = _free_port()
    # heads=6 over 4 ranks, and 3 groups of 2 heads per rank, are rejected before any collective
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_bad_worker, args=(r, 4, port, str(tmp_path))) for r in range(4)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0


def _bad_worker(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from minimaxh3_b200.ulysses import ulysses_attention

        x = torch.zeros(1, 8, 6, 64, dtype=torch.bfloat16)
        with pytest.raises(ValueError):
            ulysses_attention(x, x, x, attn_fn=_oracle_attn, absmax_fn=_oracle_absmax, quant_fn=_oracle_quant)
        x = torch.zeros(1, 8, 8, 64, dtype=torch.bfloat16)             # 2 heads per rank, 3 groups
        with pytest.raises(ValueError):
            ulysses_attention(x, x, x, attn_fn=_oracle_attn, absmax_fn=_oracle_absmax, quant_fn=_oracle_quant,
                              head_groups=3)
    finally:
        dist.destroy_process_group()


# --- packed variable-length batches (cu_seqlens global, per-(sequence, head) scales) ----------------------------


def _bounds(seg, S):
    return [min(max(int(c), 0), S) for c in seg.tolist()]


def _oracle_absmax_seg(x, groups=1, head_off=0, heads_sel=None, seg=None):
    """Restatement of mh3_absmax_seg: [nseq, nsel] over the shard rows of each segment (0 when empty)."""
    x = x[0]
    heads, _ = _selected(x.shape[1], groups, head_off, heads_sel)
    b = _bounds(seg, x.shape[0])
    rows = [x[lo:max(lo, hi), heads].float().abs() for lo, hi in zip(b, b[1:])]
    return torch.stack([r.amax(dim=(0, 2)) if r.shape[0] else torch.zeros(len(heads)) for r in rows])


def _oracle_quant_seg(x, scale, P, out_dtype, head_off=0, heads_sel=None, seg=None):
    """Restatement of mh3_quantize_seg: rows of segment z / scale[z]; zeros outside every segment."""
    x = x[0]
    S, H, D = x.shape
    heads, hs = _selected(H, P, head_off, heads_sel)
    b = _bounds(seg, S)
    y = torch.zeros(S, len(heads), D)
    for z, (lo, hi) in enumerate(zip(b, b[1:])):
        if hi > lo:
            y[lo:hi] = x[lo:hi, heads].float() / scale[z][None, :, None]
    if out_dtype == torch.float8_e4m3fn:
        y = torch.clamp(y, -448.0, 448.0)
    return y.to(out_dtype).reshape(1, S, P, hs, D).permute(2, 0, 1, 3, 4).contiguous()


def _oracle_attn_varlen(q8, k8, v, sq, sk, sv, ls2, cu_seqlens=None, max_seqlen=0):
    """Float64 attention inside each packed sequence of [T, Hg, D] operands, scales [nseq, Hg, 1]."""
    cu = cu_seqlens.tolist()
    o = torch.zeros(q8.shape, dtype=torch.float64)
    for z, (a, b) in enumerate(zip(cu, cu[1:])):
        if b > a:
            deq = [(t[a:b].double() * s[z].double()[None]).permute(1, 0, 2)[None]
                   for t, s in ((q8, sq), (k8, sk), (v, sv))]
            o[a:b] = OA.sdpa_dequant_oracle(*deq, ls2, base2=True)[0].permute(1, 0, 2)
    return o


def _packed_worker(rank, world, port, S, H, D, cu, pv, out_dir, head_groups):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from minimaxh3_b200.ulysses import ulysses_attention

        q, k, v = _inputs(1, S, H, D)
        Sl = S // world
        sl = slice(rank * Sl, (rank + 1) * Sl)
        out = ulysses_attention(q[:, sl], k[:, sl], v[:, sl], pv_dtype=pv, attn_fn=_oracle_attn_varlen,
                                absmax_fn=_oracle_absmax_seg, quant_fn=_oracle_quant_seg, head_groups=head_groups,
                                cu_seqlens=cu)
        torch.save(out, os.path.join(out_dir, f"out{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _packed_reference(S, H, D, cu, pv):
    """One process: per-(sequence, head) scales over whole sequences, attention inside each."""
    q, k, v = (t[0] for t in _inputs(1, S, H, D))
    seg = torch.tensor(cu, dtype=torch.int32)
    ops_in, scales = [], []
    for x, dt in ((q, torch.float8_e4m3fn), (k, torch.float8_e4m3fn), (v, pv)):
        s = (torch.clamp(_oracle_absmax_seg(x[None], seg=seg), min=1e-12).double() / 448.0).float()  # [nseq, H]
        ops_in.append(_oracle_quant_seg(x[None], s, 1, dt, seg=seg)[0, 0])
        scales.append(s[..., None])
    o = _oracle_attn_varlen(*ops_in, *scales, OA.LOG2E / math.sqrt(D), cu_seqlens=seg)
    return o.to(torch.bfloat16)[None]


@pytest.mark.parametrize("world,cu,pv,head_groups", [
    (2, [0, 50, 100, 120], torch.float16, 1),             # a sequence across the rank boundary; 8 rows outside
    (4, [0, 0, 97, 256], torch.float16, 2),               # an empty sequence; head groups
    (2, [10, 128], torch.float8_e4m3fn, 2),               # rows before the first sequence; e4m3 PV
])
def test_packed_ulysses_matches_single_process(tmp_path, world, cu, pv, head_groups):
    """Sequences packed along S keep global cu_seqlens: the sharded result equals one process
    attending inside each sequence with per-(sequence, head) scales; rows outside are zeros."""
    S, H, D = 64 * world, 8, 64
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_packed_worker, args=(r, world, port, S, H, D, cu, pv, str(tmp_path), head_groups))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0
    got = torch.cat([torch.load(tmp_path / f"out{r}.pt") for r in range(world)], dim=1)
    ref = _packed_reference(S, H, D, cu, pv)
    assert got.shape == ref.shape
    outside = torch.ones(S, dtype=torch.bool)
    outside[cu[0]:cu[-1]] = False
    assert torch.count_nonzero(got[0, outside]) == 0
    r = OA.compare(got.float(), ref.float())
    assert r["cos"] > 0.99999 and r["max_abs"] < 1e-2, r


def test_packed_ulysses_rejects_bad_offsets(tmp_path):
    from minimaxh3_b200.ulysses import _Packing

    with pytest.raises(ValueError):
        _Packing([0, 70, 60], 2, 0, 64, "cpu")              # decreasing
    with pytest.raises(ValueError):
        _Packing([0, 129], 2, 0, 64, "cpu")                 # past P * S_local
    with pytest.raises(ValueError):
        _Packing([0], 2, 0, 64, "cpu")
    pk = _Packing([5, 70, 100], 2, 1, 64, "cpu")
    assert pk.seg.tolist() == [0, 6, 36] and pk.cu.tolist() == [5, 70, 100] and pk.max_seqlen == 65
