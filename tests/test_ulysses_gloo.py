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
        s = torch.clamp(x.float().abs().amax(dim=(1, 3)), min=1e-12) / 448.0   # [B,H]
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
