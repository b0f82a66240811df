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


def _oracle_absmax(x):
    return x.float().abs().amax(dim=(1, 3))


def _oracle_quant(x, scale, P, out_dtype):
    """Restatement of mh3_quantize_bh: x [B,S_l,H,D] / scale[B,H] -> [P, B, S_l, H/P, D]."""
    B, S_l, H, D = x.shape
    y = x.float() / scale[:, None, :, None]
    if out_dtype == torch.float8_e4m3fn:
        y = torch.clamp(y, -448.0, 448.0)
    y = y.to(out_dtype)
    return y.reshape(B, S_l, P, H // P, D).permute(2, 0, 1, 3, 4).contiguous()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(B, S, H, D):
    g = torch.Generator().manual_seed(0)
    return [torch.randn(B, S, H, D, generator=g).to(torch.bfloat16) for _ in range(3)]


def _worker(rank, world, port, B, S, H, D, pv, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from minimaxh3_b200.ulysses import ulysses_attention

        q, k, v = _inputs(B, S, H, D)
        Sl = S // world
        sl = slice(rank * Sl, (rank + 1) * Sl)
        out = ulysses_attention(q[:, sl], k[:, sl], v[:, sl], pv_dtype=pv, attn_fn=_oracle_attn,
                                absmax_fn=_oracle_absmax, quant_fn=_oracle_quant)
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


@pytest.mark.parametrize("world,pv", [(2, torch.float16), (4, torch.float8_e4m3fn)])
def test_ulysses_matches_single_process(tmp_path, world, pv):
    B, S, H, D = 1, 64 * world, 8, 64
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, B, S, H, D, pv, str(tmp_path))) for r in range(world)]
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
    # heads=6 over 4 ranks is rejected before any collective
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
    finally:
        dist.destroy_process_group()
