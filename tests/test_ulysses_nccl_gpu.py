"""Ulysses over NCCL on 2 GPUs: bit-identical to one GPU over the whole sequence,
for every head grouping of the pipeline, for the host-resident variant and
for sequences packed with global cu_seqlens (against the drop-in varlen path).

Every rank quantises with the global per-(batch, head) scales, so the head
shard each rank attends over holds exactly the bytes a single GPU would use;
the kernel then computes each head independently.  Skipped with fewer than
two GPUs.  NVLS is switched off (plain NCCL peer transfers).
"""
import math
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(B, S, H, D):
    g = torch.Generator().manual_seed(3)
    xs = []
    for _ in range(3):
        x = torch.randn(B, S, H, D, generator=g)
        x[..., 7] *= 8.0
        xs.append(x.to(torch.bfloat16))
    return xs


# sequences packed along S (global offsets): one crosses the rank boundary, the last 40 rows lie outside
PACKED_CU = [0, 1000, 2900, 3800]


def _packed_single_gpu(q, k, v, cu):
    """The drop-in varlen path on one GPU over the whole packed sequence; rows outside every sequence zeroed."""
    from minimaxh3_b200.kernels.fp8_attention import fp8_attention_varlen

    cut = torch.tensor(cu, dtype=torch.int32, device=q.device)
    o = fp8_attention_varlen(q[0], k[0], v[0], cut, cut, max(b - a for a, b in zip(cu, cu[1:])))
    o[:cu[0]] = 0
    o[cu[-1]:] = 0
    return o[None]


def _worker(rank, world, port, shape, out_dir):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from minimaxh3_b200.kernels.fp8_attention import fp8_attention
        from minimaxh3_b200.ulysses import ulysses_attention, ulysses_attention_host

        B, S, H, D = shape
        q, k, v = (t.cuda() for t in _inputs(B, S, H, D))
        Sl = S // world
        sl = slice(rank * Sl, (rank + 1) * Sl)
        shard = [t[:, sl].contiguous() for t in (q, k, v)]
        outs = {G: ulysses_attention(*shard, head_groups=G) for G in (1, 2, 4)}
        packed = {G: ulysses_attention(*shard, head_groups=G, cu_seqlens=PACKED_CU) for G in (1, 2)}
        packed_peer = [ulysses_attention(*shard, cu_seqlens=PACKED_CU, exchange="peer") for _ in range(2)]
        # host-resident shards, with the cross-attention to replicated text K/V per head group
        gt = torch.Generator().manual_seed(11)
        kt, vt = (torch.randn(B, H, 256, D, generator=gt).to(torch.bfloat16).cuda() for _ in range(2))
        hq, hk, hv = (t.cpu().pin_memory() for t in shard)
        ho, hc = ulysses_attention_host(hq, hk, hv, head_groups=2, cross_kv=(kt, vt))
        cross = fp8_attention(shard[0].transpose(1, 2), kt, vt).transpose(1, 2)
        # the device path with the cross-attention issued during the first exchange
        dev_o, dev_c = ulysses_attention(*shard, head_groups=2, cross_kv=(kt, vt))
        # the copy-engine exchange through the peers' mapped buffers (both send sets)
        peer = [ulysses_attention(*shard, exchange="peer", cross_kv=(kt, vt)) for _ in range(3)]
        torch.cuda.synchronize()
        hp = ulysses_attention_host(hq, hk, hv, head_groups=2, cu_seqlens=PACKED_CU)
        torch.cuda.synchronize()
        torch.save({"out": {G: o.cpu() for G, o in outs.items()}, "host": ho.clone(), "host_cross": hc.clone(),
                    "cross": cross.cpu(), "packed": {G: o.cpu() for G, o in packed.items()},
                    "host_packed": hp.clone(), "dev_cross": (dev_o.cpu(), dev_c.cpu()),
                    "peer": [(o.cpu(), c.cpu()) for o, c in peer], "packed_peer": [o.cpu() for o in packed_peer]},
                   os.path.join(out_dir, f"out{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ulysses_two_gpus_bit_identical(tmp_path):
    from minimaxh3_b200 import ops

    B, S, H, D = 1, 2 * 1920, 8, 128
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, (B, S, H, D), str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    res = [torch.load(tmp_path / f"out{r}.pt") for r in range(2)]
    got = torch.cat([x["out"][1] for x in res], dim=1)
    for x in res:
        for G in (2, 4):                       # head-group pipeline: same bytes
            assert torch.equal(x["out"][G], x["out"][1])
        assert torch.equal(x["host"], x["out"][1])         # host-resident variant
        assert torch.equal(x["host_cross"], x["cross"])    # its per-group cross-attention
        assert torch.equal(x["dev_cross"][0], x["out"][1])  # device path with cross_kv
        assert torch.equal(x["dev_cross"][1], x["cross"])
        for o, c in x["peer"]:                              # copy-engine exchange
            assert torch.equal(o, x["out"][1]) and torch.equal(c, x["cross"])
    # one GPU, whole sequence, same global per-(b,h) scales
    q, k, v = (t.cuda() for t in _inputs(B, S, H, D))
    ops_in = []
    scales = []
    for x, dt in ((q, torch.float8_e4m3fn), (k, torch.float8_e4m3fn), (v, torch.float16)):
        s = (torch.clamp(x.float().abs().amax(dim=(1, 3)), min=1e-12).double() / 448.0).float()
        y = x.float() / s[:, None, :, None]
        if dt == torch.float8_e4m3fn:
            y = torch.clamp(y, -448, 448)
        ops_in.append(y.to(dt).permute(0, 2, 1, 3).contiguous())
        scales.append(s[..., None].contiguous())
    ref = ops.attention_e4m3(*ops_in, *scales, logit_scale_log2=1.4426950408889634 / math.sqrt(D))
    ref = ref.permute(0, 2, 1, 3).cpu()
    assert torch.equal(got, ref)
    # packed sequences: global cu_seqlens, per-(sequence, head) scales reduced over the ranks
    packed_ref = _packed_single_gpu(q, k, v, PACKED_CU).cpu()
    for G in (1, 2):
        assert torch.equal(torch.cat([x["packed"][G] for x in res], dim=1), packed_ref)
    assert torch.equal(torch.cat([x["host_packed"] for x in res], dim=1), packed_ref)
    for i in range(2):                                       # copy-engine exchange, packed
        assert torch.equal(torch.cat([x["packed_peer"][i] for x in res], dim=1), packed_ref)


def _single_rank_worker(port, out_dir):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(0)
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", 0))
    try:
        from minimaxh3_b200.kernels.fp8_attention import fp8_attention
        from minimaxh3_b200.ulysses import ulysses_attention, ulysses_attention_host

        B, S, H, D = 1, 1000, 8, 128
        q, k, v = (t.cuda() for t in _inputs(B, S, H, D))
        gt = torch.Generator().manual_seed(11)
        kt, vt = (torch.randn(B, H, 256, D, generator=gt).to(torch.bfloat16).cuda() for _ in range(2))
        dev_out = ulysses_attention(q, k, v)
        cross = fp8_attention(q.transpose(1, 2), kt, vt).transpose(1, 2)
        dev_o, dev_c = ulysses_attention(q, k, v, head_groups=4, cross_kv=(kt, vt))
        peer = [ulysses_attention(q, k, v, exchange="peer", cross_kv=(kt, vt)) for _ in range(3)]
        hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
        res = []
        for G in (4, 4, 2):                      # the second call reuses the first one's device buffers
            o, c = ulysses_attention_host(hq, hk, hv, head_groups=G, cross_kv=(kt, vt))
            torch.cuda.synchronize()
            res.append((o.clone(), c.clone()))
        cu = [0, 400, 400, 900]                  # an empty sequence; rows 900.. outside every sequence
        packed = ulysses_attention(q, k, v, cu_seqlens=cu)
        packed_peer = ulysses_attention(q, k, v, cu_seqlens=cu, exchange="peer")
        packed_host = ulysses_attention_host(hq, hk, hv, head_groups=2, cu_seqlens=torch.tensor(cu))
        torch.cuda.synchronize()
        torch.save({"dev": dev_out.cpu(), "cross": cross.cpu(), "host": res, "packed": packed.cpu(),
                    "dev_cross": (dev_o.cpu(), dev_c.cpu()), "peer": [(o.cpu(), c.cpu()) for o, c in peer],
                    "packed_peer": packed_peer.cpu(),
                    "packed_host": packed_host.clone(), "packed_ref": _packed_single_gpu(q, k, v, cu).cpu()},
                   os.path.join(out_dir, "single.pt"))
    finally:
        dist.destroy_process_group()


def test_host_resident_pipeline_on_one_rank(tmp_path):
    """ulysses_attention_host on a one-rank NCCL group equals the device path and per-group
    cross-attention bit for bit, also when a call reuses the previous call's device buffers;
    with cu_seqlens both equal ``fp8_attention_varlen``."""
    ctx = mp.get_context("spawn")
    p = ctx.Process(target=_single_rank_worker, args=(_free_port(), str(tmp_path)))
    p.start()
    p.join(timeout=300)
    assert p.exitcode == 0
    r = torch.load(tmp_path / "single.pt")
    for o, c in r["host"]:
        assert torch.equal(o, r["dev"])
        assert torch.equal(c, r["cross"])
    assert torch.equal(r["dev_cross"][0], r["dev"]) and torch.equal(r["dev_cross"][1], r["cross"])
    for o, c in r["peer"]:
        assert torch.equal(o, r["dev"]) and torch.equal(c, r["cross"])
    assert torch.equal(r["packed"], r["packed_ref"])          # Ulysses with cu_seqlens = the drop-in varlen path
    assert torch.equal(r["packed_peer"], r["packed_ref"])
    assert torch.equal(r["packed_host"], r["packed_ref"])
    assert torch.count_nonzero(r["packed"][0, 900:]) == 0
