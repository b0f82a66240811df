"""Benchmark of the MiniMax-H3 FP8 attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mh3|reference]

Default arm (``--impl mh3``), N=1: benchmark configuration 2 - FP8 self-attention
forward, B=1 H=40 S=32760 D=128, e4m3 q/k/v with per-(batch, head) scales
(synthetic N(0,1) with one of 128 channels x8, seed 0), bf16 out.  With the
default 16-bit PV product (``--pv f16``) a step is one exact e4m3->f16
widening of V plus one ``mh3_fp8_attention_fwd`` launch; with ``--pv e4m3``
it is the attention launch alone.  ``value`` is whole-job TFLOP/s
(4*B*H*S^2*D per step) with inputs resident in HBM (504 MB of e4m3 inputs,
larger than the 126 MB L2).  ``e2e`` times
``minimaxh3_b200.streaming.fp8_attention_host`` on pinned host bf16 q/k/v
(1.0 GB in, 0.34 GB out per step): head chunks are copied in, quantised and
attended by the drop-in ``fp8_attention``, and copied back, with the three
stages overlapping on separate streams.

N>1 (torchrun): benchmark configuration 5, the sharded configuration - S=75600 H=40
D=128 self-attention with Ulysses head parallelism (per-(b,h) scales
all-reduced, e4m3 q/k and f16 v exchanged, local FP8 attention over H/N
heads, bf16 back) plus cross-attention of the local query shard to 512
replicated text tokens, issued while the input exchange runs.  The exchange
is copy-engine pulls from the peers' buffers mapped through CUDA IPC
(``--exchange peer``, default) or NCCL all-to-alls (``--exchange nccl``).
``value`` = total FLOPs of both attentions / max-over-ranks device time
("strong" scaling: total work fixed).

The N=1 line also carries, measured after its timed regions on the same
box: ``competitor_same_box`` - the reference's own Triton attention
(``_fp8_attn_kernel`` alone, and ``fp8_attention`` end to end, from the
unmodified copy that baseline/install_reference.py places in baseline/_ref)
against this package's, 3 warm-ups then the median of 20; and ``extras`` -
config 4 (FP8 linear, incl. the reference's ``FP8Linear`` module), config 3
(varlen), a synthetic DiT block and config 5 on one GPU.  The N>1 line
carries config 5 on rank 0's GPU alone (``n1_same_workload``).

``--impl reference``: the reference's CPU implementation of this path
(``routed_sdpa`` falling back to torch SDPA on CPU tensors,
kernels/attention_router.py:93-102) on rank 0's host cores, on a bounded
sample of the same workload (one head, a block of query rows against all
32760 keys), same metric and unit.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

B, H, S, D = 1, 40, 32760, 128
LOG2E_ = 1.4426950408889634
NOMINAL_FP8_TFLOPS = 4500.0


# DRAM bytes (read + write) of one config-2 attention launch from the ncu
# capture summarised in profiles/attn_fwd_config2.md: H=8 measured
# (134.7 MB read + 43.6 MB write), scaled to H=40 by the heads processed
# (each (batch, head) is an independent set of CTAs reading its own Q, K, V).
ATTN_TRAFFIC_BYTES_H40 = {"f16": 5 * (134.672e6 + 43.554e6)}


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            mp = json.load(f)
        return {"fp8_tflops": 2.0 * float(mp["bf16_tflops"]), "hbm_gbs": float(mp["hbm_gbs"]),
                "source": "2x measured bf16 dense burst (MEASURED_PEAKS.json)"}
    except Exception:
        return {"fp8_tflops": 2.0 * 1590.0, "hbm_gbs": 6650.0, "source": "2x fallback bf16 1.59 PF"}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region.

    Samples every ``period_ms``; ``__enter__`` returns once the first sample
    has arrived, so sampling covers the whole region even when it is short
    (that first sample is taken just before the region starts).  Enter it
    before the barrier that starts the timed region: the wait for the first
    sample differs between processes.  ``enabled=False`` (ranks whose clocks
    are not reported) samples nothing."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int, period_ms: int = 50, enabled: bool = True):
        self.index = index
        self.period_ms = period_ms
        self.enabled = enabled
        self.proc = None
        self.lines = []

    def _read(self):
        for ln in self.proc.stdout:
            if ln.strip():
                self.lines.append(ln)
                self._first.set()

    def __enter__(self):
        import threading

        self.lines = []
        self._first = threading.Event()
        if not self.enabled:
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", str(self.period_ms)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._reader = threading.Thread(target=self._read, daemon=True)
            self._reader.start()
            # sampling is running before the timed region starts (nvidia-smi takes a while to come up)
            self._first.wait(timeout=5.0)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self._reader.join(timeout=5)

    def summary(self):
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws > 1:
        import datetime

        import torch.distributed as dist

        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        # NCCL may print a version banner on stdout when it creates the
        # communicator (eagerly here: device_id is given); stdout carries only
        # the result line, so fd 1 points at stderr until the first collective
        # has run and C-level buffers are flushed.
        import ctypes

        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
            dist.barrier()
        finally:
            ctypes.CDLL(None).fflush(None)
            os.dup2(saved, 1)
            os.close(saved)
        return dist, dist.get_rank(), ws, local
    return None, 0, 1, 0


def _synthetic_qkv(device, seed=0, dtype=torch.bfloat16):
    """q, k, v ~ N(0,1) bf16 with one (1% of 128) channel x8 per tensor."""
    g = torch.Generator(device=device).manual_seed(seed)
    gc = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(3):
        x = torch.randn(B, H, S, D, generator=g, device=device, dtype=torch.float32)
        ch = int(torch.randperm(D, generator=gc)[0])
        x[..., ch] *= 8.0
        out.append(x.to(dtype))
        del x
    return out


def _per_bh_e4m3(x):
    xf = x.float()
    s = torch.clamp(xf.abs().amax(dim=(2, 3)), min=1e-12) / 448.0
    x8 = torch.clamp(xf / s[..., None, None], -448, 448).to(torch.float8_e4m3fn)
    return x8, s[..., None].contiguous()


REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def _reference_kernels():
    """The reference's own ``kernels`` package (unmodified copy placed in baseline/_ref by
    baseline/install_reference.py): its Triton FP8 attention and FP8 linear."""
    if not os.path.isfile(os.path.join(REF_DIR, "kernels", "fp8_attention.py")):
        raise FileNotFoundError("baseline/_ref has no reference copy (run baseline/install_reference.py)")
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import importlib

    return importlib.import_module("kernels.fp8_attention"), importlib.import_module("kernels.fp8_linear")


def _reference_cpu_path():
    """``(fn, kind, source)``: the reference's CPU path for attention.

    With the unmodified copy in baseline/_ref, the reference's own
    ``routed_sdpa`` inside its ``denoiser_scope`` (kernels/attention_router.py:
    56-102,133-139): on CPU tensors ``is_supported`` is false and it takes its
    torch SDPA fallback (``kind`` "reference").  Without the copy, the
    oracle's restatement of that fallback (``kind`` "port").
    """
    try:
        _reference_kernels()  # puts baseline/_ref on sys.path (raises without the copy)
        import importlib

        router = importlib.import_module("kernels.attention_router")

        def fn(q, k, v):
            with router.denoiser_scope():
                return router.routed_sdpa(q, k, v)

        return fn, "reference", "baseline/_ref kernels/attention_router.py routed_sdpa (unmodified; CPU tensors " \
                                "take its torch SDPA fallback)"
    except Exception:  # noqa: BLE001 - no reference copy, or it does not import here
        from oracle.router_ref import cpu_sdpa_fallback

        return cpu_sdpa_fallback, "port", "oracle/router_ref.py cpu_sdpa_fallback (attention_router.py:93-102)"


def _median_ms(fn, stream, warmup=3, reps=20):
    """The competitor protocol: warm-ups, then the median of CUDA-event timings."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn()
        e1.record(stream)
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    return statistics.median(ts)


def triton_competitor(q, k, v, stream):
    """The reference's GPU path on the same box and inputs (the first named competitor).

    (i) ``_fp8_attn_kernel`` alone - autotuned, warp-specialised on cc 10 - on
    the operands its own wrapper makes (kernels/fp8_attention.py:300-402),
    against this package's attention kernel on the drop-in path's operands
    (per-128-row Q/K scales, f16 V/scale_v); (ii) ``fp8_attention(q, k, v)``
    end to end on device-resident bf16 inputs, reference against this
    package's drop-in.  3 warm-ups (the first call autotunes), median of 20.
    """
    import triton

    from minimaxh3_b200 import ops
    from minimaxh3_b200.kernels.fp8_attention import fp8_attention as mh3_fp8_attention

    RF, _ = _reference_kernels()
    Bq, Hq, Sq, Dq = q.shape
    flop = 4.0 * Bq * Hq * Sq * k.shape[2] * Dq
    res = {"source": "viragadel6/minimaxh3 kernels/fp8_attention.py, unmodified copy in baseline/_ref",
           "protocol": "3 warm-ups (autotune on the first), median of 20 CUDA-event timings",
           "inputs": "the headline workload's bf16 q, k, v on the device"}
    res["triton_ref_e2e_ms"] = _median_ms(lambda: RF.fp8_attention(q, k, v), stream)
    res["mh3_e2e_ms"] = _median_ms(lambda: mh3_fp8_attention(q, k, v), stream)
    res["e2e_speedup"] = res["triton_ref_e2e_ms"] / res["mh3_e2e_ms"]
    # (i) kernels alone: the reference wrapper's quantisation, then only its attention kernel
    c = (1.0 / math.sqrt(Dq)) * RF.LOG2E
    Sk = k.shape[2]
    nq, nk = triton.cdiv(Sq, 128), triton.cdiv(Sk, 128)
    dev = q.device
    q8 = torch.empty((Bq, Hq, Sq, Dq), dtype=torch.float8_e4m3fn, device=dev)
    sq = torch.empty((Bq, Hq, nq), dtype=torch.float32, device=dev)
    RF._quantize_q_kernel[(nq, Bq * Hq)](q, q8, sq, Sq=Sq, H=Hq, D=Dq, stride_qb=q.stride(0),
                                         stride_qh=q.stride(1), stride_qs=q.stride(2), stride_qd=q.stride(3),
                                         c=float(c), BLOCK_M=128)
    k_mean = k.float().mean(dim=2, keepdim=True).contiguous()
    k8 = torch.empty((Bq, Hq, Sk, Dq), dtype=torch.float8_e4m3fn, device=dev)
    sk = torch.empty((Bq, Hq, nk), dtype=torch.float32, device=dev)
    RF._quantize_k_kernel[(nk, Bq * Hq)](k, k_mean, k8, sk, Sk=Sk, H=Hq, D=Dq, stride_kb=k.stride(0),
                                         stride_kh=k.stride(1), stride_ks=k.stride(2), stride_kd=k.stride(3),
                                         BLOCK_N=128)
    del k_mean
    v8t = torch.empty((Bq, Hq, Dq, Sk), dtype=torch.float8_e4m3fn, device=dev)
    sv = torch.empty((Bq, Hq, Dq), dtype=torch.float32, device=dev)
    RF._quantize_v_kernel[(Bq * Hq,)](v, v8t, sv, Sk=Sk, H=Hq, D=Dq, stride_vb=v.stride(0), stride_vh=v.stride(1),
                                      stride_vs=v.stride(2), stride_vd=v.stride(3))
    out = torch.empty_like(q)
    is_cc10 = torch.cuda.get_device_capability(dev) >= (10, 0)

    def ref_kernel():
        RF._fp8_attn_kernel[(nq, Bq * Hq)](q8, k8, v8t, sq, sk, sv, q8, q8, out, Sq=Sq, Sk=Sk, H=Hq, D=Dq,
                                           Sq_bucket=Sq // 512, Sk_bucket=Sk // 512, HAS_MASK=False,
                                           HAS_BIAS=False, DO_REPAIR=False, repair_tau=-1.0, IS_CC10=is_cc10,
                                           BLOCK_M=128)

    res["triton_ref_kernel_ms"] = _median_ms(ref_kernel, stream)
    best = getattr(RF._fp8_attn_kernel, "best_config", None)
    res["triton_ref_best_config"] = str(best) if best is not None else None
    del q8, k8, v8t, out
    m8q, m8k, m8v, msq, msk, msv, _ = ops.quantize_qkv(q, k, v, c, v_dtype=torch.float16)
    mout = torch.empty_like(q)
    res["mh3_kernel_ms"] = _median_ms(
        lambda: ops.attention_e4m3(m8q, m8k, m8v, msq, msk, msv, logit_scale_log2=1.0, out=mout), stream)
    res["triton_ref_kernel_tflops"] = flop / res["triton_ref_kernel_ms"] / 1e9
    res["mh3_kernel_tflops"] = flop / res["mh3_kernel_ms"] / 1e9
    res["kernel_speedup"] = res["triton_ref_kernel_ms"] / res["mh3_kernel_ms"]
    return res


def cpu_reference_sample(seconds: float = 10.0):
    """The reference's CPU path (routed_sdpa -> torch SDPA fallback) on a bounded sample of config 2."""
    ref_sdpa, kind, source = _reference_cpu_path()

    g = torch.Generator().manual_seed(0)
    rows = 512
    q = torch.randn(1, 1, rows, D, generator=g)
    k = torch.randn(1, 1, S, D, generator=g)
    v = torch.randn(1, 1, S, D, generator=g)
    flop = 4.0 * rows * S * D
    for _ in range(2):
        ref_sdpa(q, k, v)
    n, t0 = 0, time.perf_counter()
    while True:
        ref_sdpa(q, k, v)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return {"value": flop * n / el / 1e12, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
            "kind": kind, "source": source,
            "sample": f"torch SDPA fp32 on CPU, 1 head x {rows} query rows x {S} keys x D={D}, {n} calls "
                      f"in {el:.1f}s (the reference's routed_sdpa CPU fallback)"}


def cpu_config1():
    """Config 1 (the reference's CPU-runnable case) on the host: routed_sdpa's torch SDPA fallback, fp32
    q,k,v [1,8,1024,128] seed 0, 3 warm-ups then the median of 20."""
    import platform
    import statistics

    ref_sdpa, _, _ = _reference_cpu_path()

    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(1, 8, 1024, 128, generator=g) for _ in range(3))
    for _ in range(3):
        ref_sdpa(q, k, v)
    ts = []
    for _ in range(20):
        t0 = time.perf_counter()
        ref_sdpa(q, k, v)
        ts.append(time.perf_counter() - t0)
    med = statistics.median(ts)
    return {"ms": med * 1e3, "tflops": 4.0 * 8 * 1024 * 1024 * 128 / med / 1e12, "cpu_count": os.cpu_count(),
            "torch_threads": torch.get_num_threads(), "cpu": platform.processor() or platform.machine()}


def run_reference_arm(args, rank):
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    ref_sdpa, kind, source = _reference_cpu_path()

    g = torch.Generator().manual_seed(0)
    rows = 256
    q = torch.randn(1, 1, rows, D, generator=g)
    k = torch.randn(1, 1, S, D, generator=g)
    v = torch.randn(1, 1, S, D, generator=g)
    flop = 4.0 * rows * S * D
    for _ in range(max(args.warmup, 1)):
        ref_sdpa(q, k, v)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        ref_sdpa(q, k, v)
    el = time.perf_counter() - t0
    val = flop * args.steps / el / 1e12
    line = {"metric": "FP8 attention TFLOPS (S=32760 H=40 D=128)", "value": val, "unit": "TFLOP/s",
            "impl": "reference", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": el / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config2 sample: 1 head x 256 query rows x 32760 keys, D=128, CPU"},
            "cpu_baseline": {"value": val, "unit": "TFLOP/s", "kind": kind, "source": source,
                             "cores": torch.get_num_threads(),
                             "sample": "torch SDPA fp32 on CPU (routed_sdpa fallback), 1 head x 256 rows x "
                                       "32760 keys per step"},
            "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def config5_single_gpu(dev, steps=3, warmup=1):
    """Config 5's work on ONE GPU: S=75600 H=40 D=128 self-attention (per-(b,h) scales over the whole
    sequence, e4m3 Q/K, f16 V/scale, the same quantisation kernels the sharded path runs) plus the
    cross-attention of all 75600 tokens to 512 text tokens - the N=1 point of the sharded workload,
    device-resident, timed with CUDA events."""
    from minimaxh3_b200 import ops
    from minimaxh3_b200.kernels.fp8_attention import fp8_attention

    S5, H5, D5, T = 75600, 40, 128, 512
    g = torch.Generator(device=dev).manual_seed(1000)
    gc = torch.Generator().manual_seed(0)
    xs = []
    for _ in range(3):
        x = torch.randn(1, S5, H5, D5, generator=g, device=dev)
        x[..., int(torch.randperm(D5, generator=gc)[0])] *= 8.0
        xs.append(x.to(torch.bfloat16))
        del x
    q, k, v = xs
    gt = torch.Generator(device=dev).manual_seed(7)
    kt, vt = (torch.randn(1, H5, T, D5, generator=gt, device=dev).to(torch.bfloat16) for _ in range(2))
    ls2 = LOG2E_ / math.sqrt(D5)
    out = torch.empty(1, S5, H5, D5, dtype=torch.bfloat16, device=dev)

    def step():
        amax = torch.stack([ops.absmax_bh(t) for t in (q, k, v)])        # [3, B, H]
        sc = ops.scale_from_absmax(amax)
        q8 = ops.quantize_bh(q, sc[0])[0].transpose(1, 2)                 # [B, H, S, D] views
        k8 = ops.quantize_bh(k, sc[1])[0].transpose(1, 2)
        v16 = ops.quantize_bh(v, sc[2], out_dtype=torch.float16)[0].transpose(1, 2)
        ops.attention_e4m3(q8, k8, v16, sc[0][..., None], sc[1][..., None], sc[2][..., None],
                           logit_scale_log2=ls2, out=out.transpose(1, 2))
        return fp8_attention(q.transpose(1, 2), kt, vt)

    stream = torch.cuda.current_stream(dev)
    ms = _time_cuda(step, steps, warmup, stream)
    flop = 4.0 * H5 * S5 * S5 * D5 + 4.0 * H5 * S5 * T * D5
    return {"workload": "config5 on one GPU: self-attention B=1 H=40 S=75600 D=128 + cross-attention to 512 "
                        "tokens (no collectives)", "ms_per_step": ms, "value": flop / ms / 1e9, "unit": "TFLOP/s",
            "steps": steps}


def run_ulysses_arm(args, dist, rank, world, local):
    from minimaxh3_b200.kernels.fp8_attention import fp8_attention
    from minimaxh3_b200.ulysses import default_head_groups, ulysses_attention, ulysses_attention_host

    dev = torch.device("cuda", local)
    S5, H5, D5, T = 75600, 40, 128, 512
    Sl = S5 // world
    G = args.head_groups
    G_host = args.host_head_groups or default_head_groups(H5 // world)
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    gc = torch.Generator().manual_seed(0)
    shard = []
    for _ in range(3):
        x = torch.randn(1, Sl, H5, D5, generator=g, device=dev)
        x[..., int(torch.randperm(D5, generator=gc)[0])] *= 8.0
        shard.append(x.to(torch.bfloat16))
    q, k, v = shard
    gt = torch.Generator(device=dev).manual_seed(7)
    kt, vt = (torch.randn(1, H5, T, D5, generator=gt, device=dev).to(torch.bfloat16) for _ in range(2))
    flop_self = 4.0 * H5 * S5 * S5 * D5
    flop_cross = 4.0 * H5 * S5 * T * D5
    stream = torch.cuda.current_stream(dev)
    attn_ev = []                                  # (start, end) around every local attention launch
    o_buf = torch.empty_like(q)

    def step(ev=None):
        # the cross-attention runs while the input exchange is in flight
        return ulysses_attention(q, k, v, events=ev, head_groups=G, out=o_buf, cross_kv=(kt, vt),
                                 exchange=args.exchange)

    for _ in range(args.warmup):
        step()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local, args.clock_period_ms, enabled=rank == 0) as clk:
        torch.cuda.synchronize(dev)
        dist.barrier()
        torch.cuda.synchronize(dev)
        t0.record(stream)
        for i in range(args.steps):
            step(attn_ev)
        t1.record(stream)
        torch.cuda.synchronize(dev)
    dist.barrier()
    ms = t0.elapsed_time(t1)
    attn_ms = sum(a.elapsed_time(b) for a, b in attn_ev) / args.steps
    t = torch.tensor([ms, attn_ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, attn_ms = float(t[0]), float(t[1])
    value = (flop_self + flop_cross) * args.steps / (ms / 1e3) / 1e12
    achieved = flop_self / world / (attn_ms / 1e3) / 1e12
    peaks = _peaks()
    # e2e: the local shard comes from pinned host memory and both outputs go
    # back, each head group's copies overlapping the other groups' compute
    hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
    ho, hc = (torch.empty_like(hq).pin_memory() for _ in range(2))

    def e2e_step():
        ulysses_attention_host(hq, hk, hv, out=ho, head_groups=G_host, cross_kv=(kt, vt), cross_out=hc)

    e2e_step()
    torch.cuda.synchronize(dev)
    dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    n_e2e = max(1, min(args.steps, 3))
    e0.record(stream)
    for _ in range(n_e2e):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    t = torch.tensor([e0.elapsed_time(e1)], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t[0])
    # Check after the timed regions: one step through each exchange must give the same bits on
    # every rank (the copy-engine pulls against NCCL's all-to-alls), reduced over the ranks.
    o_peer, c_peer = ulysses_attention(q, k, v, head_groups=1, cross_kv=(kt, vt), exchange="peer")
    o_nccl, c_nccl = ulysses_attention(q, k, v, head_groups=1, cross_kv=(kt, vt), exchange="nccl")
    same = torch.tensor([1 if torch.equal(o_peer, o_nccl) and torch.equal(c_peer, c_nccl) else 0],
                        device=dev, dtype=torch.int32)
    dist.all_reduce(same, op=dist.ReduceOp.MIN)
    exchange_check = {"peer_equals_nccl_bitwise": bool(int(same.item())), "ranks": world}
    del o_peer, c_peer, o_nccl, c_nccl
    if rank != 0:
        return
    # The same workload on rank 0's GPU alone (no collectives), so the sharded value can be
    # compared with its own N=1 point; the other ranks wait at the final barrier meanwhile.
    torch.cuda.empty_cache()
    try:
        n1 = config5_single_gpu(dev)
        n1["efficiency_of_this_line"] = value / (world * n1["value"])
    except Exception as e:  # noqa: BLE001
        n1 = {"unavailable": f"{type(e).__name__}: {str(e)[:300]}"}
    line = {
        "metric": "FP8 attention TFLOPS (S=32760 H=40 D=128)",
        "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "e4m3 QK^T, f16 PV", "data": "synthetic",
        "config": {"workload": f"config5: Ulysses self-attention B=1 H=40 S=75600 D=128 over {world} GPUs "
                               f"(S/P={Sl}, H/P={H5 // world}) + cross-attention to 512 text tokens",
                   "parallelism": f"ulysses{world}", "head_groups": G, "e2e_head_groups": G_host,
                   "exchange": args.exchange,
                   "inputs_vs_l2": "per-rank inputs > 126 MB L2 (no flush)"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["fp8_tflops"], "unit": "TFLOP/s",
                     "frac": achieved / peaks["fp8_tflops"], "traffic": None, "peak_source": peaks["source"],
                     "kernel": "mh3::attn::fwd_kernel (local head shard, one launch per head group)",
                     "avg_launch_ms": attn_ms / G, "launches_per_step": G},
        "e2e": {"value": (flop_self + flop_cross) * n_e2e / (e2e_ms / 1e3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": 3 * Sl * H5 * D5 * 2 * world,
                "d2h_bytes_per_step": 2 * Sl * H5 * D5 * 2 * world,
                "api": "minimaxh3_b200.ulysses.ulysses_attention_host (cross_kv: fp8_attention per head group)"},
        # per step and head group: 3 absmax + 3 quantize_bh + 1 attention;
        # per step: the cross-attention's 5 quantisation kernels + 1 attention
        "gpu_launches": (7 * G + 6) * args.steps, "clocks": clk.summary(),
        "n1_same_workload": n1,
        "exchange_check": exchange_check,
    }
    print(json.dumps(line), flush=True)


def run_gpu_arm(args, dist, rank, world, local):
    if world > 1:
        return run_ulysses_arm(args, dist, rank, world, local)
    global H
    H = args.heads
    FLOP_PER_CALL = 4.0 * B * H * S * S * D
    from minimaxh3_b200 import ops
    from minimaxh3_b200.streaming import fp8_attention_host

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    q, k, v = _synthetic_qkv(dev)
    (q8, sq), (k8, sk), (v8, sv) = _per_bh_e4m3(q), _per_bh_e4m3(k), _per_bh_e4m3(v)
    ls2 = 1.4426950408889634 / math.sqrt(D)
    out = torch.empty(B, H, S, D, dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream(dev)
    v16 = torch.empty(B, H, S, D, dtype=torch.float16, device=dev)
    lib = ops._lib.load()
    attn_ev = []

    def step(record=None):
        vin = v8
        if args.pv == "f16":
            rc = lib.mh3_widen_e4m3_to_f16(v8.data_ptr(), v16.data_ptr(), v8.numel(), stream.cuda_stream)
            ops._lib.check(rc, "widen")
            vin = v16
        if record is not None:
            record[0].record(stream)
        ops.attention_e4m3(q8, k8, vin, sq, sk, sv, logit_scale_log2=ls2, out=out)
        if record is not None:
            record[1].record(stream)

    for _ in range(args.warmup):
        step()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(local, args.clock_period_ms, enabled=rank == 0) as clk:
        torch.cuda.synchronize(dev)
        if dist:
            dist.barrier()
        torch.cuda.synchronize(dev)
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(stream)
        for i in range(args.steps):
            step((starts[i], ends[i]))
        t_end.record(stream)
        torch.cuda.synchronize(dev)
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    total_ms = t_start.elapsed_time(t_end)
    per_launch = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    if dist:
        t = torch.tensor([total_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    value = FLOP_PER_CALL * args.steps * world / (total_ms / 1e3) / 1e12
    avg_launch_ms = sum(per_launch) / len(per_launch)
    achieved = FLOP_PER_CALL / (avg_launch_ms / 1e3) / 1e12
    peaks = _peaks()
    if args.no_extras:
        if rank == 0:
            print(json.dumps({"value": value, "avg_launch_ms": avg_launch_ms, "achieved": achieved, "heads": H}))
        return

    # The reference's own Triton path on the same box and inputs (after the timed region).
    try:
        competitor = triton_competitor(q, k, v, stream)
    except Exception as e:  # noqa: BLE001 - reported in the line, not fatal
        competitor = {"unavailable": f"{type(e).__name__}: {str(e)[:300]}"}
    torch.cuda.empty_cache()

    # End to end through the drop-in API: pinned host bf16 in, bf16 out back to host.
    e2e_steps = max(1, min(args.steps, 3))
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    del q, k, v
    hout = torch.empty((B, H, S, D), dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        # host-resident inputs streamed through the GPU in head chunks:
        # H2D copy, quantise + attention and D2H copy overlap
        fp8_attention_host(hq, hk, hv, out=hout)

    e2e_step()
    torch.cuda.synchronize(dev)
    if dist:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_val = FLOP_PER_CALL * e2e_steps * world / (e2e_ms / 1e3) / 1e12
    h2d = 3 * B * H * S * D * 2
    d2h = B * H * S * D * 2

    if rank != 0:
        return
    cpu = cpu_reference_sample(seconds=args.cpu_seconds) if world == 1 else None
    if cpu is not None:
        cpu["config1"] = cpu_config1()
    line = {
        "metric": "FP8 attention TFLOPS (S=32760 H=40 D=128)",
        "value": value,
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": total_ms / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "e4m3 QK^T, " + ("f16 PV" if args.pv == "f16" else "e4m3 PV"),
        "data": "synthetic",
        "config": {"workload": "config2: FP8 self-attention fwd B=1 H=40 S=32760 D=128, per-(b,h) scales, "
                               "bf16 out", "pv": args.pv, "inputs_vs_l2": "inputs 504 MB > 126 MB L2 (no flush)",
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU"},
        "pct_of_fp8_peak": achieved / peaks["fp8_tflops"],
        "pct_of_nominal_fp8_peak": achieved / NOMINAL_FP8_TFLOPS,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["fp8_tflops"], "unit": "TFLOP/s",
                     "frac": achieved / peaks["fp8_tflops"],
                     "traffic": ATTN_TRAFFIC_BYTES_H40.get(args.pv) if H == 40 else None,
                     "traffic_source": "ncu dram__bytes_read+write, H=8 capture x5 (profiles/attn_fwd_config2.md)",
                     "peak_source": peaks["source"],
                     # half the FLOPs (PV) run at the 16-bit rate with f16 P/V:
                     # the attainable peak is the harmonic mix of the two rates
                     "peak_mixed": (1.0 / (0.5 / peaks["fp8_tflops"] + 0.5 / (peaks["fp8_tflops"] / 2))
                                    if args.pv == "f16" else peaks["fp8_tflops"]),
                     "kernel": "mh3::attn::fwd_kernel", "avg_launch_ms": avg_launch_ms},
        "e2e": {"value": e2e_val, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "api": "minimaxh3_b200.streaming.fp8_attention_host (pinned bf16 in/out, per head chunk: "
                       "H2D, quantise + attention, D2H on three overlapping streams)",
                "steps": e2e_steps},
        "gpu_launches": args.steps * (2 if args.pv == "f16" else 1),
        "clocks": clk.summary(),
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    line["competitor_same_box"] = competitor
    # The rest of the metric on the same box (untimed by the driver's clock check: after the line's
    # own timed regions): config 4 linear, config 3 varlen, ms per synthetic DiT block.
    del hq, hk, hv, hout
    torch.cuda.empty_cache()
    extras = {}
    for name, fn in (("config4_linear", lambda: linear_results(32760, 5, 3)),
                     ("config3_varlen", lambda: varlen_results(5, 3)),
                     ("dit_block", lambda: block_results(5, 3)),
                     ("config5_single_gpu", lambda: config5_single_gpu(dev))):
        try:
            extras[name] = fn()
        except Exception as e:  # noqa: BLE001
            extras[name] = {"unavailable": f"{type(e).__name__}: {str(e)[:300]}"}
        torch.cuda.empty_cache()
    line["extras"] = extras
    print(json.dumps(line), flush=True)


def _time_cuda(fn, steps, warmup, stream):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def run_linear_workload(args):
    print(json.dumps(linear_results(args.linear_rows, args.steps, args.warmup)), flush=True)


def linear_results(M, steps, warmup):
    """Benchmark configuration 4: FP8 scaled linear with fused epilogue (not the headline).

    M=32760 tokens, K=5120, N in {5120, 15360, 13824}; x N(0,1) bf16, W N(0,0.02),
    bias N(0,0.01), one LoRA adapter of rank 32 (A, B ~ N(0,0.01), scale 1).
    Reports, per N: the fused GEMM alone (e4m3 inputs resident), the whole
    FP8Linear.forward (row quantisation + LoRA-down + fused GEMM), and the
    reference's GPU recipe on the same box (our row quantisation +
    torch._scaled_mm + the two LoRA matmuls and the add, fp8_linear.py:87-108);
    and for an unquantised bf16 nn.Linear with the same adapter, the fused
    bf16 GEMM (ops.linear_lora) against cuBLAS linear + LoRA matmuls + add
    (runtime/lora.py:206-226).
    """
    from minimaxh3_b200 import ops
    from minimaxh3_b200.kernels.fp8_linear import FP8Linear

    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    xs = {}
    lines = []
    peaks = _peaks()
    try:
        _, RL = _reference_kernels()
    except Exception as e:  # noqa: BLE001 - reported, not fatal
        RL, ref_missing = None, f"{type(e).__name__}: {e}"
    for N, K in ((5120, 5120), (15360, 5120), (13824, 5120), (5120, 13824)):  # last: MLP-down
        x = xs.setdefault(K, torch.randn(M, K, generator=g, device=dev).to(torch.bfloat16))
        lin = torch.nn.Linear(K, N, device=dev, dtype=torch.bfloat16)
        with torch.no_grad():
            lin.weight.copy_(torch.randn(N, K, generator=g, device=dev) * 0.02)
            lin.bias.copy_(torch.randn(N, generator=g, device=dev) * 0.01)
        mod = FP8Linear.from_linear(lin)
        A = (torch.randn(32, K, generator=g, device=dev) * 0.01).to(torch.bfloat16)
        Bm = (torch.randn(N, 32, generator=g, device=dev) * 0.01).to(torch.bfloat16)
        mod.adapters = [(A, Bm, 1.0)]
        x8, sa = ops.quantize_rows(x)
        sb = mod.w_scale.reshape(-1)
        flop = 2.0 * M * N * K
        t_gemm = _time_cuda(lambda: ops.scaled_gemm(x8, mod.w8, row_scale=sa, col_scale=sb, bias=mod.bias),
                            steps, warmup, stream)
        t_fwd = _time_cuda(lambda: mod(x), steps, warmup, stream)
        t_refmod = None
        if RL is not None:
            # the reference's own FP8Linear (Triton row quantisation + torch._scaled_mm + LoRA matmuls)
            rlin = torch.nn.Linear(K, N, device=dev, dtype=torch.bfloat16)
            with torch.no_grad():
                rlin.weight.copy_(torch.randn(N, K, generator=g, device=dev) * 0.02)
                rlin.bias.copy_(mod.bias)
            rmod = RL.FP8Linear.from_linear(rlin)
            rmod.adapters = [(A, Bm, 1.0)]
            t_refmod = _median_ms(lambda: rmod(x), stream)
            del rmod, rlin

        def ref_recipe():
            out = torch._scaled_mm(x8, mod.w8.t(), scale_a=sa, scale_b=mod.w_scale, bias=mod.bias,
                                   out_dtype=torch.bfloat16)
            return out + ((x @ A.t()) @ Bm.t()).to(out.dtype)

        t_ref = _time_cuda(ref_recipe, steps, warmup, stream)
        t_cub = _time_cuda(lambda: torch._scaled_mm(x8, mod.w8.t(), scale_a=sa, scale_b=mod.w_scale, bias=mod.bias,
                                                    out_dtype=torch.bfloat16), steps, warmup, stream)
        # unquantised nn.Linear + the same adapter (runtime/lora.py:206-226): one fused bf16
        # GEMM against the reference's cuBLAS linear + two LoRA matmuls + add
        w16 = (torch.randn(N, K, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        t_l16 = _time_cuda(lambda: ops.linear_lora(x, w16, mod.bias, [(A, Bm, 1.0)]), steps, warmup, stream)

        def ref_bf16():
            out = torch.nn.functional.linear(x, w16, mod.bias)
            return out + ((x @ A.t()) @ Bm.t()).to(out.dtype)

        t_r16 = _time_cuda(ref_bf16, steps, warmup, stream)
        del w16
        lines.append({"N": N, "K": K, "gemm_ms": t_gemm, "gemm_tflops": flop / t_gemm / 1e9,
                      "cublas_scaled_mm_tflops": flop / t_cub / 1e9,
                      "gemm_frac_of_fp8_peak": flop / t_gemm / 1e9 / peaks["fp8_tflops"],
                      "fp8linear_forward_ms": t_fwd, "fp8linear_forward_tflops": flop / t_fwd / 1e9,
                      "reference_recipe_ms": t_ref, "reference_recipe_tflops": flop / t_ref / 1e9,
                      "bf16_linear_lora_tflops": flop / t_l16 / 1e9,
                      "bf16_reference_recipe_tflops": flop / t_r16 / 1e9,
                      "reference_fp8linear_forward_ms": t_refmod,
                      "reference_fp8linear_forward_tflops": flop / t_refmod / 1e9 if t_refmod else None,
                      "forward_speedup_vs_reference_module": t_refmod / t_fwd if t_refmod else None})
        del mod, lin, x8, sa
    return {"workload": f"config4: FP8 scaled linear M={M} K=5120 (N 5120/15360/13824) and the MLP-down "
                        "shape K=13824 N=5120, LoRA r=32", "unit": "TFLOP/s", "peak": peaks,
            "reference_module": "baseline/_ref kernels/fp8_linear.py FP8Linear (median of 20 after 3 warm-ups)"
            if RL is not None else f"unavailable: {ref_missing}", "results": lines}


def run_bf16_gemm_workload(args):
    """Unquantised bf16 linear (+ LoRA r=32) against cuBLAS at config 4's shapes, M = --linear-rows.

    Interleaved timing (5 rounds, each function 5 calls per round, medians) of: this package's
    bf16 main GEMM, the same with the LoRA K-steps, the LoRA-down product, ``ops.linear_lora``,
    cuBLAS ``F.linear`` and the reference recipe (``F.linear`` + LoRA matmuls + add).  Then one
    more call of the main GEMM and of ``F.linear`` at N=K=5120 between cudaProfilerStart/Stop,
    the pair an ``ncu --profile-from-start off -c 2`` capture compares.
    """
    import statistics

    from minimaxh3_b200 import ops

    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev)
    M = args.linear_rows
    g = torch.Generator(device=dev).manual_seed(0)
    results = {}
    keep = None
    for N, K in ((13824, 5120), (5120, 13824), (5120, 5120)):
        x = torch.randn(M, K, generator=g, device=dev).to(torch.bfloat16)
        w = (torch.randn(N, K, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        bias = (torch.randn(N, generator=g, device=dev) * 0.01).to(torch.bfloat16)
        A = (torch.randn(32, K, generator=g, device=dev) * 0.01).to(torch.bfloat16)
        Bm = (torch.randn(N, 32, generator=g, device=dev) * 0.01).to(torch.bfloat16)
        a2 = ops.scaled_gemm(x, A)
        fns = {
            "mh3_main_gemm": lambda: ops.scaled_gemm(x, w, bias=bias),
            "mh3_main_gemm_with_lora_ksteps": lambda: ops.scaled_gemm(x, w, bias=bias, a2=a2, b2=Bm),
            "mh3_lora_down": lambda: ops.scaled_gemm(x, A),
            "mh3_linear_lora": lambda: ops.linear_lora(x, w, bias, [(A, Bm, 1.0)]),
            "cublas_linear": lambda: torch.nn.functional.linear(x, w, bias),
            "reference_recipe": lambda: torch.nn.functional.linear(x, w, bias) + ((x @ A.t()) @ Bm.t()),
        }
        samples = {k: [] for k in fns}
        for _ in range(5):
            for k, fn in fns.items():
                samples[k].append(_time_cuda(fn, 5, 1, stream))
        flop = 2.0 * M * N * K
        results[f"N={N},K={K}"] = {k: {"ms": statistics.median(v), "tflops": flop / statistics.median(v) / 1e9}
                                   for k, v in samples.items()}
        if N == K:
            keep = (x, w, bias)
        del a2
    x, w, bias = keep
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStart()
    ops.scaled_gemm(x, w, bias=bias)
    torch.nn.functional.linear(x, w, bias)
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    print(json.dumps({"workload": f"bf16 linear + LoRA r=32 vs cuBLAS, M={M}", "unit": "TFLOP/s",
                      "results": results}), flush=True)


def run_varlen_workload(args):
    print(json.dumps(varlen_results(args.steps, args.warmup, args.heads)), flush=True)


def varlen_results(steps, warmup, heads=40):
    """Benchmark configuration 3: packed varlen, cu_seqlens [0, 33784, 50676], H=40 D=128.

    e4m3 q/k/v with per-(sequence, head) scales (synthetic N(0,1) with one
    channel x8), f16 PV, bf16 out; attention is block-diagonal per sequence.
    Algorithmic work 4*H*D*(33784^2 + 16892^2) = 2.922e13 FLOP per call.
    """
    from minimaxh3_b200 import ops

    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev)
    lens = [33784, 16892]
    T, Hh, Dd = sum(lens), heads, 128
    g = torch.Generator(device=dev).manual_seed(0)
    gc = torch.Generator().manual_seed(0)
    cu = torch.tensor([0, lens[0], T], dtype=torch.int32, device=dev)
    packed, scales = [], []
    for _ in range(3):
        x = torch.randn(T, Hh, Dd, generator=g, device=dev)
        x[..., int(torch.randperm(Dd, generator=gc)[0])] *= 8.0
        x = x.to(torch.bfloat16).float()
        s = torch.stack([x[a:b].abs().amax(dim=(0, 2)) for a, b in ((0, lens[0]), (lens[0], T))])
        s = torch.clamp(s, min=1e-12) / 448.0                       # [nseq, H]
        seq_of = torch.repeat_interleave(torch.arange(2, device=dev), torch.tensor(lens, device=dev))
        packed.append(torch.clamp(x / s[seq_of][..., None], -448, 448))
        scales.append(s[..., None].contiguous())
        del x
    q8, k8 = (t.to(torch.float8_e4m3fn) for t in packed[:2])
    v16 = packed[2].to(torch.float16)
    del packed
    ls2 = 1.4426950408889634 / math.sqrt(Dd)
    out = torch.empty(T, Hh, Dd, dtype=torch.bfloat16, device=dev)
    call = lambda: ops.attention_e4m3(q8, k8, v16, *scales, logit_scale_log2=ls2, cu_seqlens_q=cu,
                                      cu_seqlens_k=cu, max_seqlen_q=max(lens), out=out)
    ms = _time_cuda(call, steps, warmup, stream)
    del q8, k8, v16, out
    # the drop-in route: bf16 packed q/k/v -> per-(sequence, head) quantisation + the same kernel
    from minimaxh3_b200.kernels.fp8_attention import fp8_attention_varlen

    qkv = []
    for _ in range(3):
        x = torch.randn(T, Hh, Dd, generator=g, device=dev, dtype=torch.bfloat16)
        x[..., int(torch.randperm(Dd, generator=gc)[0])] *= 8.0
        qkv.append(x)
    dropin = lambda: fp8_attention_varlen(*qkv, cu, cu, max(lens))
    ms_dropin = _time_cuda(dropin, steps, warmup, stream)
    del qkv
    flop = 4.0 * Hh * Dd * sum(L * L for L in lens)
    peaks = _peaks()
    return {"workload": f"config3: varlen cu_seqlens [0,33784,50676], H={Hh} D=128, per-(seq,head) "
                        "scales, f16 PV", "unit": "TFLOP/s", "ms": ms, "tflops": flop / ms / 1e9,
            "frac_of_fp8_peak": flop / ms / 1e9 / peaks["fp8_tflops"], "flop": flop,
            "dropin_ms": ms_dropin, "dropin_tflops": flop / ms_dropin / 1e9,
            "dropin": "fp8_attention_varlen: bf16 packed q/k/v, mh3_absmax_seg + mh3_quantize_seg + attention"}


def run_block_workload(args):
    print(json.dumps(block_results(args.steps, args.warmup)), flush=True)


def block_results(steps, warmup):
    """ms per synthetic DiT block at config 2 / 4 shapes (the full transformer
    and its block count are not available): QKV projection FP8Linear
    (5120 -> 15360), self-attention through the drop-in fp8_attention on
    [1, 40, 32760, 128] views of it, out-projection FP8Linear (5120 -> 5120),
    cross-attention of the 32760 tokens to 512 text tokens, MLP-up FP8Linear
    (5120 -> 13824).  Random-init weights N(0, 0.02), bias N(0, 0.01), one
    LoRA adapter r=32 on each linear, activations N(0, 1) bf16."""
    from minimaxh3_b200.kernels.fp8_attention import fp8_attention
    from minimaxh3_b200.kernels.fp8_linear import FP8Linear

    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    M, C, Hh, Dd, T = 32760, 5120, 40, 128, 512

    def lin(n_in, n_out):
        layer = torch.nn.Linear(n_in, n_out, device=dev, dtype=torch.bfloat16)
        with torch.no_grad():
            layer.weight.copy_(torch.randn(n_out, n_in, generator=g, device=dev) * 0.02)
            layer.bias.copy_(torch.randn(n_out, generator=g, device=dev) * 0.01)
        mod = FP8Linear.from_linear(layer)
        mod.adapters = [((torch.randn(32, n_in, generator=g, device=dev) * 0.01).to(torch.bfloat16),
                         (torch.randn(n_out, 32, generator=g, device=dev) * 0.01).to(torch.bfloat16), 1.0)]
        return mod

    qkv, proj, mlp_up = lin(C, 3 * C), lin(C, C), lin(C, 13824)
    x = torch.randn(M, C, generator=g, device=dev).to(torch.bfloat16)
    tk, tv = (torch.randn(1, Hh, T, Dd, generator=g, device=dev).to(torch.bfloat16) for _ in range(2))

    def block():
        y = qkv(x).view(1, M, 3, Hh, Dd)
        q, k, v = (y[:, :, i].transpose(1, 2) for i in range(3))   # [1, H, M, D] strided views
        a = fp8_attention(q, k, v).transpose(1, 2).reshape(M, C)
        h = proj(a)
        c = fp8_attention(h.view(1, M, Hh, Dd).transpose(1, 2), tk, tv).transpose(1, 2).reshape(M, C)
        return mlp_up(c)

    ms = _time_cuda(block, steps, warmup, stream)
    flop = (2.0 * M * C * (3 * C + C + 13824) + 4.0 * Hh * M * M * Dd + 4.0 * Hh * M * T * Dd)
    return {"workload": "synthetic DiT block: QKV GEMM N=15360 + self-attention S=32760 + out-proj "
                        "N=5120 + cross-attention to 512 tokens + MLP-up N=13824 (LoRA r=32 on each "
                        "linear); per DiT step = this x num_blocks (num_blocks not available)",
            "unit": "ms", "ms_per_block": ms, "tflops": flop / ms / 1e9}


def run_quant_workload(args):
    """Drop-in Q/K/V quantisation at config 2 shapes (HBM-bound; not the headline).

    ``mh3_quantize_qkv`` on bf16 q, k, v [1, 40, 32760, 128] (the reference's
    per-128-row Q/K blocks, K centred on its channel mean, V per channel,
    kernels/fp8_attention.py:39-170,338), V out as f16 (the default PV
    operand) and as e4m3.  Algorithmic bytes: q, k, v read once (bf16) and
    q8, k8, v8 written once; the kernels read K and V twice (statistics pass,
    then the quantising pass), which ``bytes_moved`` counts.
    """
    from minimaxh3_b200 import ops

    global H
    H = args.heads  # 40 = config 2; fewer for ncu captures
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev)
    q, k, v = _synthetic_qkv(dev)
    n = q.numel()
    peaks = _peaks()
    lines = []
    for vd, vbytes in ((torch.float16, 2), (torch.float8_e4m3fn, 1)):
        ms = _time_cuda(lambda: ops.quantize_qkv(q, k, v, 1.4426950408889634 / math.sqrt(D), v_dtype=vd),
                        args.steps, args.warmup, stream)
        algo = n * (3 * 2 + 1 + 1 + vbytes)
        moved = n * (5 * 2 + 1 + 1 + vbytes)
        lines.append({"v_out": str(vd).replace("torch.", ""), "ms": ms, "algorithmic_bytes": algo,
                      "achieved_gbs": algo / ms / 1e6, "frac_of_hbm": algo / ms / 1e6 / peaks["hbm_gbs"],
                      "bytes_moved": moved, "moved_gbs": moved / ms / 1e6})
    print(json.dumps({"workload": f"config2 drop-in quantisation: bf16 q,k,v [1,{H},32760,128] -> e4m3 + scales",
                      "unit": "GB/s", "peak_hbm_gbs": peaks["hbm_gbs"], "results": lines}), flush=True)


def run_step_workload(args):
    """Step-residual cache reductions (runtime/step_cache.py:39-52; not the headline).

    The per-step relative change of block 0's output plus the copy of it kept
    for the next step, on a bf16 hidden state [1, T, 5120] (``--step-tokens``
    T, by default config 5's 75600 tokens x the DiT width, 774 MB): ``ops.step_diff(copy=True)`` against the
    reference's arithmetic (two fp32 copies, a difference, two abs, two means,
    ``.item()``, clone).  Algorithmic bytes: h1 and h1_prev read once, h1_prev
    written once.
    """
    from minimaxh3_b200 import ops

    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    T = args.step_tokens
    h1 = torch.randn(1, T, 5120, generator=g, device=dev).to(torch.bfloat16)
    prev = (h1.float() + 0.01 * torch.randn(1, T, 5120, generator=g, device=dev)).to(torch.bfloat16)
    peaks = _peaks()

    def fused():
        sd, sp = ops.step_diff(h1, prev, copy=True).tolist()
        return (sd / h1.numel()) / max(sp / h1.numel(), 1e-6)

    def reference():
        rel = torch.mean(torch.abs(h1.float() - prev.float())) / torch.clamp(torch.mean(torch.abs(prev.float())),
                                                                            min=1e-6)
        r = float(rel.item())
        h1.detach().clone()          # the kept copy (step_cache.py:151)
        return r

    ms = _time_cuda(fused, args.steps, args.warmup, stream)
    ms_ref = _time_cuda(reference, args.steps, args.warmup, stream)
    algo = 3 * h1.numel() * 2
    print(json.dumps({"workload": f"step cache: relative change + kept copy of a bf16 [1, {T}, 5120] hidden state",
                      "unit": "ms", "fused_ms": ms, "reference_arithmetic_ms": ms_ref, "algorithmic_bytes": algo,
                      "fused_gbs": algo / ms / 1e6, "frac_of_hbm": algo / ms / 1e6 / peaks["hbm_gbs"],
                      "includes": "one device->host read of the sums (the step's host sync)"}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="mh3", choices=["mh3", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--heads", type=int, default=40, help="heads (40 = config 2; fewer for ncu captures)")
    ap.add_argument("--no-extras", action="store_true",
                    help="kernel timing only (no e2e, no CPU baseline): the ncu capture command")
    ap.add_argument("--workload", default="attention",
                    choices=["attention", "linear", "quant", "varlen", "block", "step", "bf16_gemm"],
                    help="attention = config 2 (the headline line); linear = config 4 measurements")
    ap.add_argument("--pv", default="f16", choices=["f16", "e4m3"],
                    help="PV product operands: f16 P/V (default, meets the tolerance) or e4m3")
    ap.add_argument("--linear-rows", type=int, default=32760,
                    help="linear workload: token rows M (32760 = config 4; smaller for ncu captures)")
    ap.add_argument("--step-tokens", type=int, default=75600,
                    help="step workload: hidden-state tokens (75600 = config 5; smaller for ncu captures)")
    ap.add_argument("--clock-period-ms", type=int, default=50,
                    help="nvidia-smi clock sampling period during the timed region")
    ap.add_argument("--exchange", default="peer", choices=["nccl", "peer"],
                    help="N>1: Ulysses exchange by copy-engine pulls from peer buffers (CUDA IPC) or by NCCL "
                         "all-to-alls")
    ap.add_argument("--head-groups", type=int, default=1,
                    help="N>1: head groups of the device-resident Ulysses pipeline (the value line)")
    ap.add_argument("--host-head-groups", type=int, default=0,
                    help="N>1: head groups of the host-resident e2e pipeline (0 = ulysses.default_head_groups)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "mh3":
        args.warmup = 3
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        run_reference_arm(args, rank)
        return
    if args.workload == "quant":
        run_quant_workload(args)
        return
    if args.workload == "step":
        run_step_workload(args)
        return
    if args.workload == "varlen":
        run_varlen_workload(args)
        return
    if args.workload == "block":
        run_block_workload(args)
        return
    if args.workload == "linear":
        run_linear_workload(args)
        return
    if args.workload == "bf16_gemm":
        run_bf16_gemm_workload(args)
        return
    dist, rank, world, local = _dist()
    try:
        run_gpu_arm(args, dist, rank, world, local)
    finally:
        if dist:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
