"""``mh3_quantize_qkv_noalloc``: Q/K/V quantisation with no caller workspace.

Callers that cannot allocate device memory when they call this path (a
plugin whose enqueue step must not allocate, a latency-critical loop that
cannot afford cudaMalloc's implicit device synchronisation, a host program
whose device memory belongs to another framework's pool) use this entry
point; its scratch is a fixed array inside the library.  This test calls it
through the C ABI and checks, on two calls in a row with different inputs,
that its outputs equal those of ``mh3_quantize_qkv`` given a normal
workspace - bit for bit, the tolerance the quantisation tests use.  It also
checks that a size beyond the fixed scratch is rejected.  The file name
makes pytest collect it last.
"""
import pytest
import torch

from minimaxh3_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _make(seed, B, H, Sq, Sk, D, dtype=torch.bfloat16):
    g = torch.Generator(device=DEV).manual_seed(seed)
    q, k, v = (torch.randn(B, H, S, D, generator=g, device=DEV).to(dtype) for S in (Sq, Sk, Sk))
    k = k + 0.5
    return q, k, v


def _outputs(B, H, Sq, Sk, D, v_dtype=torch.float8_e4m3fn):
    e4 = torch.float8_e4m3fn
    return dict(q8=torch.empty(B, H, Sq, D, dtype=e4, device=DEV), k8=torch.empty(B, H, Sk, D, dtype=e4, device=DEV),
                v8=torch.empty(B, H, Sk, D, dtype=v_dtype, device=DEV),
                scale_q=torch.empty(B, H, (Sq + 127) // 128, device=DEV),
                scale_k=torch.empty(B, H, (Sk + 127) // 128, device=DEV),
                scale_v=torch.empty(B, H, D, device=DEV), k_mean=torch.empty(B, H, D, device=DEV))


def _args(q, k, v, outs, workspace):
    B, H, Sq, D = q.shape
    a = _lib.QkvQuantArgs()
    a.batch, a.heads, a.seqlen_q, a.seqlen_k, a.head_dim = B, H, Sq, k.shape[2], D
    a.in_dtype = _lib.MH3_DTYPE_F16 if q.dtype == torch.float16 else _lib.MH3_DTYPE_BF16
    a.q, a.q_stride_b, a.q_stride_h, a.q_stride_s = q.data_ptr(), q.stride(0), q.stride(1), q.stride(2)
    a.k, a.k_stride_b, a.k_stride_h, a.k_stride_s = k.data_ptr(), k.stride(0), k.stride(1), k.stride(2)
    a.v, a.v_stride_b, a.v_stride_h, a.v_stride_s = v.data_ptr(), v.stride(0), v.stride(1), v.stride(2)
    a.q_premul = 0.127
    a.v_out_dtype = _lib.MH3_DTYPE_F16 if outs["v8"].dtype == torch.float16 else _lib.MH3_DTYPE_E4M3
    for name, t in outs.items():
        setattr(a, name, t.data_ptr())
    a.workspace = workspace
    return a


def _same(x, y):
    if x.dtype == torch.float8_e4m3fn:
        return torch.equal(x.view(torch.uint8), y.view(torch.uint8))
    return torch.equal(x, y)


def _compare_calls(B, H, Sq, Sk, D, in_dtype, v_dtype, seeds):
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    for call, seed in enumerate(seeds):
        q, k, v = _make(seed, B, H, Sq, Sk, D, in_dtype)
        ref = _outputs(B, H, Sq, Sk, D, v_dtype)
        ws = torch.empty(int(lib.mh3_qkv_workspace_bytes(B, H, Sk, D)), dtype=torch.uint8, device=DEV)
        _lib.check(lib.mh3_quantize_qkv(_args(q, k, v, ref, ws.data_ptr()), stream), "mh3_quantize_qkv")
        got = _outputs(B, H, Sq, Sk, D, v_dtype)
        _lib.check(lib.mh3_quantize_qkv_noalloc(_args(q, k, v, got, None), stream), "mh3_quantize_qkv_noalloc")
        torch.cuda.synchronize()
        for name in ref:
            assert _same(got[name], ref[name]), (call, name)


@pytest.mark.parametrize("in_dtype,D,v_dtype", [(torch.bfloat16, 128, torch.float8_e4m3fn),
                                               (torch.float16, 128, torch.float16),
                                               (torch.bfloat16, 64, torch.float16),
                                               (torch.float16, 64, torch.float8_e4m3fn)])
def test_noalloc_matches_workspace_entry_point_on_two_calls(in_dtype, D, v_dtype):
    _compare_calls(1, 8, 700, 4100, D, in_dtype, v_dtype, (11, 12))


def test_noalloc_accepts_exactly_its_scratch_size():
    """B*H*ceil(Sk/256)*D = 2^20: the statistics need exactly 8 MiB."""
    lib = _lib.load()
    B, H, Sk, D = 1, 32, 65536, 128
    assert lib.mh3_qkv_workspace_bytes(B, H, Sk, D) == 8 << 20
    _compare_calls(B, H, 256, Sk, D, torch.bfloat16, torch.float16, (21, 22))


def test_noalloc_rejects_sizes_beyond_its_scratch():
    lib = _lib.load()
    for B, H, Sk, D in ((1, 64, 1 << 20, 128), (1, 32, 65537, 128)):  # far beyond; one 256-key chunk beyond
        assert lib.mh3_qkv_workspace_bytes(B, H, Sk, D) > 8 << 20
        a = _lib.QkvQuantArgs()
        a.batch, a.heads, a.seqlen_q, a.seqlen_k, a.head_dim = B, H, 128, Sk, D
        rc = lib.mh3_quantize_qkv_noalloc(a, None)
        assert rc == _lib.MH3_ERR_TOO_LARGE
        assert b"8 MiB" in lib.mh3_last_error()
