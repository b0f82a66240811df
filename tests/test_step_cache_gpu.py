"""mh3_step_diff against float64 sums, and the fused step cache against its CPU run."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("n", [1, 7, 1000, 8 * 592 + 3, 3_000_001, 12_582_917])  # the last: unrolled loads per thread
def test_step_diff_sums_copy_and_determinism(dtype, n):
    from minimaxh3_b200 import ops

    g = torch.Generator(device="cuda").manual_seed(n)
    h1 = torch.randn(n, generator=g, device="cuda").to(dtype)
    prev = (torch.randn(n, generator=g, device="cuda") * 2).to(dtype)
    keep = prev.clone()
    ref_d = (h1.double() - prev.double()).abs().sum().item()
    ref_p = prev.double().abs().sum().item()
    s1 = ops.step_diff(h1, prev).tolist()
    assert torch.equal(prev, keep)                       # copy=False leaves prev alone
    s2 = ops.step_diff(h1, prev).tolist()
    assert s1 == s2                                      # fixed reduction order
    assert abs(s1[0] - ref_d) <= 1e-6 * ref_d and abs(s1[1] - ref_p) <= 1e-6 * ref_p
    s3 = ops.step_diff(h1, prev, copy=True).tolist()
    assert s3 == s1 and torch.equal(prev, h1)            # same sums, prev now holds h1


def test_step_diff_rejects_mismatched_inputs():
    from minimaxh3_b200 import ops

    a = torch.zeros(16, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        ops.step_diff(a, torch.zeros(16, dtype=torch.float16, device="cuda"))
    with pytest.raises(ValueError):
        ops.step_diff(a, torch.zeros(32, dtype=torch.bfloat16, device="cuda")[::2])


def test_fused_cache_decides_like_the_cpu_run():
    from test_step_cache_cpu import _Toy, _inputs

    from minimaxh3_b200.step_cache import StepResidualCache

    steps, thr = 14, 0.012
    runs = {}
    for dev in ("cpu", "cuda"):
        model = _Toy()
        cache = StepResidualCache().attach(model)
        cache.begin(steps, thr, warmup=3, tail=2)
        outs, skipped = [], []
        for x, t in _inputs(steps):
            before = model.blocks[1].calls
            outs.append(model(x.to(dev), t.to(dev)).cpu())
            skipped.append(model.blocks[1].calls == before)
        cache.end()
        runs[dev] = (outs, skipped)
    assert runs["cuda"][1] == runs["cpu"][1] and any(runs["cuda"][1])
    for a, b in zip(runs["cuda"][0], runs["cpu"][0]):
        assert torch.allclose(a, b, atol=1e-5, rtol=1e-5)
