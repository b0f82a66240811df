"""Step-residual cache decisions (runtime/step_cache.py:80-200) on CPU tensors.

On CPU the cache uses the reference's arithmetic; the skip pattern and the
outputs must follow the rule restated here: after block 0 the relative
change of its output is accumulated, and a step inside [warmup, steps-tail)
skips the middle blocks while the accumulated change stays under the
threshold (the residual out - h1 of the last computed step is added back).
"""
import math

import torch
import torch.nn as nn

from minimaxh3_b200.step_cache import StepResidualCache


class _Block(nn.Module):
    def __init__(self, i):
        super().__init__()
        self.i = i
        self.calls = 0

    def forward(self, x, temb):
        self.calls += 1
        return x * (1.0 + 0.01 * (self.i + 1)) + 0.001 * temb


class _Toy(nn.Module):
    def __init__(self):
        super().__init__()
        self.blocks = nn.ModuleList([_Block(i) for i in range(4)])

    def forward(self, x, temb):
        for b in self.blocks:
            x = b(x, temb)
        return x


def _inputs(steps):
    g = torch.Generator().manual_seed(0)
    base = torch.randn(2, 64, 32, generator=g)
    return [(base * (1.0 + 0.002 * s), torch.full((2, 64, 32), float(s))) for s in range(steps)]


def _expected_skips(inputs, threshold, warmup, tail):
    h_prev, acc, skips, have_res = None, 0.0, [], False
    n = len(inputs)
    for s, (x, t) in enumerate(inputs):
        h1 = x * 1.01 + 0.001 * t
        if h_prev is not None:
            rel = float(torch.mean(torch.abs(h1 - h_prev)) / torch.clamp(torch.mean(torch.abs(h_prev)), min=1e-6))
            acc += rel
        else:
            acc = math.inf
        h_prev = h1.clone()
        skip = warmup <= s < n - tail and have_res and acc < threshold
        if not skip:
            acc = 0.0
            have_res = True
        skips.append(skip)
    return skips


def test_skip_pattern_and_outputs_follow_the_rule():
    steps, thr = 14, 0.012
    model = _Toy()
    cache = StepResidualCache().attach(model)
    inputs = _inputs(steps)
    cache.begin(steps, thr, warmup=3, tail=2)
    outs, skipped = [], []
    for x, t in inputs:
        before = model.blocks[1].calls
        outs.append(model(x, t))
        skipped.append(model.blocks[1].calls == before)
    cache.end()
    exp = _expected_skips(inputs, thr, 3, 2)
    assert skipped == exp and any(exp) and not all(exp)
    # a skipped step returns h1 + (out - h1) of the last computed step
    last_res = None
    for (x, t), o, sk in zip(inputs, outs, skipped):
        h1 = x * 1.01 + 0.001 * t
        if sk:
            assert torch.allclose(o, h1 + last_res, atol=1e-5)
        else:
            full = h1
            for i in range(1, 4):
                full = full * (1.0 + 0.01 * (i + 1)) + 0.001 * t
            assert torch.allclose(o, full, atol=1e-5)
            last_res = full - h1


def test_inactive_below_nine_steps_or_zero_threshold():
    model = _Toy()
    cache = StepResidualCache().attach(model)
    cache.begin(8, 0.5)
    assert not cache.active
    cache.begin(20, 0.0)
    assert not cache.active
    cache.begin(20, 0.5)
    assert cache.active


class _PairBlock(nn.Module):
    """A block whose hidden state is a (video, audio) tuple, as in joint audio-video DiTs."""

    def __init__(self, i):
        super().__init__()
        self.i = i
        self.calls = 0

    def forward(self, x, a, temb):
        self.calls += 1
        f = 1.0 + 0.01 * (self.i + 1)
        return x * f + 0.001 * temb, a * f + 0.002 * temb


class _PairToy(nn.Module):
    def __init__(self):
        super().__init__()
        self.blocks = nn.ModuleList([_PairBlock(i) for i in range(3)])

    def forward(self, x, a, temb):
        for b in self.blocks:
            x, a = b(x, a, temb)
        return x, a


def test_tuple_states_follow_the_rule():
    steps, thr = 14, 0.012
    model = _PairToy()
    cache = StepResidualCache().attach(model)
    g = torch.Generator().manual_seed(1)
    bx, ba = torch.randn(2, 16, 8, generator=g), torch.randn(2, 4, 8, generator=g)
    cache.begin(steps, thr, warmup=3, tail=2)
    h_prev, acc, have_res, last_res, n_skip = None, 0.0, False, None, 0
    for s in range(steps):
        x, a, t = bx * (1.0 + 0.002 * s), ba * (1.0 + 0.002 * s), float(s)
        before = model.blocks[1].calls
        ox, oa = model(x, a, t)
        skipped = model.blocks[1].calls == before
        h1 = (x * 1.01 + 0.001 * t, a * 1.01 + 0.002 * t)
        if h_prev is not None:
            rels = [float(torch.mean(torch.abs(u - v)) / torch.clamp(torch.mean(torch.abs(v)), min=1e-6))
                    for u, v in zip(h1, h_prev)]
            acc += sum(rels) / len(rels)
        else:
            acc = math.inf
        h_prev = tuple(u.clone() for u in h1)
        expect = 3 <= s < steps - 2 and have_res and acc < thr
        assert skipped == expect
        n_skip += skipped
        if skipped:
            assert torch.allclose(ox, h1[0] + last_res[0], atol=1e-5)
            assert torch.allclose(oa, h1[1] + last_res[1], atol=1e-5)
        else:
            acc, have_res = 0.0, True
            last_res = (ox - h1[0], oa - h1[1])
    cache.end()
    assert 0 < n_skip < steps
