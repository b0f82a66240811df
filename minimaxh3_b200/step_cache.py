"""Step-residual cache for the DiT denoising loop, with one-pass CUDA reductions.

Drop-in for ``StepResidualCache`` of the reference's runtime/step_cache.py
(constructed and driven by runtime/model_manager.py:124,317-330 and
runtime/generator.py:199-234 through ``attach``, ``begin``, ``end`` and
``active``).  Its skip rule, which decides which blocks run, is kept:

* block 0 always runs; its output h1 is compared with the previous step's,
  ``mean|h1 - h1_prev| / max(mean|h1_prev|, 1e-6)`` (averaged over the
  tensors of a tuple state), and the change is accumulated (runtime/
  step_cache.py:39-52, :124-131);
* a step whose index lies in ``[warmup, num_steps - tail)``, that has a
  residual from an earlier computed step and whose accumulated change is
  below ``threshold`` skips blocks 1..n-2 (they return their input hidden
  state) and the last block returns its input plus that residual
  (:133-160); any other step computes everything, resets the accumulated
  change and records ``residual = out_last - h1`` (:161-168);
* the cache is active only for ``threshold > 0``, more than 8 steps and at
  least 2 blocks (:180-185).

The design is this package's own: the per-generation state lives in one
``_Run`` record created by ``begin`` and dropped by ``end``; each block gets
the wrapper of its role (first, middle, last); states (a tensor or a
tuple/list of them) go through a small tree map.  On CUDA hidden states
(bf16 / f16 / f32, contiguous) the change and the copy of h1 kept for the
next step come from one pass of ``mh3_step_diff`` that writes h1 over the
previous step's buffer; the residual is written into one persistent buffer.
Other tensors use the reference's fp32 arithmetic.  The skip decision is
read on the host once per step: it steers Python control flow.
"""
from __future__ import annotations

import functools
import math
from dataclasses import dataclass, field
from typing import Any, Callable

import torch
import torch.nn as nn

from .kernels.fp8_linear import find_primary_block_list

# Keyword names under which diffusers blocks pass their hidden states, in the
# order the skip path hands them back (the reference's order, step_cache.py:58-64).
_HIDDEN_KEYS = ("hidden_states", "video_hidden_states", "audio_hidden_states", "encoder_hidden_states", "x")


def _tree_map(fn: Callable, a, *rest):
    """Apply ``fn`` leaf-wise over a tensor or a (nested) tuple/list of tensors.

    Leaves that are not tensors (in ``a`` or in a partner) are returned as
    they are in ``a``; sequences are zipped to the shortest.
    """
    if isinstance(a, torch.Tensor):
        if all(isinstance(r, torch.Tensor) for r in rest):
            return fn(a, *rest)
        return a
    if isinstance(a, (tuple, list)) and all(isinstance(r, (tuple, list)) for r in rest):
        mapped = [_tree_map(fn, *leaves) for leaves in zip(a, *rest)]
        return tuple(mapped) if isinstance(a, tuple) else mapped
    return a


def _snapshot(state):
    return _tree_map(lambda t: t.detach().clone(), state)


def _fusable(*ts: torch.Tensor) -> bool:
    t0 = ts[0]
    return all(t.is_cuda and t.is_contiguous() and t.dtype == t0.dtype and t.shape == t0.shape
               and t.device == t0.device and t.data_ptr() % 16 == 0 for t in ts) and \
        t0.dtype in (torch.bfloat16, torch.float16, torch.float32)


def _change_and_keep(h1: torch.Tensor, prev: torch.Tensor):
    """Relative change of one tensor and a tensor holding h1 for the next step."""
    if _fusable(h1, prev):
        from . import ops

        d, p = ops.step_diff(h1.detach(), prev, copy=True).tolist()   # prev now holds h1
        n = max(h1.numel(), 1)
        return (d / n) / max(p / n, 1e-6), prev
    num = torch.mean(torch.abs(h1.float() - prev.float()))
    den = torch.clamp(torch.mean(torch.abs(prev.float())), min=1e-6)
    return float((num / den).item()), h1.detach().clone()


def _state_change(h1, prev):
    """(mean relative change over the state's tensors, state kept for the next step)."""
    if isinstance(h1, torch.Tensor) and isinstance(prev, torch.Tensor):
        return _change_and_keep(h1, prev)
    if isinstance(h1, (tuple, list)) and isinstance(prev, (tuple, list)):
        changes, kept = [], []
        for i, x in enumerate(h1):
            y = prev[i] if i < len(prev) else None
            if isinstance(x, torch.Tensor) and isinstance(y, torch.Tensor):
                c, k = _change_and_keep(x, y)
                changes.append(c)
                kept.append(k)
            else:
                kept.append(_snapshot(x))
        kept = tuple(kept) if isinstance(h1, tuple) else kept
        return (sum(changes) / len(changes) if changes else 0.0), kept
    return 0.0, _snapshot(h1)


def _residual_into(out, h1, buf):
    """``out - h1`` leaf-wise in out's dtype, reusing ``buf``'s tensors when they match."""

    def sub(o: torch.Tensor, h: torch.Tensor, b=None):
        h = h.to(dtype=o.dtype, device=o.device)
        if isinstance(b, torch.Tensor) and b.shape == o.shape and b.dtype == o.dtype and b.device == o.device:
            return torch.sub(o.detach(), h, out=b)
        return (o - h).detach()

    if buf is None or type(buf) is not type(out):
        return _tree_map(sub, out, h1)
    return _tree_map(sub, out, h1, buf)


def _input_hidden(args: tuple, kwargs: dict, like):
    """The hidden state(s) a block was called with, shaped like block 0's output ``like``."""
    found: list[torch.Tensor] = [a for a in args if isinstance(a, torch.Tensor)]
    found += [kwargs[k] for k in _HIDDEN_KEYS if isinstance(kwargs.get(k), torch.Tensor)]
    for v in kwargs.values():
        if isinstance(v, torch.Tensor) and not any(v is f for f in found):
            found.append(v)
    if isinstance(like, (tuple, list)):
        picked = found[:len(like)]
        return tuple(picked) if isinstance(like, tuple) else picked
    if found:
        return found[0]
    return args[0] if args else next(iter(kwargs.values()))


@dataclass
class _Run:
    """State of one generation between ``begin`` and ``end``."""

    num_steps: int
    threshold: float
    warmup: int
    tail: int
    step: int = -1
    drift: float = 0.0          # accumulated relative change since the last computed step
    skipping: bool = False      # the current step skips the middle blocks
    kept_h1: Any = None         # block 0's output of the previous step (compared next step)
    anchor: Any = None          # h1 of the current computed step (the residual's base)
    residual: Any = None        # out_last - h1 of the last computed step
    like: Any = field(default=None, repr=False)  # block 0's output this step (shape template)

    def in_window(self) -> bool:
        return self.warmup <= self.step < self.num_steps - self.tail


class StepResidualCache:
    """Skips the middle DiT blocks on steps whose block-0 output barely moved."""

    def __init__(self) -> None:
        self.transformer: nn.Module | None = None
        self.blocks: nn.ModuleList | None = None
        self._run: _Run | None = None

    # -- public surface used by the runtime ------------------------------------------
    @property
    def active(self) -> bool:
        return self._run is not None

    def attach(self, transformer: nn.Module) -> "StepResidualCache":
        self.transformer = transformer
        _, self.blocks = find_primary_block_list(transformer)
        inner = transformer.forward

        @functools.wraps(inner)
        def counted_forward(*args, **kwargs):
            if self._run is not None:
                self._run.step += 1
            return inner(*args, **kwargs)

        transformer.forward = counted_forward
        for idx, block in enumerate(self.blocks):
            self.wrap_block(idx, block)
        return self

    def begin(self, num_steps: int, threshold: float, warmup: int = 3, tail: int = 2) -> None:
        self.end()
        usable = float(threshold) > 0.0 and int(num_steps) > 8 and self.blocks is not None and len(self.blocks) >= 2
        if usable:
            self._run = _Run(int(num_steps), float(threshold), int(warmup), int(tail))

    def end(self) -> None:
        self._run = None

    # -- block wrappers ----------------------------------------------------------------
    def wrap_block(self, idx: int, block: nn.Module) -> None:
        plain = getattr(block, "_uncached_forward", block.forward)
        block._uncached_forward = plain
        n = len(self.blocks) if self.blocks is not None else 0
        role = self._first if idx == 0 else (self._last if idx == n - 1 else self._middle)

        @functools.wraps(plain)
        def forward(*args, **kwargs):
            run = self._run
            if run is None:
                return block._uncached_forward(*args, **kwargs)
            return role(run, block._uncached_forward, args, kwargs)

        block.forward = forward

    def _first(self, run: _Run, call, args, kwargs):
        h1 = call(*args, **kwargs)
        run.like = h1
        if run.kept_h1 is None:
            run.drift = math.inf
            run.kept_h1 = _snapshot(h1)
        else:
            change, run.kept_h1 = _state_change(h1, run.kept_h1)
            run.drift += change
        run.skipping = run.in_window() and run.residual is not None and run.drift < run.threshold
        if not run.skipping:
            run.drift = 0.0
            # kept_h1 holds this step's h1 until block 0 of the next step, after
            # the last block has used it as the residual's base.
            run.anchor = run.kept_h1
        return h1

    def _middle(self, run: _Run, call, args, kwargs):
        if run.skipping:
            return _input_hidden(args, kwargs, run.like)
        return call(*args, **kwargs)

    def _last(self, run: _Run, call, args, kwargs):
        if run.skipping:
            return _tree_map(lambda x, r: x + r.to(dtype=x.dtype, device=x.device),
                             _input_hidden(args, kwargs, run.like), run.residual)
        out = call(*args, **kwargs)
        if run.anchor is not None:
            run.residual = _residual_into(out, run.anchor, run.residual)
            run.anchor = None
        return out
