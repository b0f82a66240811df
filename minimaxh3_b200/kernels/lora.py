"""LoRA on the unquantised ``nn.Linear`` layers: one fused bf16 GEMM.

The reference keeps some linears in bf16 (edge blocks, excluded names,
shapes not divisible by 16: fp8_linear.py:125-162) and gives them LoRA by
wrapping ``nn.Linear.forward`` (runtime/lora.py:206-226):
``out = linear(x); out = apply_lora_adapters(x, out, m.adapters)`` - a cuBLAS
GEMM, then per adapter two skinny matmuls and a read-modify-write of the
whole output (fp8_linear.py:45-55).

``attach_lora_registry`` keeps that function's contract (a registry of every
``nn.Linear`` / ``FP8Linear`` by name, an ``adapters`` list on each, the
``nn.Linear`` forwards wrapped once, ``_lora_wrapped`` set) but the wrapped
forward runs ``torch.ops.mh3.linear_lora``: the adapters' rank-r product is
accumulated into the same tcgen05 accumulator as ``x W^T`` and the output is
written once.  Layers without adapters run their own forward, as in the
reference; inputs the GEMM cannot take (not CUDA, K or N not a multiple of 8)
run the reference's two-step form.
"""
from __future__ import annotations

import functools

import torch
import torch.nn as nn

from .. import ops as _ops
from .fp8_linear import FP8Linear, apply_lora_adapters


@torch.library.custom_op("mh3::linear_lora", mutates_args=())
def _linear_lora_op(x2d: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, lora_a: list[torch.Tensor],
                    lora_b: list[torch.Tensor], lora_scale: list[float]) -> torch.Tensor:
    return _ops.linear_lora(x2d, weight, bias, list(zip(lora_a, lora_b, lora_scale)))


@_linear_lora_op.register_fake
def _(x2d, weight, bias, lora_a, lora_b, lora_scale):
    return x2d.new_empty((x2d.shape[0], weight.shape[0]), dtype=torch.bfloat16)


def fused_supported(module: nn.Linear, x: torch.Tensor) -> bool:
    """Whether the fused GEMM takes this layer and input."""
    w = module.weight
    return (x.is_cuda and w is not None and w.is_cuda and x.dtype in (torch.bfloat16, torch.float16)
            and w.dtype in (torch.bfloat16, torch.float16) and module.in_features % 8 == 0
            and module.out_features % 8 == 0)


def linear_lora_forward(module: nn.Linear, x: torch.Tensor) -> torch.Tensor:
    """``module(x)`` plus its adapters' deltas, in x's dtype and shape ``[..., out_features]``."""
    adapters = module.adapters
    lead = x.shape[:-1]
    x2d = x.reshape(-1, module.in_features)
    bias = None if module.bias is None else module.bias.to(torch.bfloat16)
    out = torch.ops.mh3.linear_lora(x2d, module.weight, bias, [a for a, _, _ in adapters],
                                    [b for _, b, _ in adapters], [float(s) for _, _, s in adapters])
    return out.reshape(*lead, module.out_features).to(x.dtype)


def attach_lora_registry(transformer: nn.Module) -> dict[str, nn.Module]:
    """runtime/lora.py:206-226 with the fused forward for ``nn.Linear`` layers."""
    registry: dict[str, nn.Module] = {}
    for name, mod in transformer.named_modules():
        if isinstance(mod, (nn.Linear, FP8Linear)):
            registry[name] = mod
            if not hasattr(mod, "adapters") or not isinstance(mod.adapters, list):
                mod.adapters = []
            if isinstance(mod, nn.Linear) and not getattr(mod, "_lora_wrapped", False):
                orig_forward = mod.forward

                def _make_forward(m: nn.Linear, fn):
                    @functools.wraps(fn)
                    def _forward(x: torch.Tensor) -> torch.Tensor:
                        if not m.adapters:
                            return fn(x)
                        if fused_supported(m, x):
                            return linear_lora_forward(m, x)
                        return apply_lora_adapters(x, fn(x), m.adapters)

                    return _forward

                mod.forward = _make_forward(mod, orig_forward)
                mod._lora_wrapped = True
    return registry
