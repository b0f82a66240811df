"""Drop-in replacement for the reference's ``kernels/fp8_linear.py``.

Same public surface as viragadel6/minimaxh3 ``kernels/fp8_linear.py``:
``quantize_rows`` (:27-42), ``apply_lora_adapters`` (:45-55), ``FP8Linear``
with buffers ``w8`` / ``w_scale`` / ``bias`` and the mutable ``adapters``
list (:58-108), ``find_primary_block_list`` (:111-122) and
``convert_transformer_to_fp8`` (:125-162).

``FP8Linear.forward`` runs the activation quantisation and one sm_100a
tcgen05 GEMM whose epilogue applies the row/column scales, adds the bias,
adds every LoRA adapter's rank-r delta and writes bf16 once - where the
reference runs ``torch._scaled_mm`` and then one read-modify-write of the
output per adapter (:95-108, :45-55).  Registered as
``torch.ops.mh3.fp8_linear`` with a fake implementation for
``torch.compile``.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from .. import ops as _ops


def quantize_rows(x2d: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row e4m3 quantisation: (x8 [M,K], x_scale [M,1] f32).  fp8_linear.py:27-42."""
    if x2d.ndim != 2 or not x2d.is_cuda:
        raise ValueError("quantize_rows expects a 2D CUDA tensor")
    if x2d.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        # the reference's kernel loads any float dtype and computes in fp32 (:19)
        x2d = x2d.to(torch.float32)
    return _ops.quantize_rows(x2d)


def apply_lora_adapters(x: torch.Tensor, out: torch.Tensor, adapters) -> torch.Tensor:
    """``out + sum_i ((x A_i^T) B_i^T * scale_i)`` in the adapters' dtype (fp8_linear.py:45-55).

    Used for the plain ``nn.Linear`` layers that stay unquantised
    (runtime/lora.py wraps their forward with it); ``FP8Linear`` folds its
    adapters into the GEMM epilogue instead.
    """
    if not adapters:
        return out
    for A, B, scale in adapters:
        delta = (x.to(A.dtype) @ A.t()) @ B.t()
        out = out + (delta * scale).to(out.dtype)
    return out


class FP8Linear(nn.Module):
    """e4m3 weights with per-output-channel scales; fused scaled GEMM forward."""

    def __init__(self, in_features: int, out_features: int) -> None:
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.adapters: list[tuple[torch.Tensor, torch.Tensor, float]] = []

    @classmethod
    @torch.no_grad()
    def from_linear(cls, linear: nn.Linear) -> "FP8Linear":
        """Quantise ``linear``'s weight once (per output channel) and free it (:65-85)."""
        mod = cls(linear.in_features, linear.out_features)
        weight = linear.weight.detach()
        if not weight.is_cuda:
            weight = weight.cuda()
        w8, w_scale_col = quantize_rows(weight)
        mod.register_buffer("w8", w8)
        mod.register_buffer("w_scale", w_scale_col.view(1, -1).contiguous())
        bias = None
        if linear.bias is not None:
            bias = linear.bias.detach().to(device=w8.device, dtype=torch.bfloat16).contiguous()
        mod.register_buffer("bias", bias)
        if isinstance(getattr(linear, "adapters", None), list):
            mod.adapters = list(linear.adapters)
        linear.weight = None
        linear.bias = None
        return mod

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        x2d = x.reshape(-1, self.in_features)
        As = [a for a, _, _ in self.adapters]
        Bs = [b for _, b, _ in self.adapters]
        scales = [float(s) for _, _, s in self.adapters]
        out = torch.ops.mh3.fp8_linear(x2d, self.w8, self.w_scale, self.bias, As, Bs, scales)
        return out.reshape(*lead, self.out_features).to(x.dtype)


@torch.library.custom_op("mh3::fp8_linear", mutates_args=())
def _fp8_linear_op(x2d: torch.Tensor, w8: torch.Tensor, w_scale: torch.Tensor, bias: torch.Tensor | None,
                   lora_a: list[torch.Tensor], lora_b: list[torch.Tensor], lora_scale: list[float]) -> torch.Tensor:
    return _ops.fp8_linear(x2d, w8, w_scale, bias, list(zip(lora_a, lora_b, lora_scale)))


@_fp8_linear_op.register_fake
def _(x2d, w8, w_scale, bias, lora_a, lora_b, lora_scale):
    return x2d.new_empty((x2d.shape[0], w8.shape[0]), dtype=torch.bfloat16)


def find_primary_block_list(transformer: nn.Module) -> tuple[str, nn.ModuleList]:
    """The longest non-empty ModuleList, preferring homogeneous ones (:111-122).

    Ties go to the first such list in ``named_modules`` order, as with the
    reference's ``max``.
    """
    homogeneous, every = [], []
    for name, mod in transformer.named_modules():
        if isinstance(mod, nn.ModuleList) and len(mod) > 0:
            every.append((name, mod))
            if len({type(child) for child in mod}) == 1:
                homogeneous.append((name, mod))
    pool = homogeneous or every
    if not pool:
        raise ValueError("No non-empty nn.ModuleList found in transformer")
    best = pool[0]
    for item in pool[1:]:
        if len(item[1]) > len(best[1]):
            best = item
    return best


def _patterns(exclude_patterns) -> list[str]:
    items = exclude_patterns.split(",") if isinstance(exclude_patterns, str) else list(exclude_patterns)
    return [p.strip().lower() for p in items if p.strip()]


def convert_transformer_to_fp8(transformer: nn.Module, exclude_patterns, keep_edge_blocks: int) -> int:
    """Swap eligible ``nn.Linear`` layers of the primary blocks for ``FP8Linear`` (:125-162).

    Eligible: inside blocks [keep, n-keep) of the primary block list, in and
    out features both multiples of 16, and no exclusion pattern occurring in
    the lower-cased dotted path ``<list>.<idx>.<sub>``.  Returns the count.
    """
    pats = _patterns(exclude_patterns)
    list_name, blocks = find_primary_block_list(transformer)
    n = len(blocks)
    lo = max(0, int(keep_edge_blocks))
    hi = max(lo, n - int(keep_edge_blocks))
    count = 0
    for idx in range(lo, hi):
        block = blocks[idx]
        for sub_name, sub in list(block.named_modules()):
            if not isinstance(sub, nn.Linear):
                continue
            if sub.in_features % 16 or sub.out_features % 16:
                continue
            path = (f"{list_name}.{idx}.{sub_name}" if sub_name else f"{list_name}.{idx}").lower()
            if any(p in path for p in pats):
                continue
            new = FP8Linear.from_linear(sub)
            if not sub_name:
                blocks[idx] = new
            else:
                parent_name, _, attr = sub_name.rpartition(".")
                parent = block.get_submodule(parent_name) if parent_name else block
                setattr(parent, attr, new)
            count += 1
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
    return count
