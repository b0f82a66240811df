"""The LoRA registry of unquantised linears (runtime/lora.py:206-226 contract), on CPU.

Registry contents, the ``adapters`` lists and the one-time wrapping follow
the reference; a layer without adapters runs its own forward and inputs the
fused GEMM cannot take (here: CPU tensors) get the reference's two-step
``out + sum scale (x A^T) B^T``.
"""
import torch
import torch.nn as nn

from minimaxh3_b200.kernels.lora import attach_lora_registry, fused_supported


class _Block(nn.Module):
    def __init__(self):
        super().__init__()
        self.proj = nn.Linear(16, 24)
        self.out = nn.Linear(24, 16, bias=False)
        self.norm = nn.LayerNorm(16)


def test_registry_wraps_linears_once():
    m = nn.Sequential(_Block(), _Block())
    reg = attach_lora_registry(m)
    assert sorted(reg) == ["0.out", "0.proj", "1.out", "1.proj"]
    for mod in reg.values():
        assert mod.adapters == [] and mod._lora_wrapped
    fwd = m[0].proj.forward
    attach_lora_registry(m)
    assert m[0].proj.forward is fwd                      # not wrapped twice


def test_no_adapters_is_the_plain_forward_and_cpu_gets_two_step_lora():
    torch.manual_seed(0)
    lin = nn.Linear(16, 24)
    attach_lora_registry(nn.Sequential(lin))
    x = torch.randn(5, 16)
    assert torch.equal(lin(x), x @ lin.weight.t() + lin.bias)
    A, B = torch.randn(4, 16), torch.randn(24, 4)
    lin.adapters = [(A, B, 0.5)]
    assert not fused_supported(lin, x)
    ref = x @ lin.weight.t() + lin.bias + 0.5 * ((x @ A.t()) @ B.t())
    assert torch.allclose(lin(x), ref, atol=1e-5)
