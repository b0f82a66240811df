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


def test_folded_lora_operands_are_cached_until_an_input_changes():
    """ops._lora_operands reuses the folded (A_cat, B_cat) of a layer until an adapter tensor,
    its scale or the weight scale changes (an in-place edit bumps a tensor's version)."""
    from minimaxh3_b200 import ops

    g = torch.Generator().manual_seed(3)
    A = torch.randn(8, 64, generator=g).to(torch.bfloat16)
    Bm = torch.randn(32, 8, generator=g).to(torch.bfloat16)
    ws = torch.rand(1, 32, generator=g) + 0.5
    first = ops._lora_operands([(A, Bm, 1.0)], 32, 64, "cpu", col_scale=ws.reshape(-1), scale_src=ws)
    again = ops._lora_operands([(A, Bm, 1.0)], 32, 64, "cpu", col_scale=ws.reshape(-1), scale_src=ws)
    assert again[0] is first[0] and again[1] is first[1]
    fresh = ops._fold_lora([(A, Bm, 1.0)], 32, 64, "cpu", col_scale=ws.reshape(-1))
    assert torch.equal(fresh[0], first[0]) and torch.equal(fresh[1], first[1])
    Bm.mul_(2.0)
    edited = ops._lora_operands([(A, Bm, 1.0)], 32, 64, "cpu", col_scale=ws.reshape(-1), scale_src=ws)
    assert edited[1] is not first[1] and not torch.equal(edited[1], first[1])
    rescaled = ops._lora_operands([(A, Bm, 0.5)], 32, 64, "cpu", col_scale=ws.reshape(-1), scale_src=ws)
    assert torch.equal(rescaled[1].float(), (edited[1].float() * 0.5).to(torch.bfloat16).float())
    ws.mul_(2.0)
    new_scale = ops._lora_operands([(A, Bm, 0.5)], 32, 64, "cpu", col_scale=ws.reshape(-1), scale_src=ws)
    assert new_scale[1] is not rescaled[1]
