"""Argument checks of the host-resident attention API (no GPU needed)."""
import pytest
import torch

from minimaxh3_b200.streaming import fp8_attention_host


def test_fp8_attention_host_validates_before_any_device_work():
    q = torch.zeros(1, 2, 8, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        fp8_attention_host(q, q[:, :1].contiguous(), q[:, :1].contiguous())  # head counts differ
    with pytest.raises(ValueError):
        fp8_attention_host(q, q, q, out=torch.zeros(1, 2, 8, 32, dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        fp8_attention_host(q.transpose(2, 3), q, q)  # not contiguous
