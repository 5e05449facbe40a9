"""The torch.library registrations: present, CUDA-only (no CPU kernel), layout
bytes round-trip."""

import pytest
import torch

from starkv import ops, torch_ops


def test_ops_are_registered():
    for name in ("decode_attn", "k_attn", "v_attn", "quant_append"):
        assert hasattr(torch.ops.starkv, name)


def test_layout_bytes_round_trip():
    lay = ops.make_layout(2, 8, 8, [16, 32, 96, 48, 16, 16, 64, 80], [64, 192], [4, 4], 300, True, torch.float16)
    back = torch_ops._layout(torch_ops.layout_tensor(lay))
    assert bytes(back) == bytes(lay)


def test_no_cpu_kernel():
    lay = ops.make_layout(1, 4, 4, [16] * 4, [64], [4], 128, True, torch.float16)
    with pytest.raises(NotImplementedError):
        torch.ops.starkv.k_attn(torch_ops.layout_tensor(lay), torch.zeros(1, 4, 128, dtype=torch.float16),
                                torch.zeros(128 * 64, dtype=torch.float16), torch.zeros(64),
                                torch.zeros(4 * 128 * 16, dtype=torch.int8), torch.ones(64, dtype=torch.float16), 5)
