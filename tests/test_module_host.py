"""CPU checks of the layer-loop schedule's host logic (no kernel is launched)."""

import pytest
import torch

from hrm_layer_ops.module import (ModuleNorms, module_bytes_per_token, reference_order_bytes_per_token,
                                  transformer_module)


def test_bytes_per_token():
    H, I = 2048, 5632
    # injection + pre-norm 8H; per layer two fused add+norm (8H each) + SwiGLU 6I
    assert module_bytes_per_token(H, I, 4) == 8 * H + 4 * (16 * H + 6 * I) == 282_624
    # reference order: add + copy (10H); per layer 2 norms, 2 adds, a copy, SwiGLU;
    # a copy before each later layer; final norm + copy
    assert reference_order_bytes_per_token(H, I, 4) == 10 * H + 4 * (24 * H + 6 * I) + 3 * 4 * H + 8 * H == 393_216


def test_norm_weights_lookup():
    w = [torch.zeros(4), torch.ones(4)]
    n = ModuleNorms(attn=w, final=w[1])
    assert n.at("attn", 1) is w[1] and n.at("ffn", 0) is None and ModuleNorms().at("attn", 0) is None


def test_rejects_empty_module_before_any_launch():
    z = torch.zeros((2, 8), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="at least one layer"):
        transformer_module(z, z, z, 0, None, None, None, None)
