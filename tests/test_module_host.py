"""Host-side behaviour of the drop-in module that needs no GPU: constructor, parameter names and
shapes, state-dict round trip with the reference's fixtures, and loud failure off-GPU."""

import numpy as np
import pytest
import torch

import golden_cases as gc
from megaslide_b200 import DeformableSlideAttention3D


def test_parameter_names_and_shapes_match_reference():
    case = gc.load("c1_window_small")
    ref_names = sorted(case["params"])
    m = DeformableSlideAttention3D(32, 4, (3, 7, 7))
    sd = m.state_dict()
    assert sorted(sd) == ref_names
    for k in ref_names:
        assert tuple(sd[k].shape) == case["params"][k].shape, k
    m.load_state_dict({k: torch.from_numpy(v) for k, v in case["params"].items()})


def test_offset_head_zero_initialised_and_attributes():
    m = DeformableSlideAttention3D(16, 2, (3, 3, 3), offset_scale=0.5, dropout=0.1)
    assert torch.count_nonzero(m.offset_net[-1].weight) == 0
    assert torch.count_nonzero(m.offset_net[-1].bias) == 0
    assert (m.hidden_size, m.num_heads, m.head_dim) == (16, 2, 8)
    assert (m.k_t, m.k_h, m.k_w) == (3, 3, 3)
    assert m.offset_scale == 0.5 and m.dropout.p == 0.1
    assert m.offset_net[2].out_channels == 2 * 27 * 3


def test_default_init_matches_module_construction_order():
    """Same submodules in the same order as the reference: a torch seed gives identical weights
    to constructing nn.Linear / nn.Conv3d in that order."""
    torch.manual_seed(3)
    m = DeformableSlideAttention3D(8, 2, (1, 3, 3))
    torch.manual_seed(3)
    lins = [torch.nn.Linear(8, 8) for _ in range(4)]
    dw = torch.nn.Conv3d(8, 8, (1, 3, 3), padding=(0, 1, 1), groups=8)
    off0 = torch.nn.Conv3d(8, 8, 3, padding=1, groups=8)
    assert torch.equal(m.q_proj.weight, lins[0].weight) and torch.equal(m.out_proj.bias, lins[3].bias)
    assert torch.equal(m.dw_conv.weight, dw.weight) and torch.equal(m.offset_net[0].weight, off0.weight)


def test_cpu_tensors_fail_loudly():
    m = DeformableSlideAttention3D(8, 2, (1, 3, 3))
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.randn(1, 8, 8), (2, 2, 2))


def test_shape_assertions_as_reference():
    m = DeformableSlideAttention3D(8, 2, (1, 3, 3))
    with pytest.raises(AssertionError, match="Expected N=8"):
        m(torch.randn(1, 9, 8), (2, 2, 2))
    with pytest.raises(AssertionError):
        m(torch.randn(1, 8, 4), (2, 2, 2))


def test_golden_fixtures_regenerate_deterministically():
    case = gc.load("c1_full")
    assert case["x"].shape == (1, 2048, 256)
    again = gc.load("c1_full")
    assert np.array_equal(case["x"], again["x"])
