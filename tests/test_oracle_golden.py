"""The CPU oracle against the reference module's own outputs (golden fixtures made by
tests/golden/make_golden.py from infinity/video/attention.py).  This pins the oracle that every
GPU parity test uses."""

import numpy as np
import pytest

import golden_cases as gc

# oracle = float64 arithmetic on float32 coordinates; reference = float32 throughout
RTOL = 2e-5


@pytest.mark.parametrize("name", gc.NAMES)
def test_oracle_matches_reference(name):
    case = gc.load(name)
    res = gc.run_oracle(case)
    errs = gc.case_errors(res, case)
    bad = {k: v for k, v in errs.items() if not v <= RTOL}
    assert not bad, f"{name}: {bad}"


def test_zero_offsets_hit_exact_voxel_centres():
    """With the zero-initialised offset head and odd sizes some sample coordinates are exact
    integers, where the trilinear derivative jumps; matching offset gradients there means the
    float32 coordinate arithmetic rounds exactly like the reference's."""
    case = gc.load("zero_offsets_odd")
    assert np.all(case["ref"]["offsets"] == 0)
    T, H, W = case["video_shape"]
    # centre sample of frame 2 (T=5): (2 + 1 - 1) * 5/4 - 1/2 = 2.0 exactly
    assert (2 * 2) * T / (T - 1) / 2 - 0.5 == 2.0
    res = gc.run_oracle(case)
    errs = gc.case_errors(res, case)
    assert errs["grad.offset_net.2.weight"] < RTOL


def test_noncausal_reference_construction():
    """tests/test_megaslide_video.py:52-69 of the reference: changing the token at t=1 changes the
    output at t=0 (k_t = 3)."""
    from oracle import dsa_oracle as O

    case = gc.load("noncausal_211")
    y1, _ = O.module_forward(case["params"], case["x"], (2, 1, 1), heads=1, kernel_size=(3, 1, 1))
    y0, _ = O.module_forward(case["params"], np.zeros_like(case["x"]), (2, 1, 1), heads=1, kernel_size=(3, 1, 1))
    assert not np.allclose(y1[:, 0], y0[:, 0])
    np.testing.assert_allclose(y1, case["ref"]["y"], rtol=1e-6, atol=1e-7)


def test_dropout_mask_rate_and_determinism():
    from oracle import dsa_oracle as O

    rng = np.random.default_rng(0)
    B, T, H, W, nh, d = 1, 2, 3, 3, 2, 4
    C = nh * d
    q, k, v = (rng.normal(size=(B, T * H * W, C)) for _ in range(3))
    off = np.zeros((B, T * H * W, nh * 27 * 3), np.float32)
    a1, _ = O.attn_forward(q, k, v, off, (T, H, W), nh, (3, 3, 3), dropout_p=0.3, seed=7)
    a2, _ = O.attn_forward(q, k, v, off, (T, H, W), nh, (3, 3, 3), dropout_p=0.3, seed=7)
    a3, _ = O.attn_forward(q, k, v, off, (T, H, W), nh, (3, 3, 3), dropout_p=0.3, seed=8)
    a0, _ = O.attn_forward(q, k, v, off, (T, H, W), nh, (3, 3, 3))
    assert np.array_equal(a1, a2)
    assert not np.allclose(a1, a3)
    assert not np.allclose(a1, a0)
