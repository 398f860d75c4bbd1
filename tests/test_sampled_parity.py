"""The sampled-row parity checker bench.py runs after its timed region (oracle/sampled.py), on CPU: a
capture built from the oracle's own whole-volume forward / backward passes every check, and a
mistake planted in one captured tensor (on the CPU, in the oracle's values) fails the matching one."""

import math

import numpy as np
import pytest
import torch

from oracle import dsa_oracle as O
from oracle import sampled

LOG2E = 1.4426950408889634


def _capture(seed=0, B=2, T=5, H=6, W=7, C=16, nh=2, ks=(3, 3, 5)):
    torch.manual_seed(seed)
    from megaslide_b200 import DeformableSlideAttention3D

    m = DeformableSlideAttention3D(C, nh, ks)
    with torch.no_grad():
        m.offset_net[2].weight.normal_(0, 0.3)
        m.offset_net[2].bias.normal_(0, 0.3)
    params = {k: v.detach().double().numpy() for k, v in m.state_dict().items()}
    rng = np.random.default_rng(seed)
    N = T * H * W
    x = rng.normal(size=(B, N, C))
    g = rng.normal(size=(B, N, C))
    y, cache = O.module_forward(params, x, (T, H, W), heads=nh, kernel_size=ks)
    dx, grads, _ = O.module_backward(cache, g)
    dattn = g @ params["out_proj.weight"]
    dq, dk, dv, doff, _, _ = O.attn_backward(cache["q"], cache["k"], cache["v"], cache["off32"], dattn, (T, H, W), nh,
                                             ks)
    f = lambda a: torch.from_numpy(np.ascontiguousarray(a.reshape(B * N, -1), dtype=np.float32))  # noqa: E731
    bias = params["offset_net.2.bias"].astype(np.float32)
    off_raw = (cache["off32"].astype(np.float64) - bias).astype(np.float32)  # the GEMM output, before the bias
    cap = dict(x2=f(x), qkv=torch.cat([f(cache["q"]), f(cache["k"]), f(cache["v"])], 1), hact=f(cache["hact"]),
               off=f(off_raw), offset_bias=torch.from_numpy(bias), attn=f(cache["attn"]),
               lse=torch.from_numpy(_lse(cache, nh, ks, T, H, W).astype(np.float32)), y=f(y), dy2=f(g), dattn=f(dattn),
               dqkv=torch.cat([f(dq), f(dk), f(dv)], 1), doff=f(doff), dx=f(dx))
    m.offset_net[2].weight.grad = torch.from_numpy(grads["offset_net.2.weight"]).float()
    m.offset_net[2].bias.grad = torch.from_numpy(grads["offset_net.2.bias"]).float()
    return m, cap, (T, H, W), B


def _lse(cache, nh, ks, T, H, W):
    _, lse = O.attn_forward(cache["q"], cache["k"], cache["v"], cache["off32"], (T, H, W), nh, ks)
    return lse * LOG2E  # the kernels store base-2 units


def test_checker_passes_oracle_capture():
    m, cap, vs, B = _capture()
    res = sampled.check(m, cap, vs, batch=B, dtype=torch.float32, n_rows=64, n_dx=8)
    bad = {k: v for k, v in res.items() if isinstance(v, dict) and not v["ok"]}
    assert res["ok"], bad
    for key in ("out_max_rel", "dq_fro", "doff_fro", "dk_block_fro", "dv_block_fro", "sum_dv_eq_sum_dout",
                "sum_dk_zero", "y_max_rel", "dx_fro", "doffset_w_proj", "doffset_b_fro"):
        assert key in res, key


@pytest.mark.parametrize("target,entry", [("dqkv_q", "dq_fro"), ("doff", "doff_fro"), ("attn", "out_max_rel"),
                                          ("dqkv_kv", "dk_block_fro"), ("y", "y_max_rel")])
def test_checker_catches_planted_mistake(target, entry):
    m, cap, vs, B = _capture(seed=1)
    C = cap["x2"].shape[1]
    if target == "dqkv_q":
        cap["dqkv"][:, :C] *= 1.05
    elif target == "dqkv_kv":
        cap["dqkv"][:, C:2 * C] *= 1.05
    else:
        cap[target] *= 1.05
    res = sampled.check(m, cap, vs, batch=B, dtype=torch.float32, n_rows=64, n_dx=8)
    assert not res[entry]["ok"], res[entry]
    assert not res["ok"]


def test_checker_time_window():
    """A rank's view of a time-sharded run: query frames [2, 4), K/V window [0, 5) of a 5-frame volume."""
    m, cap, vs, B = _capture(seed=2)
    T, H, W = vs
    HW = H * W
    C = cap["x2"].shape[1]
    q0, q1 = 2, 4
    sel_q = torch.cat([torch.arange(b * T * HW + q0 * HW, b * T * HW + q1 * HW) for b in range(B)])
    sc = dict(q=cap["qkv"][sel_q, :C], kv=cap["qkv"][:, C:], xw=cap["x2"].reshape(B, T * HW, C), win=(0, T),
              own=(q0, q1), hact=cap["hact"][sel_q], off=cap["off"][sel_q], offset_bias=cap["offset_bias"],
              attn=cap["attn"][sel_q], lse=cap["lse"][:, :, q0 * HW:q1 * HW].contiguous(), y=cap["y"][sel_q],
              dattn=cap["dattn"][sel_q], dq=cap["dqkv"][sel_q, :C], doff=cap["doff"][sel_q])
    # dK / dV of the own queries only, as a rank's backward produces before the halo return
    cache_dkv = _dkv_from_queries(m, cap, vs, B, sel_q.numpy())
    sc["dkv"] = cache_dkv
    res = sampled.check(m, sc, vs, batch=B, dtype=torch.float32, n_rows=48, q_frame0=q0, q_frames=q1 - q0,
                        kv_frame0=0, kv_frames=T, injected=True)
    bad = {k: v for k, v in res.items() if isinstance(v, dict) and not v["ok"]}
    assert res["ok"], bad


def _dkv_from_queries(m, cap, vs, B, rows):
    C = cap["x2"].shape[1]
    nh = m.num_heads
    ks = (m.k_t, m.k_h, m.k_w)
    r = O.attn_rows(cap["qkv"][rows, :C].numpy(), cap["off"][rows].numpy(), cap["qkv"][:, C:2 * C].numpy().copy(),
                    cap["qkv"][:, 2 * C:].numpy().copy(), rows, vs, nh, ks, dout_rows=cap["dattn"][rows].numpy(),
                    offset_bias=cap["offset_bias"].numpy(), watch_rows=np.arange(cap["qkv"].shape[0]))
    return torch.cat([torch.from_numpy(r["dk"]).float(), torch.from_numpy(r["dv"]).float()], 1)
