"""The oracle's row-sampled core op (attn_rows, used to check full-size runs at sampled rows) against
its whole-volume forward / backward, on CPU: full and time-windowed query / K-V frames, float32 and
bf16 operands, offset bias, dropout, watched dK / dV rows."""

import numpy as np
import pytest

from oracle import dsa_oracle as O


def _bf16_bits(a):
    """Round float64 -> bf16 (nearest even); returns (uint16 bit patterns, the rounded float64 values)."""
    f = np.asarray(a, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    back = (u.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    return u, back


def _case(seed=0, B=2, T=6, H=5, W=7, nh=2, d=8, ks=(3, 3, 5), ostd=1.5, bstd=0.3):
    rng = np.random.default_rng(seed)
    C = nh * d
    K = ks[0] * ks[1] * ks[2]
    N = T * H * W
    q, k, v, dout = (rng.normal(size=(B, N, C)) for _ in range(4))
    off = rng.normal(0, ostd, (B, N, nh * K * 3)).astype(np.float32)
    bias = rng.normal(0, bstd, nh * K * 3).astype(np.float32)
    return dict(B=B, T=T, H=H, W=W, nh=nh, d=d, ks=ks, C=C, N=N, q=q, k=k, v=v, dout=dout, off=off, bias=bias)


@pytest.mark.parametrize("dropout", [0.0, 0.25])
def test_rows_match_whole_volume(dropout):
    c = _case()
    B, N, C, nh, ks = c["B"], c["N"], c["C"], c["nh"], c["ks"]
    vs = (c["T"], c["H"], c["W"])
    offb = (c["off"] + c["bias"]).astype(np.float32)
    out, lse = O.attn_forward(c["q"], c["k"], c["v"], offb, vs, nh, ks, dropout_p=dropout, seed=11)
    dq, dk, dv, doff, _, _ = O.attn_backward(c["q"], c["k"], c["v"], offb, c["dout"], vs, nh, ks,
                                             dropout_p=dropout, seed=11)
    rng = np.random.default_rng(1)
    qidx = np.sort(rng.choice(B * N, 37, replace=False))
    f32 = lambda a: np.ascontiguousarray(a.reshape(B * N, -1), dtype=np.float32)  # noqa: E731
    # float32 operands: the oracle reads them as float32, so compare with the float32-rounded inputs
    q32, k32, v32, d32 = (f32(c[n]) for n in ("q", "k", "v", "dout"))
    out32, lse32 = O.attn_forward(q32.reshape(B, N, C), k32.reshape(B, N, C), v32.reshape(B, N, C), offb, vs, nh, ks,
                                  dropout_p=dropout, seed=11)
    dq32, dk32, dv32, doff32, _, _ = O.attn_backward(q32.reshape(B, N, C), k32.reshape(B, N, C), v32.reshape(B, N, C),
                                                     offb, d32.reshape(B, N, C), vs, nh, ks, dropout_p=dropout, seed=11)
    # every key row the listed queries reach gets the full dK / dV only if all queries are listed
    all_q = np.arange(B * N)
    r = O.attn_rows(q32[all_q], c["off"].reshape(B * N, -1)[all_q], k32, v32, all_q, vs, nh, ks,
                    dout_rows=d32[all_q], offset_bias=c["bias"], watch_rows=np.arange(B * N),
                    dropout_p=dropout, seed=11)
    assert r["misses"] == 0
    np.testing.assert_allclose(r["out"], out32.reshape(B * N, C), rtol=1e-10, atol=1e-10)
    np.testing.assert_allclose(r["dq"], dq32.reshape(B * N, C), rtol=1e-10, atol=1e-10)
    np.testing.assert_allclose(r["doff"], doff32.reshape(B * N, -1), rtol=1e-9, atol=1e-10)
    np.testing.assert_allclose(r["dk"], dk32.reshape(B * N, C), rtol=1e-9, atol=1e-10)
    np.testing.assert_allclose(r["dv"], dv32.reshape(B * N, C), rtol=1e-9, atol=1e-10)
    np.testing.assert_allclose(r["lse"], lse32.transpose(0, 2, 1).reshape(B * N, nh), rtol=1e-12)
    # a subset of rows: the same values for those rows
    s = O.attn_rows(q32[qidx], c["off"].reshape(B * N, -1)[qidx], k32, v32, qidx, vs, nh, ks,
                    dout_rows=d32[qidx], offset_bias=c["bias"], dropout_p=dropout, seed=11)
    np.testing.assert_allclose(s["out"], r["out"][qidx], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(s["doff"], r["doff"][qidx], rtol=1e-12, atol=1e-12)
    # float64 whole-volume run vs float32 operands: only input rounding apart
    np.testing.assert_allclose(s["out"], out.reshape(B * N, C)[qidx], rtol=1e-5, atol=1e-5)


def test_rows_bf16_operands():
    c = _case(seed=3, ostd=0.7)
    B, N, C, nh, ks = c["B"], c["N"], c["C"], c["nh"], c["ks"]
    vs = (c["T"], c["H"], c["W"])
    bits, vals = {}, {}
    for n in ("q", "k", "v", "dout"):
        bits[n], vals[n] = _bf16_bits(c[n].reshape(B * N, C))
    offb = (c["off"] + c["bias"]).astype(np.float32)
    out, _ = O.attn_forward(*(vals[n].reshape(B, N, C) for n in ("q", "k", "v")), offb, vs, nh, ks)
    dq, _, _, doff, _, _ = O.attn_backward(*(vals[n].reshape(B, N, C) for n in ("q", "k", "v")), offb,
                                           vals["dout"].reshape(B, N, C), vs, nh, ks)
    qidx = np.arange(0, B * N, 5)
    r = O.attn_rows(bits["q"][qidx], c["off"].reshape(B * N, -1)[qidx], bits["k"], bits["v"], qidx, vs, nh, ks,
                    dout_rows=bits["dout"][qidx], offset_bias=c["bias"])
    np.testing.assert_allclose(r["out"], out.reshape(B * N, C)[qidx], rtol=1e-11, atol=1e-11)
    np.testing.assert_allclose(r["dq"], dq.reshape(B * N, C)[qidx], rtol=1e-10, atol=1e-11)
    np.testing.assert_allclose(r["doff"], doff.reshape(B * N, -1)[qidx], rtol=1e-9, atol=1e-11)


def test_rows_time_windows():
    """Query frames [3, 5) against K/V frames [1, 6) of a 6-frame volume: global coordinates, window rows."""
    c = _case(seed=5, ostd=0.05, bstd=0.05)
    B, N, C, nh, ks = c["B"], c["N"], c["C"], c["nh"], c["ks"]
    T, H, W = c["T"], c["H"], c["W"]
    HW = H * W
    f32 = lambda a: np.ascontiguousarray(a, dtype=np.float32)  # noqa: E731
    q, k, v, dout = (f32(c[n]) for n in ("q", "k", "v", "dout"))
    offb = (c["off"] + c["bias"]).astype(np.float32)
    out, _ = O.attn_forward(q, k, v, offb, (T, H, W), nh, ks)
    dq, dk, dv, doff, _, _ = O.attn_backward(q, k, v, offb, dout, (T, H, W), nh, ks)
    qf0, qf, kf0, kf = 3, 2, 1, 5
    qsl = slice(qf0 * HW, (qf0 + qf) * HW)
    ksl = slice(kf0 * HW, (kf0 + kf) * HW)
    qloc = q[:, qsl].reshape(-1, C)
    r = O.attn_rows(qloc, c["off"][:, qsl].reshape(-1, nh * 45 * 3), k[:, ksl].reshape(-1, C), v[:, ksl].reshape(-1, C),
                    np.arange(qloc.shape[0]), (T, H, W), nh, ks, dout_rows=dout[:, qsl].reshape(-1, C),
                    offset_bias=c["bias"], q_frame0=qf0, q_frames=qf, kv_frame0=kf0, kv_frames=kf)
    assert r["misses"] == 0
    np.testing.assert_allclose(r["out"], out[:, qsl].reshape(-1, C), rtol=1e-10, atol=1e-10)
    np.testing.assert_allclose(r["dq"], dq[:, qsl].reshape(-1, C), rtol=1e-10, atol=1e-10)
    np.testing.assert_allclose(r["doff"], doff[:, qsl].reshape(-1, nh * 45 * 3), rtol=1e-9, atol=1e-10)
    # a window too small for the offsets reports the corners it could not read
    r2 = O.attn_rows(qloc, c["off"][:, qsl].reshape(-1, nh * 45 * 3), k[:, qsl].reshape(-1, C),
                     v[:, qsl].reshape(-1, C), np.arange(qloc.shape[0]), (T, H, W), nh, ks,
                     q_frame0=qf0, q_frames=qf, kv_frame0=qf0, kv_frames=qf, offset_bias=c["bias"])
    assert r2["misses"] > 0
