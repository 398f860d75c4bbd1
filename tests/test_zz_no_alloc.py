"""msl_dsa_attn_bwd_noalloc: the backward entry point for callers that cannot allocate device
memory (a plugin inside a host engine that owns all device memory, or code that must not pay an
allocation's implicit synchronisation mid-step).  It is called through the C ABI, twice in a row,
and must reproduce the workspace entry point msl_dsa_attn_bwd within the float32 parity tolerance.
The file sorts last so a failure here cannot hide failures of the other tests; it depends on no
other test and also passes alone in a fresh process."""

import ctypes

import numpy as np
import pytest
import torch

from megaslide_b200 import _lib, ops

pytestmark = pytest.mark.gpu

RTOL_F32 = 1e-4


def _rel(a, b):
    a = a.double().cpu()
    b = b.double().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def test_noalloc_backward_matches_workspace_entry_point():
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    rng = np.random.default_rng(21)
    B, T, H, W, nh, d, ks, G = 2, 3, 5, 6, 2, 8, (3, 3, 3), 2
    N, C, K = T * H * W, nh * d, ks[0] * ks[1] * ks[2]
    t = lambda a: torch.from_numpy(a.astype(np.float32)).to(dev)  # noqa: E731
    q, k, v, dout = (t(rng.normal(size=(B * N, C))) for _ in range(4))
    ek, ev = t(rng.normal(size=(B * G, C))), t(rng.normal(size=(B * G, C)))
    off = t(rng.normal(size=(B * N, nh * K * 3)) * 1.5)
    shape = ops.DsaShape(B, T, H, W, nh, d, ks, extra=G)
    out, lse = ops.attn_fwd(shape, q, k, v, off, ek, ev)
    want = ops.attn_bwd(shape, q, k, v, off, out, lse, dout, ek=ek, ev=ev)  # workspace entry point

    lib = _lib.load()
    geom = shape.geometry(torch.float32)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for _call in range(2):
        dq, dk, dv = (torch.full((B * N, C), float("nan"), device=dev) for _ in range(3))
        doff = torch.full((B * N, nh * K * 3), float("nan"), device=dev)
        dek, dev_ = (torch.full((B * G, C), float("nan"), device=dev) for _ in range(2))
        io = _lib.DsaBwdIO(
            q.data_ptr(), C, k.data_ptr(), C, v.data_ptr(), C, off.data_ptr(), nh * K * 3,
            ek.data_ptr(), ev.data_ptr(), C, out.data_ptr(), C, lse.data_ptr(), dout.data_ptr(), C,
            dq.data_ptr(), C, dk.data_ptr(), dv.data_ptr(), C, None, None, 0,
            doff.data_ptr(), nh * K * 3, dek.data_ptr(), dev_.data_ptr(), None)
        rc = lib.msl_dsa_attn_bwd_noalloc(ctypes.byref(geom), ctypes.byref(io), stream)
        assert rc == _lib.MSL_OK, lib.msl_last_error().decode()
        torch.cuda.synchronize()
        for got, ref in zip((dq, dk, dv, doff, dek, dev_), want):
            assert torch.isfinite(got).all()
            assert _rel(got, ref) < RTOL_F32


def test_noalloc_rejects_problems_beyond_the_static_scratch():
    lib = _lib.load()
    # float32 dK + dV accumulators of 2 x 64 x 64 x 64 tokens x 512 channels = 1 GiB > 64 MiB
    shape = ops.DsaShape(2, 64, 64, 64, 8, 64, (3, 3, 3))
    geom = shape.geometry(torch.bfloat16)
    need = lib.msl_dsa_attn_bwd_workspace_bytes(ctypes.byref(geom), 0)
    assert need > _lib.MSL_NOALLOC_SCRATCH_BYTES
    io = _lib.DsaBwdIO()
    rc = lib.msl_dsa_attn_bwd_noalloc(ctypes.byref(geom), ctypes.byref(io), None)
    assert rc == _lib.MSL_ERR_WORKSPACE
    assert "static array" in lib.msl_last_error().decode()
