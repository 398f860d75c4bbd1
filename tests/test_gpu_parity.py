"""GPU parity: the sm_100a kernels (through the C ABI) against the reference's golden fixtures and
the CPU oracle.  Tolerances are the north star's: 1e-4 relative in float32, 2e-2 in bfloat16
(bf16 results are compared with the float64 oracle run on the same bf16-rounded inputs)."""

import math

import numpy as np
import pytest
import torch

import golden_cases as gc
import megaslide_b200 as msl
from megaslide_b200 import _lib, ops
from oracle import dsa_oracle as O

pytestmark = pytest.mark.gpu

RTOL_F32 = 1e-4
RTOL_BF16 = 2e-2
# bf16 gradients: relative Frobenius error <= RTOL_BF16 plus a max-abs sanity bound.  The reference's
# own bf16 path (autocast, attention.py run by examples/run_hybrid_attention_experiment.py:150-167)
# lands 4.7-4.8% (max-abs) / 1.5-2.4% (Frobenius) away from float64 on the extra_kv and
# tiny_large_offsets fixtures, so a 2% max-abs bar on gradients is stricter than the reference meets.
MAXREL_BF16_GRAD = 5e-2
DEV = "cuda:0"


@pytest.fixture(autouse=True)
def _no_tf32():
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = old


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def fro(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def run_module(case, dtype=torch.float32):
    C = case["x"].shape[-1]
    m = msl.DeformableSlideAttention3D(C, case["heads"], case["kernel"], offset_scale=case["offset_scale"])
    m.load_state_dict({k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in case["params"].items()})
    m = m.to(DEV)
    x = torch.from_numpy(case["x"]).to(DEV, dtype).requires_grad_(True)
    extra = None
    if case["extra"] is not None:
        extra = torch.from_numpy(case["extra"]).to(DEV, dtype).requires_grad_(True)
    y = m(x, case["video_shape"], extra_kv=extra)
    y.backward(torch.from_numpy(case["dy"]).to(DEV, dtype))
    torch.cuda.synchronize()
    return dict(y=y.detach().float().cpu().numpy(), dx=x.grad.float().cpu().numpy(),
                grads={k: p.grad.float().cpu().numpy() for k, p in m.named_parameters()},
                d_extra=None if extra is None else extra.grad.float().cpu().numpy(), offsets=None)


@pytest.mark.parametrize("name", gc.NAMES)
def test_module_fp32_matches_reference_golden(name):
    case = gc.load(name)
    res = run_module(case)
    errs = gc.case_errors(res, case)
    bad = {k: v for k, v in errs.items() if not v <= RTOL_F32}
    assert not bad, f"{name}: {bad}"


def _round_bf16(a):
    return torch.from_numpy(np.asarray(a, np.float32)).bfloat16().float().numpy()


@pytest.mark.parametrize("name", ["c1_window_small", "head_dim_72", "extra_kv", "tiny_large_offsets"])
def test_module_bf16_matches_oracle(name):
    case = gc.load(name)
    case = dict(case)
    case["params"] = {k: _round_bf16(v) for k, v in case["params"].items()}
    case["x"] = _round_bf16(case["x"])
    case["dy"] = _round_bf16(case["dy"])
    if case["extra"] is not None:
        case["extra"] = _round_bf16(case["extra"])
    res = run_module(case, torch.bfloat16)
    ref = gc.run_oracle(case)
    assert rel(res["y"], ref["y"]) < RTOL_BF16
    assert fro(res["dx"], ref["dx"]) < RTOL_BF16 and rel(res["dx"], ref["dx"]) < MAXREL_BF16_GRAD
    for k, g in ref["grads"].items():
        if k == "k_proj.bias":
            continue  # mathematically zero: rounding noise only
        assert fro(res["grads"][k], g) < RTOL_BF16 and rel(res["grads"][k], g) < MAXREL_BF16_GRAD, k


CORE_CASES = [
    # B, T, H, W, nh, d, kernel, G, offset_std
    (2, 3, 5, 6, 2, 8, (3, 3, 3), 0, 1.5),
    (1, 4, 6, 5, 2, 72, (3, 7, 7), 0, 1.0),
    (1, 3, 4, 4, 1, 128, (3, 7, 7), 2, 2.0),
    (1, 2, 3, 4, 3, 2, (1, 3, 3), 3, 0.5),
    (1, 1, 4, 4, 2, 16, (3, 3, 3), 0, 1.0),
    (2, 2, 1, 1, 1, 4, (3, 1, 1), 1, 0.0),
    (1, 5, 3, 7, 3, 12, (3, 3, 3), 0, 0.0),
    (1, 3, 5, 5, 2, 64, (3, 5, 5), 4, 3.0),
]


def _core_inputs(case, seed=0):
    B, T, H, W, nh, d, ks, G, ostd = case
    rng = np.random.default_rng(seed)
    N = T * H * W
    C = nh * d
    K = ks[0] * ks[1] * ks[2]
    q, k, v = (rng.normal(size=(B, N, C)).astype(np.float32) for _ in range(3))
    off = (rng.normal(size=(B, N, nh * K * 3)) * ostd).astype(np.float32)
    ek = rng.normal(size=(B, G, C)).astype(np.float32) if G else None
    ev = rng.normal(size=(B, G, C)).astype(np.float32) if G else None
    dout = rng.normal(size=(B, N, C)).astype(np.float32)
    return q, k, v, off, ek, ev, dout


def _run_core(case, arrays, dtype, dropout_p=0.0, seed=0):
    B, T, H, W, nh, d, ks, G, _ = case
    q, k, v, off, ek, ev, dout = arrays
    N = T * H * W
    C = nh * d
    t = lambda a: None if a is None else torch.from_numpy(a).to(DEV, dtype).reshape(-1, C)  # noqa: E731
    shape = ops.DsaShape(B, T, H, W, nh, d, ks, extra=G, dropout_p=dropout_p, dropout_seed=seed)
    offt = torch.from_numpy(off).to(DEV).reshape(B * N, -1)
    qt, kt_, vt, ekt, evt, dot = t(q), t(k), t(v), t(ek), t(ev), t(dout)
    out, lse = ops.attn_fwd(shape, qt, kt_, vt, offt, ekt, evt)
    dq, dk, dv, doff, dek, dev_ = ops.attn_bwd(shape, qt, kt_, vt, offt, out, lse, dot, ek=ekt, ev=evt)
    torch.cuda.synchronize()
    f = lambda a: None if a is None else a.float().cpu().numpy().reshape(B, -1, C)  # noqa: E731
    return dict(out=f(out), lse=lse.cpu().numpy(), dq=f(dq), dk=f(dk), dv=f(dv),
                doff=doff.cpu().numpy().reshape(B, N, -1), dek=f(dek), dev=f(dev_))


def _oracle_core(case, arrays, dropout_p=0.0, seed=0):
    B, T, H, W, nh, d, ks, G, _ = case
    q, k, v, off, ek, ev, dout = arrays
    out, lse = O.attn_forward(q, k, v, off, (T, H, W), nh, ks, ek, ev, dropout_p=dropout_p, seed=seed)
    dq, dk, dv, doff, dek, dev_ = O.attn_backward(q, k, v, off, dout, (T, H, W), nh, ks, ek, ev,
                                                  dropout_p=dropout_p, seed=seed)
    return dict(out=out, lse=lse / math.log(2.0), dq=dq, dk=dk, dv=dv, doff=doff, dek=dek, dev=dev_)


def _compare(got, ref, tol, skip=()):
    for key in ("out", "lse", "dq", "dk", "dv", "doff", "dek", "dev"):
        if key in skip or ref[key] is None:
            continue
        e = rel(got[key], ref[key])
        assert e < tol, f"{key}: rel err {e:.3e}"


@pytest.mark.parametrize("case", CORE_CASES, ids=lambda c: f"B{c[0]}T{c[1]}H{c[2]}W{c[3]}nh{c[4]}d{c[5]}k{''.join(map(str, c[6]))}G{c[7]}")
def test_core_fp32_matches_oracle(case):
    arrays = _core_inputs(case)
    _compare(_run_core(case, arrays, torch.float32), _oracle_core(case, arrays), RTOL_F32)


@pytest.mark.parametrize("case", CORE_CASES, ids=lambda c: f"B{c[0]}T{c[1]}H{c[2]}W{c[3]}nh{c[4]}d{c[5]}k{''.join(map(str, c[6]))}G{c[7]}")
def test_core_bf16_matches_oracle(case):
    arrays = tuple(None if a is None else (a if i == 3 else _round_bf16(a)) for i, a in enumerate(_core_inputs(case)))
    _compare(_run_core(case, arrays, torch.bfloat16), _oracle_core(case, arrays), RTOL_BF16)


def test_core_dropout_matches_oracle_mask():
    case = (1, 3, 4, 4, 2, 8, (3, 3, 3), 2, 1.0)
    arrays = _core_inputs(case, seed=3)
    got = _run_core(case, arrays, torch.float32, dropout_p=0.25, seed=99)
    ref = _oracle_core(case, arrays, dropout_p=0.25, seed=99)
    _compare(got, ref, RTOL_F32)
    plain = _oracle_core(case, arrays)
    assert rel(ref["out"], plain["out"]) > 1e-2  # the mask did something


def test_dwconv_kernels_match_oracle():
    rng = np.random.default_rng(5)
    for (B, T, H, W, C, ks) in [(1, 4, 5, 6, 16, (3, 7, 7)), (2, 3, 4, 4, 9, (3, 3, 3)), (1, 1, 3, 3, 8, (1, 3, 3))]:
        N = T * H * W
        K = ks[0] * ks[1] * ks[2]
        x = rng.normal(size=(B, N, C)).astype(np.float32)
        w = rng.normal(size=(K, C)).astype(np.float32)
        b = rng.normal(size=(C,)).astype(np.float32)
        dy = rng.normal(size=(B, N, C)).astype(np.float32)
        shape = ops.ConvShape(B, T, H, W, C, ks)
        for dt, tol in ((torch.float32, 1e-5), (torch.bfloat16, 2e-2)):
            xr = x if dt == torch.float32 else _round_bf16(x)
            dyr = dy if dt == torch.float32 else _round_bf16(dy)
            xt = torch.from_numpy(xr).to(DEV, dt).reshape(B * N, C)
            dyt = torch.from_numpy(dyr).to(DEV, dt).reshape(B * N, C)
            wt = torch.from_numpy(w).to(DEV)
            bt = torch.from_numpy(b).to(DEV)
            y = ops.dwconv_fwd(shape, xt, wt, bt)
            dx = ops.dwconv_bwd_data(shape, dyt, wt)
            gw = torch.zeros_like(wt)
            gb = torch.zeros_like(bt)
            ops.dwconv_bwd_weight(shape, dyt, xt, gw, gb)
            yo = O.dwconv3d(xr, w, b, (T, H, W), ks)
            dxo, gwo, gbo = O.dwconv3d_backward(dyr, xr, w, (T, H, W), ks)
            assert rel(y.float().cpu().numpy().reshape(B, N, C), yo) < tol
            assert rel(dx.float().cpu().numpy().reshape(B, N, C), dxo) < tol
            assert rel(gw.cpu().numpy(), gwo) < max(tol, 1e-5)
            assert rel(gb.cpu().numpy(), gbo) < max(tol, 1e-5)


@pytest.mark.parametrize("B,T,H,W,C,ks", [(1, 4, 5, 6, 16, (3, 7, 7)), (2, 3, 9, 40, 128, (3, 7, 7)),
                                          (1, 5, 6, 33, 64, (3, 3, 3))])
@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_dwconv_bwd_data_accumulates(B, T, H, W, C, ks, dt):
    """dx (float32) += conv_transpose(dy): the generic and the tiled kernels, bf16 / float32 dy."""
    rng = np.random.default_rng(17)
    N = T * H * W
    K = ks[0] * ks[1] * ks[2]
    w = rng.normal(size=(K, C)).astype(np.float32)
    dy = rng.normal(size=(B, N, C)).astype(np.float32)
    base = rng.normal(size=(B, N, C)).astype(np.float32)
    dyr = dy if dt == torch.float32 else _round_bf16(dy)
    shape = ops.ConvShape(B, T, H, W, C, ks)
    acc = torch.from_numpy(base).to(DEV).reshape(B * N, C).contiguous()
    dyt = torch.from_numpy(dyr).to(DEV, dt).reshape(B * N, C)
    out = ops.dwconv_bwd_data(shape, dyt, torch.from_numpy(w).to(DEV), out=acc, accumulate=True)
    assert out.data_ptr() == acc.data_ptr()
    dxo, _, _ = O.dwconv3d_backward(dyr, np.zeros_like(dyr), w, (T, H, W), ks)
    assert rel(acc.cpu().numpy().reshape(B, N, C), base + dxo) < 1e-5
    with pytest.raises(TypeError):
        ops.dwconv_bwd_data(shape, dyt, torch.from_numpy(w).to(DEV), out=acc.bfloat16(), accumulate=True)


# Shapes the shared-memory tiled kernels take (channels a multiple of 64 for bf16, 32 for float32; kernel
# widths 1/3/5/7): several 32-column tiles with a ragged last one, tile rows that do not divide H,
# frame chunks, frame windows (time shards), mixed dtypes and the fused epilogues.
DWCONV_TILED_CASES = [
    # B, T, H, W, C, kernel, x dtype, y dtype, epilogue, (in_frame0, in_frames, out_frame0, out_frames)
    (2, 5, 9, 40, 128, (3, 7, 7), torch.bfloat16, torch.bfloat16, "bias2", None),
    (1, 6, 7, 33, 64, (3, 3, 3), torch.float32, torch.float32, "none", None),
    (1, 4, 5, 8, 64, (1, 3, 3), torch.bfloat16, torch.float32, "gelu", None),
    (1, 8, 6, 16, 128, (3, 5, 5), torch.bfloat16, torch.bfloat16, "none", (2, 5, 3, 3)),
    (1, 3, 4, 5, 64, (3, 1, 1), torch.bfloat16, torch.float32, "gelu_grad", None),
    (1, 3, 34, 12, 32, (3, 7, 7), torch.float32, torch.bfloat16, "none", (0, 3, 1, 1)),
]


def _gelu64(u):
    return 0.5 * u * (1.0 + torch.erf(torch.from_numpy(u) / math.sqrt(2.0)).numpy())


def _gelu_grad64(u):
    t = torch.from_numpy(u)
    return (0.5 * (1.0 + torch.erf(t / math.sqrt(2.0))) + t * torch.exp(-0.5 * t * t) / math.sqrt(2.0 * math.pi)).numpy()


@pytest.mark.parametrize("case", DWCONV_TILED_CASES, ids=lambda c: f"T{c[1]}H{c[2]}W{c[3]}C{c[4]}k{''.join(map(str, c[5]))}{c[8]}")
def test_dwconv_tiled_path_matches_oracle(case):
    B, T, H, W, C, ks, xdt, ydt, epi, win = case
    rng = np.random.default_rng(23)
    HW, N, K = H * W, T * H * W, ks[0] * ks[1] * ks[2]
    i0, ni, o0, no = win if win else (0, T, 0, T)
    x = rng.normal(size=(B, T, HW, C))
    w = rng.normal(size=(K, C)).astype(np.float32) * 0.3
    b = rng.normal(size=(C,)).astype(np.float32)
    b2 = rng.normal(size=(C,)).astype(np.float32)
    dy = rng.normal(size=(B, T, HW, C))
    aux = rng.normal(size=(B, T, HW, C))
    if xdt == torch.bfloat16:
        x, dy = _round_bf16(x), _round_bf16(dy)
    if ydt == torch.bfloat16:
        aux = _round_bf16(aux)
    shape = ops.ConvShape(B, T, H, W, C, ks, in_frame0=i0, in_frames=ni, out_frame0=o0, out_frames=no)
    dev_rows = lambda a, f0, nf, dt: torch.from_numpy(np.ascontiguousarray(a[:, f0:f0 + nf])).to(DEV, dt).reshape(-1, C)  # noqa: E731
    xt = dev_rows(x, i0, ni, xdt)
    wt, bt, b2t = (torch.from_numpy(a).to(DEV) for a in (w, b, b2))
    kw = {}
    if epi == "bias2":
        kw = dict(bias=bt, bias2=b2t)
    elif epi == "gelu":
        kw = dict(bias=bt, epilogue=_lib.MSL_EPI_GELU)
    elif epi == "gelu_grad":
        kw = dict(bias=bt, epilogue=_lib.MSL_EPI_GELU_GRAD, aux=dev_rows(aux, o0, no, ydt))
    y = ops.dwconv_fwd(shape, xt, wt, out_dtype=ydt, **kw).float().cpu().numpy().reshape(B, no, HW, C)
    full = O.dwconv3d(x.reshape(B, N, C).astype(np.float32), w, b if epi != "none" else np.zeros(C, np.float32),
                      (T, H, W), ks).reshape(B, T, HW, C)[:, o0:o0 + no].astype(np.float64)
    if epi == "bias2":
        full = full + b2
    elif epi == "gelu":
        full = _gelu64(full)
    elif epi == "gelu_grad":
        full = aux[:, o0:o0 + no] * _gelu_grad64(full)
    tol = 2e-2 if torch.bfloat16 in (xdt, ydt) else 1e-5
    assert rel(y, full) < tol
    if win is not None:
        return  # input-gradient / weight-gradient windows are covered by the time-sharded tests
    dyt = dev_rows(dy, 0, T, xdt)
    dx = ops.dwconv_bwd_data(shape, dyt, wt).float().cpu().numpy().reshape(B, N, C)
    gw = torch.zeros_like(wt)
    gb = torch.zeros_like(bt)
    ops.dwconv_bwd_weight(shape, dyt, xt, gw, gb)
    dxo, gwo, gbo = O.dwconv3d_backward(dy.reshape(B, N, C).astype(np.float32), x.reshape(B, N, C).astype(np.float32),
                                        w, (T, H, W), ks)
    tolg = 2e-2 if xdt == torch.bfloat16 else 1e-5
    assert rel(dx, dxo) < tolg
    assert rel(gw.cpu().numpy(), gwo) < max(tolg, 1e-5)
    assert rel(gb.cpu().numpy(), gbo) < max(tolg, 1e-5)


def test_dwconv_weight_grad_float32_dy_bfloat16_x():
    """The module's offset-net branch: float32 du against bf16 x (tiled weight gradient, mixed dtypes)."""
    B, T, H, W, C, ks = 1, 4, 6, 40, 128, (3, 3, 3)
    rng = np.random.default_rng(29)
    N, K = T * H * W, 27
    x = _round_bf16(rng.normal(size=(B, N, C)))
    dy = rng.normal(size=(B, N, C)).astype(np.float32)
    w = rng.normal(size=(K, C)).astype(np.float32)
    shape = ops.ConvShape(B, T, H, W, C, ks)
    gw = torch.zeros(K, C, device=DEV)
    gb = torch.zeros(C, device=DEV)
    ops.dwconv_bwd_weight(shape, torch.from_numpy(dy).to(DEV).reshape(-1, C),
                          torch.from_numpy(x).to(DEV, torch.bfloat16).reshape(-1, C), gw, gb)
    _, gwo, gbo = O.dwconv3d_backward(dy, x.astype(np.float32), w, (T, H, W), ks)
    assert rel(gw.cpu().numpy(), gwo) < 1e-5
    assert rel(gb.cpu().numpy(), gbo) < 1e-5


# ----------------------------------------------------------------- reference's structural tests
def test_reference_shape_finite_and_gradients():
    """tests/test_megaslide_video.py:37-49 of the reference."""
    torch.manual_seed(0)
    attn = msl.DeformableSlideAttention3D(hidden_size=8, num_heads=2, kernel_size=(1, 3, 3)).to(DEV)
    x = torch.randn(2, 18, 8, device=DEV, requires_grad=True)
    y = attn(x, (2, 3, 3))
    assert y.shape == x.shape and torch.isfinite(y).all()
    y.square().mean().backward()
    assert x.grad is not None and torch.isfinite(x.grad).all()
    assert any(p.grad is not None for p in attn.parameters())


def test_reference_non_causal_over_time():
    """tests/test_megaslide_video.py:52-69 of the reference."""
    attn = msl.DeformableSlideAttention3D(hidden_size=2, num_heads=1, kernel_size=(3, 1, 1))
    with torch.no_grad():
        for p in attn.parameters():
            p.zero_()
        attn.v_proj.weight.copy_(torch.eye(2))
        attn.out_proj.weight.copy_(torch.eye(2))
    attn = attn.to(DEV)
    x = torch.zeros(1, 2, 2, device=DEV)
    changed = x.clone()
    changed[:, 1, :] = torch.tensor([3.0, -2.0], device=DEV)
    assert not torch.allclose(attn(x, (2, 1, 1))[:, 0], attn(changed, (2, 1, 1))[:, 0])


def test_reference_degenerate_grid():
    """tests/test_megaslide_video.py:72-84 of the reference."""
    attn = msl.DeformableSlideAttention3D(hidden_size=4, num_heads=2, kernel_size=(3, 3, 3)).to(DEV)
    x = torch.randn(1, 1, 4, device=DEV, requires_grad=True)
    y = attn(x, (1, 1, 1))
    assert y.shape == x.shape and torch.isfinite(y).all()
    y.sum().backward()
    assert torch.isfinite(x.grad).all()
    assert torch.count_nonzero(attn.offset_net[-1].weight) == 0


def test_reference_extra_kv():
    """tests/test_hybrid_attention.py:7-48 of the reference."""
    B, T, H, W, D, nh, G = 1, 2, 2, 2, 16, 4, 4
    attn = msl.DeformableSlideAttention3D(hidden_size=D, num_heads=nh, kernel_size=(1, 1, 1)).to(DEV)
    x = torch.randn(B, T * H * W, D, device=DEV)
    a = attn(x, (T, H, W))
    b = attn(x, (T, H, W), extra_kv=torch.randn(B, G, D, device=DEV))
    c = attn(x, (T, H, W), extra_kv=torch.zeros(B, G, D, device=DEV))
    assert a.shape == b.shape == c.shape == (B, T * H * W, D)
    assert not torch.allclose(a, b, atol=1e-5)


def test_trainer_style_autograd_grad_and_no_grad():
    """The CPU-master trainer runs the block under no_grad, then re-runs it with requires_grad toggled
    on the parameters and calls torch.autograd.grad (trainer.py:284-308, 418-449)."""
    torch.manual_seed(1)
    m = msl.DeformableSlideAttention3D(32, 4, (3, 3, 3)).to(DEV)
    for p in m.parameters():
        p.requires_grad_(False)
    x = torch.randn(1, 2 * 3 * 4, 32, device=DEV)
    with torch.no_grad():
        y0 = m(x, (2, 3, 4))
    for p in m.parameters():
        p.requires_grad_(True)
    xi = x.clone().requires_grad_(True)
    y1 = m(xi, (2, 3, 4))
    assert torch.equal(y0, y1.detach())
    grads = torch.autograd.grad(y1, (xi, *m.parameters()), grad_outputs=torch.ones_like(y1), allow_unused=True)
    assert all(g is not None and torch.isfinite(g).all() for g in grads)


def test_bf16_autocast_input():
    torch.manual_seed(2)
    m = msl.DeformableSlideAttention3D(32, 4, (3, 3, 3)).to(DEV)
    x = torch.randn(1, 24, 32, device=DEV, requires_grad=True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = m(x, (2, 3, 4))
    assert y.dtype == torch.bfloat16
    y.float().sum().backward()
    assert x.grad.dtype == torch.float32 and torch.isfinite(x.grad).all()
    y32 = m(x, (2, 3, 4))
    assert rel(y.float().detach().cpu().numpy(), y32.detach().cpu().numpy()) < 3e-2


def test_launches_counted_and_native_library_loaded():
    n0 = msl.launch_count()
    m = msl.DeformableSlideAttention3D(16, 2, (3, 3, 3)).to(DEV)
    x = torch.randn(1, 27, 16, device=DEV, requires_grad=True)
    m(x, (3, 3, 3)).sum().backward()
    torch.cuda.synchronize()
    assert msl.launch_count() - n0 >= 9
    import os

    maps = open(f"/proc/{os.getpid()}/maps").read()
    assert "libmegaslide_b200.so" in maps


# ----------------------------------------------------------------- tensor-core forward (bf16)
TC_CASES = [
    # B, T, H, W, nh, d, kernel, G, offset_std
    (1, 3, 9, 11, 2, 72, (3, 7, 7), 0, 1.0),      # partial 8x8 tiles, config-2 head_dim
    (2, 2, 16, 16, 2, 64, (3, 7, 7), 3, 0.5),     # extra keys, even chunk count (padded rows)
    (1, 2, 8, 8, 1, 128, (3, 3, 3), 0, 3.0),      # config-5 head_dim
    (1, 3, 6, 7, 2, 24, (3, 3, 3), 2, 2.0),       # odd number of 16-byte chunks: k8 tail
    (1, 2, 32, 32, 1, 16, (1, 3, 3), 0, 20.0),    # offsets of ~10 voxels: envelope split in chunks
    (1, 1, 5, 5, 2, 40, (1, 3, 3), 0, 0.0),       # T=1, zero offsets
]


def _tc_ids(c):
    return f"B{c[0]}T{c[1]}H{c[2]}W{c[3]}nh{c[4]}d{c[5]}k{''.join(map(str, c[6]))}G{c[7]}o{c[8]}"


def _run_fwd(case, arrays, algo, dropout_p=0.0, seed=0, status=None):
    B, T, H, W, nh, d, ks, G, _ = case
    q, k, v, off, ek, ev, _dout = arrays
    N = T * H * W
    C = nh * d
    t = lambda a: None if a is None else torch.from_numpy(a).to(DEV, torch.bfloat16).reshape(-1, C)  # noqa: E731
    shape = ops.DsaShape(B, T, H, W, nh, d, ks, extra=G, dropout_p=dropout_p, dropout_seed=seed, algo=algo)
    offt = torch.from_numpy(off).to(DEV).reshape(B * N, -1)
    out, lse = ops.attn_fwd(shape, t(q), t(k), t(v), offt, t(ek), t(ev), status=status)
    torch.cuda.synchronize()
    return out.float().cpu().numpy().reshape(B, N, C), lse.cpu().numpy()


@pytest.mark.parametrize("case", TC_CASES, ids=_tc_ids)
def test_tc_forward_matches_oracle_and_cuda_core_path(case):
    arrays = tuple(None if a is None else (a if i == 3 else _round_bf16(a))
                   for i, a in enumerate(_core_inputs(case, seed=7)))
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    out_tc, lse_tc = _run_fwd(case, arrays, algo=2, status=status)
    assert int(status.item()) == 0
    out_simt, lse_simt = _run_fwd(case, arrays, algo=1)
    ref = _oracle_core(case, arrays)
    assert rel(out_tc, ref["out"]) < RTOL_BF16
    assert rel(lse_tc, ref["lse"]) < 1e-3
    assert rel(out_tc, out_simt) < RTOL_BF16


def test_tc_forward_dropout_matches_oracle_mask():
    case = (1, 3, 8, 8, 2, 32, (3, 3, 3), 2, 1.0)
    arrays = tuple(None if a is None else (a if i == 3 else _round_bf16(a))
                   for i, a in enumerate(_core_inputs(case, seed=9)))
    out_tc, _ = _run_fwd(case, arrays, algo=2, dropout_p=0.3, seed=1234)
    ref = _oracle_core(case, arrays, dropout_p=0.3, seed=1234)
    assert rel(out_tc, ref["out"]) < RTOL_BF16


def test_tc_path_rejects_float32():
    case = (1, 2, 4, 4, 1, 16, (3, 3, 3), 0, 1.0)
    B, T, H, W, nh, d, ks, G, _ = case
    q = torch.randn(B * T * H * W, nh * d, device=DEV)
    off = torch.zeros(B * T * H * W, nh * 27 * 3, device=DEV)
    shape = ops.DsaShape(B, T, H, W, nh, d, ks, algo=2)
    with pytest.raises(msl.MslError, match="tensor-core"):
        ops.attn_fwd(shape, q, q, q, off)


# ----------------------------------------------------------------- tensor-core backward (bf16)
TC_BWD_CASES = [
    # B, T, H, W, nh, d, kernel, G(=0), offset_std
    (1, 3, 9, 11, 2, 72, (3, 7, 7), 0, 1.0),      # partial 4x8 tiles, config-2 head_dim (odd chunk count)
    (2, 2, 16, 16, 2, 64, (3, 7, 7), 0, 0.5),
    (1, 2, 8, 8, 1, 128, (3, 3, 3), 0, 3.0),      # largest head_dim (d-tile split over 8 warps)
    (1, 3, 6, 7, 2, 24, (3, 3, 3), 0, 2.0),       # k8 tail in every product
    (1, 2, 32, 32, 1, 16, (1, 3, 3), 0, 20.0),    # offsets of ~10 voxels: envelope split in chunks
    (1, 1, 5, 5, 2, 40, (1, 3, 3), 0, 0.0),       # T=1, zero offsets (samples on grid points)
    (1, 4, 5, 6, 1, 32, (3, 3, 3), 0, 6.0),       # many samples clamped onto the borders
    (2, 2, 16, 16, 2, 64, (3, 7, 7), 3, 0.5),     # extra keys (hybrid attention): dS . EK into dQ, d(ek), d(ev)
    (1, 3, 9, 11, 2, 72, (3, 7, 7), 64, 1.0),     # 64 extra keys, config-2 head_dim
]


def _run_tc_train(case, arrays, algo, dropout_p=0.0, seed=0, accumulate=False, doff_dtype=torch.float32,
                  offset_bias=None, expect_status=0):
    """Forward with the softmax weights saved (algo 2) or not (algo 1), then the backward."""
    B, T, H, W, nh, d, ks, G, _ = case
    q, k, v, off, ek, ev, dout = arrays
    N = T * H * W
    C = nh * d
    t = lambda a: None if a is None else torch.from_numpy(a).to(DEV, torch.bfloat16).reshape(-1, C)  # noqa: E731
    shape = ops.DsaShape(B, T, H, W, nh, d, ks, extra=G, dropout_p=dropout_p, dropout_seed=seed, algo=algo)
    offt = torch.from_numpy(off).to(DEV).reshape(B * N, -1)
    qt, kt_, vt, dot, ekt, evt = t(q), t(k), t(v), t(dout), t(ek), t(ev)
    probs, saved = ops.saved_buffers(shape, torch.bfloat16, DEV) if algo == 2 else (None, None)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    ob = None if offset_bias is None else torch.from_numpy(offset_bias).to(DEV)
    out, lse = ops.attn_fwd(shape, qt, kt_, vt, offt, ekt, evt, probs=probs, saved=saved, status=status,
                            offset_bias=ob)
    kw = {}
    if accumulate:
        kw = dict(dk_acc=torch.full((B * N, C), 0.5, device=DEV), dv_acc=torch.full((B * N, C), -0.25, device=DEV))
    dq, dk, dv, doff, dek, dev_ = ops.attn_bwd(shape, qt, kt_, vt, offt, out, lse, dot, ek=ekt, ev=evt, probs=probs,
                                               saved=saved, status=status, doff_dtype=doff_dtype, offset_bias=ob,
                                               **kw)
    assert doff.dtype == doff_dtype
    torch.cuda.synchronize()
    assert int(status.item()) == expect_status
    if accumulate:
        dk, dv = dk - 0.5, dv + 0.25
    f = lambda a: a.float().cpu().numpy().reshape(B, -1, C)  # noqa: E731
    res = dict(out=f(out), lse=lse.cpu().numpy(), dq=f(dq), dk=f(dk), dv=f(dv),
               doff=doff.float().cpu().numpy().reshape(B, N, -1))
    if G:
        res["dek"], res["dev"] = f(dek), f(dev_)
    if probs is not None:
        res["probs"] = probs.cpu().numpy()
    return res


def _compare_grads_bf16(got, ref, what):
    assert rel(got["out"], ref["out"]) < RTOL_BF16, f"{what} out"
    for key in ("dq", "dk", "dv", "doff") + (("dek", "dev") if got.get("dek") is not None else ()):
        ef, em = fro(got[key], ref[key]), rel(got[key], ref[key])
        assert ef < RTOL_BF16 and em < MAXREL_BF16_GRAD, f"{what} {key}: fro {ef:.3e} max {em:.3e}"


@pytest.mark.parametrize("algo", [1, 2])
def test_offset_bias_equals_the_materialised_sum(algo):
    """offset_bias: the kernels add the per-column bias as they read the offsets; the results are those of
    offsets + bias materialised in float32 (bit for bit, but dK / dV: the order of their float32 atomics
    differs from run to run, and the bf16 results then round a few elements the other way)."""
    case = TC_BWD_CASES[0]
    B, T, H, W, nh, d, ks, G, _ = case
    arrays = tuple(None if a is None else (a if i == 3 else _round_bf16(a))
                   for i, a in enumerate(_core_inputs(case, seed=29)))
    bias = (np.random.default_rng(3).normal(size=(nh * ks[0] * ks[1] * ks[2] * 3,)) * 0.7).astype(np.float32)
    summed = list(arrays)
    summed[3] = (arrays[3] + bias).astype(np.float32)
    ref = _run_tc_train(case, tuple(summed), algo=algo)
    got = _run_tc_train(case, arrays, algo=algo, offset_bias=bias)
    for key in ("out", "lse", "dq", "doff"):
        assert np.array_equal(got[key], ref[key]), key
    for key in ("dk", "dv"):
        assert fro(got[key], ref[key]) < 1e-3, key


@pytest.mark.parametrize("algo", [1, 2])
def test_bwd_bf16_offset_gradients_are_the_rounded_float32_ones(algo):
    """doff_dtype=bf16: both backward paths store the float32 offset gradient rounded to nearest even."""
    case = TC_BWD_CASES[0]
    arrays = tuple(None if a is None else (a if i == 3 else _round_bf16(a))
                   for i, a in enumerate(_core_inputs(case, seed=23)))
    full = _run_tc_train(case, arrays, algo=algo)["doff"]
    half = _run_tc_train(case, arrays, algo=algo, doff_dtype=torch.bfloat16)["doff"]
    expect = torch.from_numpy(full).bfloat16().float().numpy()
    assert np.array_equal(half, expect)


@pytest.mark.parametrize("case", TC_BWD_CASES, ids=_tc_ids)
def test_tc_backward_matches_oracle_and_cuda_core_path(case):
    arrays = tuple(None if a is None else (a if i == 3 else _round_bf16(a))
                   for i, a in enumerate(_core_inputs(case, seed=11)))
    got = _run_tc_train(case, arrays, algo=2)
    # the saved softmax weights are a distribution over the window of every (sample, head, query) (with
    # extra keys: the window's share of one)
    sums = got["probs"].astype(np.float64).sum(-1)
    if case[7] == 0:
        assert np.abs(sums - 1.0).max() < 1e-5
    else:
        assert sums.max() < 1.0 + 1e-5
    assert got["probs"].min() >= 0.0
    ref = _oracle_core(case, arrays)
    _compare_grads_bf16(got, ref, "tc vs oracle")
    simt = _run_tc_train(case, arrays, algo=1)
    _compare_grads_bf16(got, simt, "tc vs cuda-core")


LOAD_PATH_CASES = [
    (1, 3, 9, 11, 2, 72, (3, 7, 7), 0, 1.0),
    (2, 2, 16, 16, 2, 64, (3, 7, 7), 0, 0.5),     # even chunk count: boxes read 8 channels of the next head
    (1, 2, 32, 32, 2, 32, (1, 3, 3), 0, 20.0),    # envelope split in chunks
    (1, 4, 12, 20, 1, 72, (3, 5, 5), 0, 6.0),     # boxes past the volume's borders (zero fill)
]


@pytest.mark.parametrize("case", LOAD_PATH_CASES, ids=_tc_ids)
def test_tc_tma_and_cp_async_loads_agree_bitwise(case, monkeypatch):
    """The chunk loads by TMA tensor copies (default) and by cp.async (MSL_TC_LOADS=cpasync) fill
    every key the products use with the same values: forward, dQ and the offset gradient agree bit
    for bit; dK / dV are sums of float atomics from many CTAs (order-dependent rounding)."""
    arrays = tuple(None if a is None else (a if i == 3 else _round_bf16(a))
                   for i, a in enumerate(_core_inputs(case, seed=23)))
    monkeypatch.delenv("MSL_TC_LOADS", raising=False)
    tma = _run_tc_train(case, arrays, algo=2)
    monkeypatch.setenv("MSL_TC_LOADS", "cpasync")
    cpa = _run_tc_train(case, arrays, algo=2)
    for key in ("out", "lse", "probs", "dq", "doff"):
        assert np.array_equal(tma[key], cpa[key]), key
    for key in ("dk", "dv"):
        assert fro(tma[key], cpa[key]) < 1e-3, key


def test_tc_backward_dropout_matches_oracle_mask():
    case = (1, 3, 8, 8, 2, 32, (3, 3, 3), 0, 1.0)
    arrays = tuple(None if a is None else (a if i == 3 else _round_bf16(a))
                   for i, a in enumerate(_core_inputs(case, seed=13)))
    got = _run_tc_train(case, arrays, algo=2, dropout_p=0.3, seed=4321)
    ref = _oracle_core(case, arrays, dropout_p=0.3, seed=4321)
    _compare_grads_bf16(got, ref, "tc dropout vs oracle")


def test_tc_backward_accumulate_mode():
    case = (1, 3, 8, 8, 2, 32, (3, 3, 3), 0, 1.5)
    arrays = tuple(None if a is None else (a if i == 3 else _round_bf16(a))
                   for i, a in enumerate(_core_inputs(case, seed=17)))
    got = _run_tc_train(case, arrays, algo=2, accumulate=True)
    ref = _oracle_core(case, arrays)
    _compare_grads_bf16(got, ref, "tc accumulate vs oracle")


def test_tc_backward_requires_probs_when_forced():
    case = (1, 2, 4, 4, 1, 16, (3, 3, 3), 0, 1.0)
    B, T, H, W, nh, d, ks, G, _ = case
    x = torch.randn(B * T * H * W, nh * d, device=DEV, dtype=torch.bfloat16)
    off = torch.zeros(B * T * H * W, nh * 27 * 3, device=DEV)
    shape = ops.DsaShape(B, T, H, W, nh, d, ks, algo=2)
    out, lse = ops.attn_fwd(shape, x, x, x, off)
    with pytest.raises(msl.MslError, match="probs"):
        ops.attn_bwd(shape, x, x, x, off, out, lse, x)
    # the CUDA-core forward cannot fill probs: asking for them there is an error, not silent garbage
    simt = ops.DsaShape(B, T, H, W, nh, d, ks, algo=1)
    with pytest.raises(msl.MslError, match="probs"):
        ops.attn_fwd(simt, x, x, x, off, probs=ops.probs_buffer(simt, DEV))


def test_module_bf16_training_uses_tensor_core_backward(monkeypatch):
    """A bf16 training step of the module saves probs and the per-sample records in the forward and
    hands them to the backward."""
    from megaslide_b200.attention import DeformableSlideAttention3D

    seen = []
    real_bwd = ops.attn_bwd

    def spy(*a, **kw):
        seen.append(kw.get("probs") is not None and kw.get("saved") is not None)
        return real_bwd(*a, **kw)

    monkeypatch.setattr(ops, "attn_bwd", spy)
    torch.manual_seed(0)
    T, H, W, C, nh = 2, 8, 8, 64, 2
    m = DeformableSlideAttention3D(C, nh, kernel_size=(3, 3, 3)).to(DEV, torch.bfloat16)
    x = torch.randn(1, T * H * W, C, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    y = m(x, (T, H, W))
    y.float().square().mean().backward()
    torch.cuda.synchronize()
    assert torch.isfinite(x.grad.float()).all()
    for p in m.parameters():
        assert p.grad is not None and torch.isfinite(p.grad.float()).all()
    # with extra keys (HybridAttention3D's register tokens) as well
    e = torch.randn(1, 16, C, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    m(x, (T, H, W), extra_kv=e).float().square().mean().backward()
    torch.cuda.synchronize()
    assert e.grad is not None and torch.isfinite(e.grad.float()).all()
    assert seen == [True, True]


@pytest.mark.parametrize("heads,taps,pad", [(3, 27, 5), (3, 27, 1), (4, 147, 0)])
def test_offsets_absmax_with_bias(heads, taps, pad):
    """Per-axis max |(offsets + bias) * scale| over a strided offsets view, with and without the bias:
    scalar rows (row stride not a multiple of 4), 16-byte rows with a tail, 16-byte rows only."""
    rng = np.random.default_rng(41 + pad)
    n = heads * taps * 3
    off = (rng.normal(size=(257, n + pad)) * 2.0).astype(np.float32)
    bias = (rng.normal(size=(n,)) * 3.0).astype(np.float32)
    offt = torch.from_numpy(off).to(DEV)[:, :n]
    for b in (None, bias):
        full = off[:, :n] + (0 if b is None else b)
        want = np.abs(full.astype(np.float32) * np.float32(0.5)).reshape(-1, heads * taps, 3).max(axis=(0, 1))
        got = ops.offsets_absmax(offt, heads, taps, 0.5, bias=None if b is None else torch.from_numpy(b).to(DEV))
        assert np.array_equal(got.cpu().numpy(), want.astype(np.float32))


@pytest.mark.parametrize("rows,cols,src_pad,dst_pad", [(1000, 1152, 0, 2304), (37, 72, 8, 0), (5, 13, 3, 1),
                                                       (3, 64, 4, 0)])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_convert_f32_matches_torch(rows, cols, src_pad, dst_pad, dt):
    """float32 -> dtype conversion of strided row views: the 8-wide path (aligned rows, cols % 8 == 0) and
    the scalar one give torch's round-to-nearest-even conversion bit for bit."""
    g = torch.Generator(device=DEV)
    g.manual_seed(rows * 131 + cols)
    src = torch.randn(rows, cols + src_pad, device=DEV, generator=g)[:, :cols]
    dst_full = torch.zeros(rows, cols + dst_pad, device=DEV, dtype=dt)
    dst = dst_full[:, dst_pad:] if dst_pad else dst_full
    ops.convert_f32(src, dst)
    assert torch.equal(dst, src.to(dt))
    if dst_pad:
        assert not dst_full[:, :dst_pad].any()


def test_tc_oversized_envelope_falls_back_to_cuda_core():
    """Temporal offsets of tens of frames (T=48, W=8: a raw offset of 1 moves 3.4 frames): the tiles' key
    envelopes span more frames than the tensor-core sample records encode (29).  Those tiles are
    computed by the CUDA-core gather inside the tensor-core kernels, forward and backward alike; the
    results match the oracle and the CUDA-core kernels, and the status word reports the fallback
    (MSL_STATUS_TC_RANGE, informational) and nothing else."""
    case = (1, 48, 8, 8, 2, 72, (3, 7, 7), 0, 3.0)
    arrays = tuple(None if a is None else (a if i == 3 else _round_bf16(a))
                   for i, a in enumerate(_core_inputs(case, seed=31)))
    got = _run_tc_train(case, arrays, algo=2, expect_status=_lib.MSL_STATUS_TC_RANGE)
    ref = _oracle_core(case, arrays)
    _compare_grads_bf16(got, ref, "tc (fallback tiles) vs oracle")
    simt = _run_tc_train(case, arrays, algo=1)
    _compare_grads_bf16(got, simt, "tc (fallback tiles) vs cuda-core")


def _timeout_worker(q):
    import os

    import torch

    import megaslide_b200 as msl
    from megaslide_b200 import _lib, ops

    try:
        dev = "cuda:0"
        B, T, H, W, nh, d, ks = 1, 2, 4, 8, 2, 64, (3, 3, 3)  # nh*d >= the 72-channel TMA box
        N, C = T * H * W, nh * d
        g = torch.Generator(device=dev).manual_seed(5)
        q_, k_, v_ = (torch.randn(B * N, C, device=dev, generator=g).to(torch.bfloat16) for _ in range(3))
        off = torch.randn(B * N, nh * 27 * 3, device=dev, generator=g)
        shape = ops.DsaShape(B, T, H, W, nh, d, ks, algo=2)
        res = {}
        os.environ["MSL_TEST_TMA_NO_COPY"] = "1"
        st = torch.zeros(1, dtype=torch.int32, device=dev)
        ops.attn_fwd(shape, q_, k_, v_, off, status=st)
        torch.cuda.synchronize()
        res["timeout_status"] = int(st.item())
        del os.environ["MSL_TEST_TMA_NO_COPY"]
        st.zero_()
        out, _ = ops.attn_fwd(shape, q_, k_, v_, off, status=st)
        ref, _ = ops.attn_fwd(ops.DsaShape(B, T, H, W, nh, d, ks, algo=1), q_, k_, v_, off)
        torch.cuda.synchronize()
        res["after_status"] = int(st.item())
        res["after_err"] = float((out.float() - ref.float()).abs().max() / ref.float().abs().max())
        # the module: a timed-out call is reported by the status word (raised here synchronously)
        m = msl.DeformableSlideAttention3D(C, nh, ks).to(dev, torch.bfloat16)
        x = torch.randn(B, N, C, device=dev).to(torch.bfloat16).requires_grad_(True)
        os.environ["MSL_TEST_TMA_NO_COPY"] = "1"
        m(x, (T, H, W))
        del os.environ["MSL_TEST_TMA_NO_COPY"]
        try:
            msl.check_status()
            res["module_raised"] = False
        except msl.MslError as e:
            res["module_raised"] = "TMA" in str(e)
        res["clean_after"] = (msl.check_status() & _lib.MSL_STATUS_TIMEOUT) == 0
        q.put(("ok", res))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put(("error", repr(e)))


def test_bounded_tma_wait_times_out_cleanly():
    """The bounded TMA wait, made to run out on purpose in a child process: with the test hook
    MSL_TEST_TMA_NO_COPY=1 every chunk's barrier is armed for bytes that no copy delivers, so each CTA's
    first wait gives up after about a second, sets MSL_STATUS_TIMEOUT, skips the phases that read the
    key buffer and returns (no copy is in flight).  The context stays usable: without the hook the same
    call is valid again, and the module reports the timed-out call through its status word."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_timeout_worker, args=(q,))
    p.start()
    kind, res = q.get(timeout=300)
    p.join(timeout=60)
    assert kind == "ok", res
    assert p.exitcode == 0
    assert res["timeout_status"] & _lib.MSL_STATUS_TIMEOUT, res
    assert res["after_status"] == 0 and res["after_err"] < RTOL_BF16, res
    assert res["module_raised"] and res["clean_after"], res
