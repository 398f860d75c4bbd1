"""CPU oracle for DeformableSlideAttention3D — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s cpu_baseline / ``--impl reference``
arm may import this module; the product package ``megaslide_b200`` never does.

It restates the reference module ``infinity/video/attention.py`` (jasonliu0704/megaslide) in
numpy float64 plus the C kernels of ``dsa_oracle.c``:

* ``module_forward`` follows ``DeformableSlideAttention3D.forward`` (attention.py:82-192):
  depthwise ``dw_conv`` term (:102), offset net dwconv3^3 -> GELU(erf) -> 1x1 conv (:70-74, :105),
  offsets * offset_scale (:106), q/k/v projections (:130-132), deformable trilinear sampling and
  local softmax attention (:113-183, :194-273), optional ``extra_kv`` (:159-173),
  ``out_proj`` + dw term (:186-192).
* ``module_backward`` is the hand-derived gradient of the same graph (what autograd computes for
  the reference).

Parameters use the reference's state-dict names and shapes (attention.py:52-74).
The raw offsets are rounded to float32 before the coordinate arithmetic, which is float32 in
the reference (the base grid is always float32, attention.py:209-216).
"""

from __future__ import annotations

import ctypes
import math
from pathlib import Path
from typing import Optional

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB: Optional[ctypes.CDLL] = None

PARAM_SHAPES_DOC = {
    "q_proj.weight": "[C, C]", "q_proj.bias": "[C]",
    "k_proj.weight": "[C, C]", "k_proj.bias": "[C]",
    "v_proj.weight": "[C, C]", "v_proj.bias": "[C]",
    "out_proj.weight": "[C, C]", "out_proj.bias": "[C]",
    "dw_conv.weight": "[C, 1, kt, kh, kw]", "dw_conv.bias": "[C]",
    "offset_net.0.weight": "[C, 1, 3, 3, 3]", "offset_net.0.bias": "[C]",
    "offset_net.2.weight": "[nh*kt*kh*kw*3, C, 1, 1, 1]", "offset_net.2.bias": "[nh*kt*kh*kw*3]",
}
PARAM_NAMES = list(PARAM_SHAPES_DOC)


class _Geom(ctypes.Structure):
    _fields_ = [
        ("B", ctypes.c_int32), ("T", ctypes.c_int32), ("H", ctypes.c_int32), ("W", ctypes.c_int32),
        ("nh", ctypes.c_int32), ("d", ctypes.c_int32), ("kt", ctypes.c_int32), ("kh", ctypes.c_int32),
        ("kw", ctypes.c_int32), ("G", ctypes.c_int32), ("softmax_scale", ctypes.c_double),
        ("offset_scale", ctypes.c_float), ("dropout_p", ctypes.c_float), ("dropout_seed", ctypes.c_uint64),
    ]


def _lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        path = _HERE / "_build" / "libdsa_oracle.so"
        if not path.exists():
            from . import build as _b  # built lazily where gcc exists (here and on the GPU box)

            _b.build()
        lib = ctypes.CDLL(str(path))
        P = ctypes.c_void_p
        lib.oracle_dsa_fwd.argtypes = [ctypes.POINTER(_Geom), P, P, P, P, P, P, P, P]
        lib.oracle_dsa_bwd.argtypes = [ctypes.POINTER(_Geom)] + [P] * 13
        lib.oracle_dsa_rows.argtypes = ([ctypes.POINTER(_Geom)] + [ctypes.c_int] * 4 + [ctypes.c_long, P, P, P,
                                        ctypes.c_long, P, P, P, P, ctypes.c_long, ctypes.c_int, P, P, P, P, P,
                                        ctypes.c_long, P, P])
        lib.oracle_dsa_rows.restype = ctypes.c_long
        i = ctypes.c_int
        lib.oracle_dwconv3d.argtypes = [i] * 8 + [P] * 4
        lib.oracle_dwconv3d_bwd.argtypes = [i] * 8 + [P] * 6
        lib.oracle_gelu.argtypes = [ctypes.c_long, P, P]
        lib.oracle_gelu_grad.argtypes = [ctypes.c_long, P, P]
        lib.oracle_num_threads.restype = ctypes.c_int
        lib.oracle_set_num_threads.argtypes = [ctypes.c_int]
        _LIB = lib
    return _LIB


def num_threads() -> int:
    return int(_lib().oracle_num_threads())


def set_num_threads(n: int) -> None:
    _lib().oracle_set_num_threads(int(n))


def _f64(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float64))


def _ptr(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _geom(video_shape, heads, head_dim, kernel_size, batch, extra, softmax_scale, offset_scale, dropout_p, seed):
    T, H, W = video_shape
    kt, kh, kw = kernel_size
    return _Geom(batch, T, H, W, heads, head_dim, kt, kh, kw, extra,
                 float(softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(head_dim)),
                 float(offset_scale), float(dropout_p), int(seed) & 0xFFFFFFFFFFFFFFFF)


# ------------------------------------------------------------------------------------ core op
def attn_forward(q, k, v, offsets, video_shape, heads, kernel_size, ek=None, ev=None, *,
                 softmax_scale=None, offset_scale=1.0, dropout_p=0.0, seed=0):
    """Deformable gather attention (attention.py:113-186 without the projections).

    q, k, v: [B, N, C]; offsets: raw offsets [B, N, nh*K*3] (rounded to float32);
    ek, ev: projected extra keys/values [B, G, C] or None.
    Returns (out [B, N, C] float64, lse [B, nh, N] natural log).
    """
    q, k, v = _f64(q), _f64(k), _f64(v)
    off = np.ascontiguousarray(np.asarray(offsets, dtype=np.float32))
    B, N, C = q.shape
    d = C // heads
    G = 0 if ek is None else int(np.asarray(ek).shape[1])
    ek64 = _f64(ek) if G else None
    ev64 = _f64(ev) if G else None
    g = _geom(video_shape, heads, d, kernel_size, B, G, softmax_scale, offset_scale, dropout_p, seed)
    out = np.zeros((B, N, C))
    lse = np.zeros((B, heads, N))
    _lib().oracle_dsa_fwd(ctypes.byref(g), _ptr(q), _ptr(k), _ptr(v), _ptr(off), _ptr(ek64), _ptr(ev64),
                          _ptr(out), _ptr(lse))
    return out, lse


def attn_backward(q, k, v, offsets, dout, video_shape, heads, kernel_size, ek=None, ev=None, *,
                  softmax_scale=None, offset_scale=1.0, dropout_p=0.0, seed=0):
    """Gradient of attn_forward.  Returns (dq, dk, dv, doffsets, dek, dev); doffsets is w.r.t. the
    raw offsets (offset_scale included); dek/dev are None without extra keys."""
    q, k, v, dout = _f64(q), _f64(k), _f64(v), _f64(dout)
    off = np.ascontiguousarray(np.asarray(offsets, dtype=np.float32))
    B, N, C = q.shape
    d = C // heads
    G = 0 if ek is None else int(np.asarray(ek).shape[1])
    ek64 = _f64(ek) if G else None
    ev64 = _f64(ev) if G else None
    g = _geom(video_shape, heads, d, kernel_size, B, G, softmax_scale, offset_scale, dropout_p, seed)
    dq, dk, dv = np.zeros_like(q), np.zeros_like(q), np.zeros_like(q)
    doff = np.zeros(off.shape)
    dek = np.zeros((B, G, C)) if G else None
    dev = np.zeros((B, G, C)) if G else None
    _lib().oracle_dsa_bwd(ctypes.byref(g), _ptr(q), _ptr(k), _ptr(v), _ptr(off), _ptr(ek64), _ptr(ev64),
                          _ptr(dout), _ptr(dq), _ptr(dk), _ptr(dv), _ptr(doff), _ptr(dek), _ptr(dev))
    return dq, dk, dv, doff, dek, dev


def _raw(a: np.ndarray) -> tuple:
    """(contiguous array, dtype code) for float32 or bf16 (uint16 bit patterns) element arrays."""
    a = np.ascontiguousarray(a)
    if a.dtype == np.float32:
        return a, 0
    if a.dtype == np.uint16:
        return a, 1
    raise TypeError(f"expected float32 or bf16 bits (uint16), got {a.dtype}")


def attn_rows(q_rows, offsets_rows, k, v, qidx, video_shape, heads, kernel_size, *, dout_rows=None,
              offset_bias=None, q_frame0=0, q_frames=None, kv_frame0=0, kv_frames=None, watch_rows=None,
              softmax_scale=None, offset_scale=1.0, dropout_p=0.0, seed=0):
    """The core op (forward and, with dout_rows, backward; no extra keys) at a list of query rows of
    a run too large for attn_forward / attn_backward, from the run's own operands.

    q_rows, dout_rows: [nq, C] rows of the listed queries; offsets_rows: float32 [nq, nh*K*3] (raw,
    before offset_bias); k, v: the run's K/V buffers [B * kv_frames*H*W, C]; qidx: int64 [nq] =
    b * (q_frames*H*W) + local query row.  Elements are float32 or bf16 bit patterns (uint16), the
    same type for q, k, v and dout.  Query frames [q_frame0, +q_frames) and K/V frames
    [kv_frame0, +kv_frames) are global frame windows of the volume video_shape (time sharding).
    watch_rows: int64 K/V buffer rows whose dK / dV (from the listed queries only) are returned.
    Returns dict(out, lse (natural log), dq, doff, dk, dv, misses) of float64 arrays (dq/doff/dk/dv
    None without dout_rows / watch_rows); misses = sample corners outside the K/V window."""
    T, H, W = video_shape
    q_frames = T if q_frames is None else q_frames
    kv_frames = T if kv_frames is None else kv_frames
    qr, dt = _raw(q_rows)
    kr, dtk = _raw(k)
    vr, dtv = _raw(v)
    if not (dt == dtk == dtv):
        raise TypeError("q, k, v must share one element type")
    nq, C = qr.shape
    d = C // heads
    kt, kh, kw = kernel_size
    K = kt * kh * kw
    off = np.ascontiguousarray(offsets_rows, dtype=np.float32).reshape(nq, heads * K * 3)
    bias = None if offset_bias is None else np.ascontiguousarray(offset_bias, dtype=np.float32)
    dor = None
    if dout_rows is not None:
        dor, dtd = _raw(dout_rows)
        if dtd != dt or dor.shape != qr.shape:
            raise TypeError("dout_rows must match q_rows")
    qidx = np.ascontiguousarray(qidx, dtype=np.int64)
    B = 1 + int(qidx.max()) // (q_frames * H * W) if nq else 1
    kv_rows = kr.shape[0]
    g = _geom(video_shape, heads, d, kernel_size, B, 0, softmax_scale, offset_scale, dropout_p, seed)
    out = np.zeros((nq, C))
    lse = np.zeros((nq, heads))
    dq = np.zeros((nq, C)) if dor is not None else None
    doff = np.zeros((nq, heads * K * 3)) if dor is not None else None
    slot = dk = dv = None
    nw = 0
    if watch_rows is not None and dor is not None:
        watch_rows = np.asarray(watch_rows, dtype=np.int64)
        nw = len(watch_rows)
        slot = np.full(kv_rows, -1, dtype=np.int32)
        slot[watch_rows] = np.arange(nw, dtype=np.int32)
        dk = np.zeros((nw, C))
        dv = np.zeros((nw, C))
    misses = _lib().oracle_dsa_rows(
        ctypes.byref(g), int(q_frame0), int(q_frames), int(kv_frame0), int(kv_frames), nq, _ptr(qidx), _ptr(qr),
        _ptr(dor), C, _ptr(off), _ptr(bias), _ptr(kr), _ptr(vr), kr.shape[1], dt, _ptr(out), _ptr(lse), _ptr(dq),
        _ptr(doff), _ptr(slot), nw, _ptr(dk), _ptr(dv))
    return dict(out=out, lse=lse, dq=dq, doff=doff, dk=dk, dv=dv, misses=int(misses))


def dwconv3d(x, w_kc, bias, video_shape, kernel_size):
    """Depthwise conv, zero padding k//2.  x [B, N, C], w_kc [kt*kh*kw, C]."""
    x, w_kc = _f64(x), _f64(w_kc)
    bias = None if bias is None else _f64(bias)
    B, N, C = x.shape
    T, H, W = video_shape
    y = np.zeros_like(x)
    _lib().oracle_dwconv3d(B, T, H, W, C, *kernel_size, _ptr(x), _ptr(w_kc), _ptr(bias), _ptr(y))
    return y


def dwconv3d_backward(dy, x, w_kc, video_shape, kernel_size):
    dy, x, w_kc = _f64(dy), _f64(x), _f64(w_kc)
    B, N, C = x.shape
    T, H, W = video_shape
    dx = np.zeros_like(x)
    dw = np.zeros_like(w_kc)
    db = np.zeros(C)
    _lib().oracle_dwconv3d_bwd(B, T, H, W, C, *kernel_size, _ptr(dy), _ptr(x), _ptr(w_kc), _ptr(dx), _ptr(dw),
                               _ptr(db))
    return dx, dw, db


def gelu(u):
    u = _f64(u)
    y = np.empty_like(u)
    _lib().oracle_gelu(u.size, _ptr(u), _ptr(y))
    return y


def gelu_grad(u):
    u = _f64(u)
    y = np.empty_like(u)
    _lib().oracle_gelu_grad(u.size, _ptr(u), _ptr(y))
    return y


# ------------------------------------------------------------------------------ module level
def _conv_w_kc(w):
    w = _f64(w)
    C = w.shape[0]
    return np.ascontiguousarray(w.reshape(C, -1).T)


def module_forward(params: dict, x, video_shape, extra_kv=None, *, heads: int, kernel_size=(3, 7, 7),
                   offset_scale: float = 1.0, dropout_p: float = 0.0, seed: int = 0, offsets=None):
    """Forward of DeformableSlideAttention3D (attention.py:82-192).  Returns (y, cache).
    offsets: raw offsets [B, N, nh*K*3] used in place of the offset predictor's output (the
    predictor does not run; module_backward then returns d(offsets) as grads["offsets"])."""
    x = _f64(x)
    B, N, C = x.shape
    T, H, W = video_shape
    assert N == T * H * W, f"Expected N={T * H * W} but got {N}"
    P = {kk: _f64(vv) for kk, vv in params.items()}
    dw = dwconv3d(x, _conv_w_kc(P["dw_conv.weight"]), P["dw_conv.bias"], video_shape, kernel_size)
    if offsets is None:
        u = dwconv3d(x, _conv_w_kc(P["offset_net.0.weight"]), P["offset_net.0.bias"], video_shape, (3, 3, 3))
        hact = gelu(u)
        W2 = P["offset_net.2.weight"].reshape(P["offset_net.2.weight"].shape[0], C)
        off = hact @ W2.T + P["offset_net.2.bias"]
    else:
        u = hact = None
        off = np.asarray(offsets)
    off32 = off.astype(np.float32)
    q = x @ P["q_proj.weight"].T + P["q_proj.bias"]
    k = x @ P["k_proj.weight"].T + P["k_proj.bias"]
    v = x @ P["v_proj.weight"].T + P["v_proj.bias"]
    ek = ev = e = None
    if extra_kv is not None:
        e = _f64(extra_kv)
        ek = e @ P["k_proj.weight"].T + P["k_proj.bias"]
        ev = e @ P["v_proj.weight"].T + P["v_proj.bias"]
    attn, lse = attn_forward(q, k, v, off32, video_shape, heads, kernel_size, ek, ev,
                             offset_scale=offset_scale, dropout_p=dropout_p, seed=seed)
    y = attn @ P["out_proj.weight"].T + P["out_proj.bias"] + dw
    cache = dict(x=x, u=u, hact=hact, off32=off32, q=q, k=k, v=v, ek=ek, ev=ev, e=e, attn=attn, P=P,
                 video_shape=tuple(video_shape), heads=heads, kernel_size=tuple(kernel_size),
                 offset_scale=offset_scale, dropout_p=dropout_p, seed=seed)
    return y, cache


def module_backward(cache: dict, dy):
    """Gradient of module_forward.  Returns (dx, grads by parameter name, d_extra_kv or None)."""
    dy = _f64(dy)
    P, x = cache["P"], cache["x"]
    B, N, C = x.shape
    vs, heads, ks = cache["video_shape"], cache["heads"], cache["kernel_size"]
    flat = lambda a: a.reshape(-1, a.shape[-1])  # noqa: E731
    grads = {}
    dattn = dy @ P["out_proj.weight"]
    grads["out_proj.weight"] = flat(dy).T @ flat(cache["attn"])
    grads["out_proj.bias"] = flat(dy).sum(0)
    dx_dw, dwk, dwb = dwconv3d_backward(dy, x, _conv_w_kc(P["dw_conv.weight"]), vs, ks)
    grads["dw_conv.weight"] = dwk.T.reshape(P["dw_conv.weight"].shape)
    grads["dw_conv.bias"] = dwb
    dq, dk, dv, doff, dek, dev = attn_backward(
        cache["q"], cache["k"], cache["v"], cache["off32"], dattn, vs, heads, ks, cache["ek"], cache["ev"],
        offset_scale=cache["offset_scale"], dropout_p=cache["dropout_p"], seed=cache["seed"])
    dx = dx_dw + dq @ P["q_proj.weight"] + dk @ P["k_proj.weight"] + dv @ P["v_proj.weight"]
    for name, g in (("q_proj", dq), ("k_proj", dk), ("v_proj", dv)):
        grads[f"{name}.weight"] = flat(g).T @ flat(x)
        grads[f"{name}.bias"] = flat(g).sum(0)
    d_extra = None
    if cache["e"] is not None:
        e = cache["e"]
        d_extra = dek @ P["k_proj.weight"] + dev @ P["v_proj.weight"]
        grads["k_proj.weight"] = grads["k_proj.weight"] + flat(dek).T @ flat(e)
        grads["k_proj.bias"] = grads["k_proj.bias"] + flat(dek).sum(0)
        grads["v_proj.weight"] = grads["v_proj.weight"] + flat(dev).T @ flat(e)
        grads["v_proj.bias"] = grads["v_proj.bias"] + flat(dev).sum(0)
    if cache["hact"] is None:  # offsets were given: their gradient instead of the predictor's
        grads["offsets"] = doff
        return dx, grads, d_extra
    W2 = P["offset_net.2.weight"].reshape(P["offset_net.2.weight"].shape[0], C)
    dh = doff @ W2
    grads["offset_net.2.weight"] = (flat(doff).T @ flat(cache["hact"])).reshape(P["offset_net.2.weight"].shape)
    grads["offset_net.2.bias"] = flat(doff).sum(0)
    du = dh * gelu_grad(cache["u"])
    dx_o, dwo, dbo = dwconv3d_backward(du, x, _conv_w_kc(P["offset_net.0.weight"]), vs, (3, 3, 3))
    grads["offset_net.0.weight"] = dwo.T.reshape(P["offset_net.0.weight"].shape)
    grads["offset_net.0.bias"] = dbo
    dx = dx + dx_o
    return dx, grads, d_extra


def offsets_from_cache(cache: dict) -> np.ndarray:
    """Raw offsets [B, N, nh*K*3] in the reference's 1x1-conv channel order."""
    return cache["off32"]
