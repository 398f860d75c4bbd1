"""Sampled-row parity of a full-size run against the CPU oracle — TEST INFRASTRUCTURE ONLY.

``bench.py`` calls this AFTER its timed region (and tests may call it) to check the run it timed:
the module / time-sharded module is given a ``capture`` dict for one extra forward + backward, and
the captured device tensors are compared, at sampled rows, with the oracle's restatement of the
reference (``infinity/video/attention.py:113-192``):

* attention core at ``n_rows`` random query rows: output, log-sum-exp, dQ and d(offsets)
  (``dsa_oracle.attn_rows``: the per-query arithmetic of ``oracle_dsa_fwd`` / ``oracle_dsa_bwd``);
* dK / dV at a watched block of 2 x 4 key rows, accumulated by the oracle over every query of the run
  that can reach the block (a box around it sized from the run's largest offsets);
* global identities of the backward: per channel, sum over rows of dV = sum over queries of d(out)
  (softmax weights and trilinear weights each sum to 1) and sum of dK = 0 (sum_s dS_s = 0);
* module output y = attn . Wo^T + bo + dw_conv(x) + bd at the sampled rows (attention.py:185-192);
* single GPU: dx at a few rows, through the q/k/v projections, the transposed dw_conv and the
  offset predictor's transposed 3x3x3 conv of GELU'(u) * (d(offsets) . W2) (attention.py:70-74,
  102-106, 130-132);
* offset predictor's 1x1 conv weight / bias gradients through random projections
  u^T dW2 v = sum_rows (doff u)(hact v) (summed over ranks when sharded).

Each entry reports its error and its tolerance (bf16: 2e-2 on outputs and relative Frobenius
norms, 5e-2 on gradient max-abs; float32: 1e-4), and ``ok``.
"""

from __future__ import annotations

import math
from typing import Optional

import numpy as np
import torch

from . import dsa_oracle as O

LOG2E = 1.4426950408889634


def _host(t: torch.Tensor) -> np.ndarray:
    """Device tensor -> numpy: float32 as float32, bf16 as uint16 bit patterns (what attn_rows reads)."""
    t = t.detach()
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    return t.float().contiguous().cpu().numpy()


def _f64(t: torch.Tensor) -> np.ndarray:
    return t.detach().double().cpu().numpy()


def _rel_max(a, ref) -> float:
    s = float(np.abs(ref).max()) if ref.size else 0.0
    return float(np.abs(a - ref).max()) / s if s > 0 else float(np.abs(a - ref).max() if a.size else 0.0)


def _rel_fro(a, ref) -> float:
    s = float(np.linalg.norm(ref))
    return float(np.linalg.norm(a - ref)) / s if s > 0 else float(np.linalg.norm(a - ref))


def _tols(dtype: torch.dtype):
    if dtype == torch.bfloat16:
        return dict(out=2e-2, fro=2e-2, grad_max=5e-2, lse=1e-2)
    return dict(out=1e-4, fro=1e-4, grad_max=1e-4, lse=1e-5)


def _entry(err: float, tol: float) -> dict:
    return {"err": err, "tol": tol, "ok": bool(err <= tol)}


def _frame_range(lo_base: int, hi_base: int, S: int, shift: float, margin: int = 2):
    """Frames / rows / columns whose samples can reach [lo_base, hi_base] (window half-size and offset
    stretch folded into `shift`), clamped to the volume."""
    return max(0, int(math.floor(lo_base - shift)) - margin), min(S - 1, int(math.ceil(hi_base + shift)) + margin)


def _conv_rows(xbuf: torch.Tensor, frame0: int, nframes: int, b: np.ndarray, t: np.ndarray, h: np.ndarray,
               w: np.ndarray, H: int, W: int, T: int, w_kc: np.ndarray, ks, transposed: bool = False) -> np.ndarray:
    """Depthwise conv (zero padding at the GLOBAL volume border) of the device buffer `xbuf`
    [B*nframes*H*W, C] (frames [frame0, frame0+nframes)) at positions (b, t, h, w), in float64 on the
    host; transposed: the adjoint (taps mirrored).  Only the rows the taps read leave the device."""
    kt, kh, kw = ks
    C = xbuf.shape[1]
    out = np.zeros((len(b), C))
    tap = 0
    sgn = -1 if transposed else 1
    for it in range(kt):
        for ih in range(kh):
            for iw in range(kw):
                tt, hh, ww = t + sgn * (it - kt // 2), h + sgn * (ih - kh // 2), w + sgn * (iw - kw // 2)
                ok = (tt >= 0) & (tt < T) & (hh >= 0) & (hh < H) & (ww >= 0) & (ww < W)
                if np.any(ok & ((tt < frame0) | (tt >= frame0 + nframes))):
                    raise ValueError("conv tap outside the buffer's frames")
                rows = np.where(ok, ((b * nframes + (tt - frame0)) * H + hh) * W + ww, 0)
                xr = xbuf.detach().index_select(0, torch.from_numpy(rows).to(xbuf.device)).double().cpu().numpy()
                out += np.where(ok[:, None], xr * w_kc[tap], 0.0)
                tap += 1
    return out


def _erf(x: np.ndarray) -> np.ndarray:
    try:
        from scipy.special import erf
    except ImportError:  # pragma: no cover
        return np.vectorize(math.erf)(x)
    return erf(x)


def _bf16_to_f64(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def _as_f64(a: np.ndarray) -> np.ndarray:
    return _bf16_to_f64(a) if a.dtype == np.uint16 else a.astype(np.float64)


def check(module, cap: dict, video_shape, *, batch: int, dtype: torch.dtype, n_rows: int = 2048, n_dx: int = 32,
          seed: int = 0, q_frame0: int = 0, q_frames: Optional[int] = None, kv_frame0: int = 0,
          kv_frames: Optional[int] = None, injected: bool = False, group=None, world: int = 1) -> dict:
    """Compares one captured forward + backward (module.capture / TimeShardedDSA3D.capture) with the
    oracle at sampled rows.  Unsharded captures hold x2/qkv/dqkv; sharded ones xw/q/kv/dq/dkv plus the
    rank's frame windows (pass q_frame0/q_frames/kv_frame0/kv_frames).  Returns a dict of entries
    {err, tol, ok} plus ``ok`` (all entries) and ``n_rows``."""
    T, H, W = video_shape
    HW = H * W
    nh, d = module.num_heads, module.head_dim
    C = nh * d
    ks = (module.k_t, module.k_h, module.k_w)
    K = ks[0] * ks[1] * ks[2]
    q_frames = T if q_frames is None else q_frames
    kv_frames = T if kv_frames is None else kv_frames
    B = batch
    tol = _tols(dtype)
    rng = np.random.default_rng(seed)
    sharded = "kv" in cap
    cap = {k: (v.detach() if isinstance(v, torch.Tensor) else v) for k, v in cap.items()}
    if sharded:
        qb, kb, vb = cap["q"], cap["kv"][:, :C], cap["kv"][:, C:]
        dqb, dkb, dvb = cap["dq"], cap["dkv"][:, :C], cap["dkv"][:, C:]
        xr = cap.get("xwin", cap.get("win"))  # frames of the captured x buffer
        xbuf_t, xf0, xnf = cap["xw"].reshape(-1, C), xr[0], xr[1] - xr[0]
    else:
        qb, kb, vb = cap["qkv"][:, :C], cap["qkv"][:, C:2 * C], cap["qkv"][:, 2 * C:]
        dqb, dkb, dvb = cap["dqkv"][:, :C], cap["dqkv"][:, C:2 * C], cap["dqkv"][:, 2 * C:]
        xbuf_t, xf0, xnf = cap["x2"], 0, T
    off, bias = cap["off"], cap["offset_bias"]
    nq_rows, nkv_rows = B * q_frames * HW, B * kv_frames * HW
    res: dict = {}
    dev = qb.device

    # ---- attention core at sampled query rows
    n_rows = min(n_rows, nq_rows)
    qidx = np.sort(rng.choice(nq_rows, n_rows, replace=False))
    it = torch.from_numpy(qidx).to(dev)
    kh_, vh_ = _host(kb), _host(vb)
    pick = lambda t: _host(t.index_select(0, it))  # noqa: E731
    bias_h = None if bias is None else bias.detach().float().cpu().numpy()
    oscale = float(module.offset_scale)
    r = O.attn_rows(pick(qb), off.index_select(0, it).float().cpu().numpy(), kh_, vh_, qidx, video_shape, nh, ks,
                    dout_rows=pick(cap["dattn"]), offset_bias=bias_h, q_frame0=q_frame0, q_frames=q_frames,
                    kv_frame0=kv_frame0, kv_frames=kv_frames, offset_scale=oscale)
    res["halo_misses"] = {"err": float(r["misses"]), "tol": 0.0, "ok": r["misses"] == 0}
    res["out_max_rel"] = _entry(_rel_max(_as_f64(pick(cap["attn"])), r["out"]), tol["out"])
    lse = cap["lse"].reshape(B, nh, q_frames * HW)
    bq_, nq_ = torch.from_numpy(qidx // (q_frames * HW)).to(dev), torch.from_numpy(qidx % (q_frames * HW)).to(dev)
    lse_g = lse[bq_, :, nq_].double().cpu().numpy() / LOG2E  # base-2 units -> natural log
    res["lse_max_abs"] = _entry(float(np.abs(lse_g - r["lse"]).max()), tol["lse"])
    dq_g = _as_f64(pick(dqb))
    res["dq_fro"] = _entry(_rel_fro(dq_g, r["dq"]), tol["fro"])
    res["dq_max_rel"] = _entry(_rel_max(dq_g, r["dq"]), tol["grad_max"])
    doff_g = cap["doff"].index_select(0, it).double().cpu().numpy()
    res["doff_fro"] = _entry(_rel_fro(doff_g, r["doff"]), tol["fro"])
    res["doff_max_rel"] = _entry(_rel_max(doff_g, r["doff"]), tol["grad_max"])

    # ---- dK / dV at a watched 2 x 4 block of key rows, from every query of this run that can reach it
    amax_t = torch.zeros(3, device=dev, dtype=torch.float32)
    for r0 in range(0, off.shape[0], 16384):  # per axis max |raw offset + bias|, in row chunks
        blk = off[r0:r0 + 16384].float().reshape(-1, off.shape[1] // 3, 3)
        if bias is not None:
            blk = blk + bias.float().reshape(-1, 3)
        amax_t = torch.maximum(amax_t, blk.abs().amax(dim=(0, 1)))
    amax = [float(a) * abs(oscale) for a in amax_t.cpu()]
    st = (ks[0] // 2) * T / max(T - 1, 1) + (amax[2] * T / (2 * (W - 1)) if W > 1 else 0) + 1
    sh = (ks[1] // 2) * H / max(H - 1, 1) + (amax[1] * H / (2 * (H - 1)) if H > 1 else 0) + 1
    sw = (ks[2] // 2) * W / max(W - 1, 1) + (amax[0] * W / (2 * (T - 1)) if T > 1 else 0) + 1
    bw = int(rng.integers(0, B))
    tk = int(rng.integers(kv_frame0, kv_frame0 + kv_frames))
    hk = int(rng.integers(0, max(1, H - 1)))
    wk = int(rng.integers(0, max(1, W - 3)))
    hs, ws = list(range(hk, min(H, hk + 2))), list(range(wk, min(W, wk + 4)))
    watch = np.array([((bw * kv_frames + tk - kv_frame0) * H + y) * W + x for y in hs for x in ws], dtype=np.int64)
    t_lo, t_hi = _frame_range(tk, tk, T, st)
    h_lo, h_hi = _frame_range(hs[0], hs[-1], H, sh)
    w_lo, w_hi = _frame_range(ws[0], ws[-1], W, sw)
    t_lo, t_hi = max(t_lo, q_frame0), min(t_hi, q_frame0 + q_frames - 1)
    contrib = np.array([bw * q_frames * HW + ((t - q_frame0) * H + y) * W + x for t in range(t_lo, t_hi + 1)
                        for y in range(h_lo, h_hi + 1) for x in range(w_lo, w_hi + 1)], dtype=np.int64)
    if len(contrib):
        ic = torch.from_numpy(contrib).to(dev)
        pc = lambda t: _host(t.index_select(0, ic))  # noqa: E731
        rc = O.attn_rows(pc(qb), off.index_select(0, ic).float().cpu().numpy(), kh_, vh_, contrib, video_shape, nh,
                         ks, dout_rows=pc(cap["dattn"]), offset_bias=bias_h, q_frame0=q_frame0, q_frames=q_frames,
                         kv_frame0=kv_frame0, kv_frames=kv_frames, watch_rows=watch, offset_scale=oscale)
        iw_ = torch.from_numpy(watch).to(dev)
        dk_g = _as_f64(_host(dkb.index_select(0, iw_)))
        dv_g = _as_f64(_host(dvb.index_select(0, iw_)))
        res["dk_block_fro"] = _entry(_rel_fro(dk_g, rc["dk"]), tol["fro"])
        res["dv_block_fro"] = _entry(_rel_fro(dv_g, rc["dv"]), tol["fro"])
        res["dk_block_queries"] = {"err": float(len(contrib)), "tol": None, "ok": True}

    # ---- identities over the whole run: sum dV = sum d(out) per channel, sum dK = 0
    if module.dropout.p == 0 or not module.training:
        sdv = dvb.float().sum(0).double()
        sdo = cap["dattn"].float().sum(0).double()
        sdk = dkb.float().sum(0).double()
        res["sum_dv_eq_sum_dout"] = _entry(float((sdv - sdo).norm() / sdo.norm().clamp_min(1e-30)), tol["fro"])
        res["sum_dk_zero"] = _entry(float(sdk.norm() / dkb.float().abs().sum(0).double().norm().clamp_min(1e-30)),
                                    tol["fro"])

    # ---- module output at the sampled rows: y = attn Wo^T + bo + dw_conv(x) + bd
    b_, n_ = qidx // (q_frames * HW), qidx % (q_frames * HW)
    t_, h_, w_ = q_frame0 + n_ // HW, (n_ // W) % H, n_ % W
    wd = module.dw_conv.weight.detach().double().reshape(C, -1).t().cpu().numpy()
    dwx = _conv_rows(xbuf_t, xf0, xnf, b_, t_, h_, w_, H, W, T, wd, ks)
    wo = module.out_proj.weight.detach().double().cpu().numpy()
    y_ref = (_as_f64(pick(cap["attn"])) @ wo.T + module.out_proj.bias.detach().double().cpu().numpy() + dwx
             + module.dw_conv.bias.detach().double().cpu().numpy())
    res["y_max_rel"] = _entry(_rel_max(_as_f64(pick(cap["y"])), y_ref), tol["out"])

    # ---- dx at a few rows (single GPU): projections + transposed dw_conv + offset predictor branch
    if not sharded and "dx" in cap:
        sel = qidx[:n_dx]
        b_, n_ = sel // (T * HW), sel % (T * HW)
        t_, h_, w_ = n_ // HW, (n_ // W) % H, n_ % W
        isel = torch.from_numpy(sel).to(dev)
        wq = torch.cat([module.q_proj.weight, module.k_proj.weight, module.v_proj.weight], 0).detach().double().cpu().numpy()
        dx_ref = _as_f64(_host(cap["dqkv"].index_select(0, isel))) @ wq
        dx_ref += _conv_rows(cap["dy2"], 0, T, b_, t_, h_, w_, H, W, T, wd, ks, transposed=True)
        if cap.get("hact") is not None:
            # du at the 27 positions whose 3x3x3 taps reach each row, then the transposed conv
            w1 = module.offset_net[0].weight.detach().double().reshape(C, -1).t().cpu().numpy()
            b1 = module.offset_net[0].bias.detach().double().cpu().numpy()
            w2 = module.offset_net[2].weight.detach().double().reshape(-1, C).cpu().numpy()
            acc = np.zeros((len(sel), C))
            tap = 0
            for it in range(3):
                for ih in range(3):
                    for iw in range(3):
                        to, ho, wo_ = t_ - (it - 1), h_ - (ih - 1), w_ - (iw - 1)
                        ok = (to >= 0) & (to < T) & (ho >= 0) & (ho < H) & (wo_ >= 0) & (wo_ < W)
                        rows = np.where(ok, ((b_ * T + to) * H + ho) * W + wo_, 0)
                        u = _conv_rows(xbuf_t, 0, T, b_, np.where(ok, to, 0), np.where(ok, ho, 0),
                                       np.where(ok, wo_, 0), H, W, T, w1, (3, 3, 3)) + b1
                        cdf = 0.5 * (1.0 + _erf(u / math.sqrt(2.0)))
                        gp = cdf + u * np.exp(-0.5 * u * u) / math.sqrt(2 * math.pi)
                        dh = cap["doff"].index_select(0, torch.from_numpy(rows).to(dev)).double().cpu().numpy() @ w2
                        acc += np.where(ok[:, None], dh * gp * w1[tap], 0.0)
                        tap += 1
            dx_ref += acc
        dx_g = cap["dx"].index_select(0, isel).double().cpu().numpy()
        res["dx_fro"] = _entry(_rel_fro(dx_g, dx_ref), tol["fro"])

    # ---- offset predictor 1x1 conv weight / bias gradients through random projections
    if not injected and cap.get("hact") is not None and module.offset_net[2].weight.grad is not None:
        g = torch.Generator(device=dev).manual_seed(20261)  # the same projections on every rank
        Oc = off.shape[1]
        u = torch.randn(8, Oc, device=dev, generator=g, dtype=torch.float64)
        v = torch.randn(8, C, device=dev, generator=g, dtype=torch.float64)
        doff64, hact64 = cap["doff"].double(), cap["hact"].double()
        rhs = ((doff64 @ u.t()) * (hact64 @ v.t())).sum(0)
        bsum = doff64.sum(0)
        if world > 1:
            torch.distributed.all_reduce(rhs, group=group)
            torch.distributed.all_reduce(bsum, group=group)
        gw = module.offset_net[2].weight.grad.double().reshape(Oc, C)
        lhs = ((u @ gw) * v).sum(1)
        res["doffset_w_proj"] = _entry(float((lhs - rhs).norm() / rhs.norm().clamp_min(1e-30)), tol["fro"])
        gb = module.offset_net[2].bias.grad.double()
        res["doffset_b_fro"] = _entry(float((gb - bsum).norm() / bsum.norm().clamp_min(1e-30)), tol["fro"])

    res["ok"] = all(v["ok"] for v in res.values() if isinstance(v, dict))
    res["n_rows"] = int(n_rows)
    return res
