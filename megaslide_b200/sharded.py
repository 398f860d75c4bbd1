"""Time-axis sharding of DeformableSlideAttention3D across ranks (one process per GPU).

Rank r owns the frames [t0_r, t1_r) of a global volume of T frames (every sample of the batch); the
coordinates of every sample use the GLOBAL T, H, W (the reference's formulas,
infinity/video/attention.py:113-127, 194-238), so a sharded run computes exactly what one process
computes on the whole volume.  Per forward:

1. the x frames one frame beyond the own range (the 3x3x3 offset conv and the kt x kh x kw dw_conv
   read kt//2 frames around each output frame) are exchanged with the neighbours;
2. the offsets of the own frames are computed and the largest temporal offset is reduced over all
   ranks (one float, MAX); from it every rank computes, for every rank, the frame range its samples
   can reach (the bound of the trilinear corners, plus one frame of margin) -- a deterministic plan
   that needs no further metadata exchange;
3. the remaining x frames of that range are exchanged and K/V are projected over the whole window;
4. the attention kernels run on the own query frames against the window (q_frame0 / kv_frame0).

The backward mirrors it: every gradient that lands on a halo frame (K/V of halo frames, the
transposed depthwise convs) is sent back to the frame's owner and added there, and the parameter
gradients (partial sums over each rank's outputs) are summed over the ranks with one all-reduce.
All exchanges are point-to-point (torch.distributed batch_isend_irecv: NCCL over NVLink for CUDA
tensors); every rank issues the same collectives in the same order.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist
from torch import Tensor, nn

from . import ops
from ._lib import MSL_EPI_GELU, MSL_EPI_GELU_GRAD, MSL_EPI_NONE, MSL_ERR_UNSUPPORTED, MslError
from .attention import DeformableSlideAttention3D, _mm_f32

Range = Tuple[int, int]


def shard_ranges(frames: int, world: int) -> List[Range]:
    """Contiguous, balanced frame ranges [t0, t1) of `frames` frames over `world` ranks."""
    if world < 1 or frames < world:
        raise ValueError(f"cannot split {frames} frames over {world} ranks (need >= 1 frame per rank)")
    base, rem = divmod(frames, world)
    out, t = [], 0
    for r in range(world):
        n = base + (1 if r < rem else 0)
        out.append((t, t + n))
        t += n
    return out


def kv_frame_range(T: int, W: int, kt: int, own: Range, max_t_offset: float) -> Range:
    """Frames [lo, hi) holding every trilinear corner the samples of query frames `own` can reach.

    The time coordinate of window row `it` of query frame t is
      g = 2 (t + it - kt//2) / max(T-1, 1) - 1 + o2 * offset_scale / (W-1)   (o2 = raw channel 2)
      p = clamp(((g + 1) T - 1) / 2, 0, T-1),  corners floor(p) and floor(p) + 1
    (the channel-2 offset moves the time axis after division by W-1: attention.py:118-127, 236).
    `max_t_offset` = max |o2 * offset_scale| over the volume.  One frame of margin on each side
    absorbs the float32 rounding of the kernels' arithmetic."""
    t0, t1 = own
    shift = (max_t_offset / (W - 1)) if W > 1 else 0.0
    den = max(T - 1, 1)

    def pix(a: int, o: float) -> float:
        g = 2.0 * a / den - 1.0 + o
        return min(T - 1.0, max(((g + 1.0) * T - 1.0) / 2.0, 0.0))

    lo = math.floor(pix(t0 - kt // 2, -shift)) - 1
    hi = math.floor(pix(t1 - 1 + kt // 2, shift)) + 1 + 1  # upper corner, margin
    return max(0, lo), min(T, hi + 1)


def conv_window(T: int, own: Range, pad: int) -> Range:
    return max(0, own[0] - pad), min(T, own[1] + pad)


def _overlap(a: Range, b: Range) -> Optional[Range]:
    lo, hi = max(a[0], b[0]), min(a[1], b[1])
    return (lo, hi) if lo < hi else None


@dataclass
class FramePlan:
    """Which frames each rank owns and which window of frames each rank holds."""

    owns: List[Range]
    windows: List[Range]


class _Pending:
    """Point-to-point transfers started on the process group's stream (NCCL: its own stream, so they
    overlap the compute queued after them); finish() makes the caller's stream wait for them and
    lands the received frames."""

    def __init__(self, reqs, on_finish):
        self.reqs = reqs
        self.on_finish = on_finish

    def finish(self):
        for req in self.reqs:
            req.wait()
        return self.on_finish()


def start_exchange(buf: Tensor, buf_range: Range, local: Tensor, plan: FramePlan, fetch: Sequence[List[Range]],
                   rank: int, group=None) -> _Pending:
    """Starts filling the frames `fetch[rank]` of `buf` (frames `buf_range`, laid out [B, frames, HW, X])
    from their owners, and sending the own frames every other rank fetches.  `local` [B, own frames, HW, X]
    holds this rank's frames (any strides).  fetch[s] = frame intervals rank s wants (the same list on
    every rank).  Returns the pending transfers; finish() lands them in `buf`.

    One message per sample: a sample's frames are contiguous in `buf` (and in `local` when its rows
    are), so they are received in place and sent without a staging copy."""
    world = len(plan.owns)
    own = plan.owns[rank]
    B = buf.shape[0]
    ops_: list = []
    recv_tmp = []
    for s in range(world):
        if s == rank:
            continue
        for iv in fetch[s]:  # frames rank s wants that this rank owns
            ov = _overlap(iv, own)
            if ov:
                for b in range(B):
                    t = local[b, ov[0] - own[0]:ov[1] - own[0]]
                    ops_.append(dist.P2POp(dist.isend, t if t.is_contiguous() else t.contiguous(), s, group))
    for iv in fetch[rank]:
        for r in range(world):
            if r == rank:
                continue
            ov = _overlap(iv, plan.owns[r])
            if ov:
                for b in range(B):
                    dst = buf[b, ov[0] - buf_range[0]:ov[1] - buf_range[0]]
                    if dst.is_contiguous():
                        ops_.append(dist.P2POp(dist.irecv, dst, r, group))
                    else:
                        t = torch.empty(dst.shape, dtype=dst.dtype, device=dst.device)
                        ops_.append(dist.P2POp(dist.irecv, t, r, group))
                        recv_tmp.append((dst, t))
    reqs = dist.batch_isend_irecv(ops_) if ops_ else []

    def land():
        for dst, t in recv_tmp:
            dst.copy_(t)

    return _Pending(reqs, land)


def exchange_into(buf: Tensor, buf_range: Range, local: Tensor, plan: FramePlan, fetch: Sequence[List[Range]],
                  rank: int, group=None) -> None:
    """start_exchange(...).finish(): fills the frames `fetch[rank]` of `buf` from their owners."""
    start_exchange(buf, buf_range, local, plan, fetch, rank, group).finish()


def start_halo_return(dwin: Tensor, plan: FramePlan, rank: int, group=None) -> _Pending:
    """Reverse of the forward exchanges, started: sends the gradient rows of `dwin` ([B, window frames,
    HW, X], frames plan.windows[rank]) that belong to other ranks to their owners and receives what the
    other ranks computed for the own frames; finish() adds those into the own frames of `dwin` (in
    place) and returns that view [B, own frames, HW, X].  One message per sample (contiguous rows: no
    staging copy, and the adds run on contiguous blocks)."""
    world = len(plan.owns)
    win, own = plan.windows[rank], plan.owns[rank]
    B = dwin.shape[0]
    ops_: list = []
    recvs = []
    for r in range(world):
        if r == rank:
            continue
        ov = _overlap(win, plan.owns[r])
        if ov:
            for b in range(B):
                src = dwin[b, ov[0] - win[0]:ov[1] - win[0]]
                ops_.append(dist.P2POp(dist.isend, src if src.is_contiguous() else src.contiguous(), r, group))
        ov = _overlap(plan.windows[r], own)
        if ov:
            for b in range(B):
                t = torch.empty((ov[1] - ov[0],) + tuple(dwin.shape[2:]), dtype=dwin.dtype, device=dwin.device)
                ops_.append(dist.P2POp(dist.irecv, t, r, group))
                recvs.append((b, ov, t))
    reqs = dist.batch_isend_irecv(ops_) if ops_ else []
    mine = dwin[:, own[0] - win[0]:own[1] - win[0]]

    def add():
        for b, ov, t in recvs:
            mine[b, ov[0] - own[0]:ov[1] - own[0]] += t
        return mine

    return _Pending(reqs, add)


def return_halo_grads(dwin: Tensor, plan: FramePlan, rank: int, group=None) -> Tensor:
    """Sends the gradient rows of `dwin` that belong to other ranks to their owners, adds what the other
    ranks send for the own frames, and returns the own frames [B, own frames, HW, X] (a new tensor;
    `dwin` is left as it was)."""
    return start_halo_return(dwin.clone(), plan, rank, group).finish()


class _GradBuckets:
    """Parameter gradients summed over the ranks in buckets: each bucket's all-reduce starts as soon as
    its gradients exist (asynchronous, on the process group's stream) and overlaps the rest of the
    backward; wait() returns every bucket's summed gradients.  All ranks add the same buckets in the
    same order."""

    def __init__(self, group):
        self.group = group
        self.items: list = []

    def add(self, parts: List[Tensor]) -> None:
        flat = torch.cat([p.reshape(-1).float() for p in parts])
        work = dist.all_reduce(flat, group=self.group, async_op=True)
        self.items.append((flat, [p.shape for p in parts], work))

    def wait(self) -> List[List[Tensor]]:
        out = []
        for flat, shapes, work in self.items:
            work.wait()
            views, o = [], 0
            for shp in shapes:
                n = math.prod(shp)
                views.append(flat[o:o + n].view(shp))
                o += n
            out.append(views)
        return out


class _ShardCfg:
    __slots__ = ("T", "H", "W", "rank", "world", "owns", "group", "heads", "head_dim", "kernel", "oscale",
                 "dropout_p", "seed", "dtype", "param_dtypes", "G", "offset_bound", "capture", "spec")


class _SpeculativeWindow:
    """The K/V window of a learned-offset step planned from the previous step's largest temporal
    offset (exact, reduced over the ranks on the device and copied to pinned memory), widened by a
    margin.  Whether the plan held is checked exactly by the attention kernels: a sample corner in a
    frame the window does not hold sets MSL_STATUS_HALO_MISS, which the next call raises.

    Every rank must plan the same windows (they fix the sizes of the halo exchange), so the plan waits
    for the previous step's reduced value instead of using whichever value happens to have arrived: the
    wait ends once the GPU has passed that step's reduction, which lies early in its forward, while the
    rest of that step (its backward included) is still queued behind it."""

    def __init__(self):
        self.known: Optional[float] = None  # the previous step's largest |temporal offset|, all ranks
        self.pending: Optional[tuple] = None  # (event, pinned value) of the last step's maximum

    def plan(self) -> Optional[float]:
        """The bound to plan with, or None when no earlier step's maximum is known yet (the same on
        every rank: each rank takes the same steps, and the value is reduced over all of them)."""
        if self.pending is not None:
            ready, value = self.pending
            ready.synchronize()
            self.known = float(value[2])
            self.pending = None
        if self.known is None or not math.isfinite(self.known):
            return None
        return self.known * 1.05 + 0.1


class DSA3DShardedFunction(torch.autograd.Function):
    """Forward/backward of one rank's frames of a time-sharded DeformableSlideAttention3D.

    Forward: the conv halo of x (max(1, kt//2) frames per side: the offset predictor's 3x3x3 conv and
    the dw_conv read them) is exchanged while q/k/v of the OWN frames are projected (one GEMM); the
    offsets and the dw_conv term follow; the K/V window of every rank comes from the largest temporal
    offset (or the caller's bound); the projected K/V rows of the halo frames are exchanged (not x:
    no projection runs twice); the attention kernels run on the own queries against the window.
    Backward: dK/dV accumulate in a float32 window buffer; its halo rows go back to their owners and
    are added there (so every GEMM is own-frame sized); the transposed convs spread into the conv
    halo, whose rows also go back; parameter gradients are summed in buckets that overlap the rest
    of the backward."""

    @staticmethod
    def forward(ctx, cfg: _ShardCfg, x, extra_kv, off_in, wq, bq, wk, bk, wv, bv, wo, bo, wd, bd, w1, b1, w2, b2):
        T, H, W, rank = cfg.T, cfg.H, cfg.W, cfg.rank
        HW = H * W
        own = cfg.owns[rank]
        nown = own[1] - own[0]
        B, N, C = x.shape
        dt = cfg.dtype
        kt, kh, kw = cfg.kernel
        nh, d, G = cfg.heads, cfg.head_dim, cfg.G
        xl = x.to(dt).reshape(B, nown, HW, C).contiguous()
        xo2 = xl.view(-1, C)
        # 1. conv halo of x, exchanged while q / k / v of the own frames are projected
        cpad = max(1, kt // 2)
        cwins = [conv_window(T, o, cpad) for o in cfg.owns]
        cw = cwins[rank]
        xc = torch.empty(B, cw[1] - cw[0], HW, C, dtype=dt, device=x.device)
        for b in range(B):  # per sample: contiguous blocks (vectorised copies)
            xc[b, own[0] - cw[0]:own[1] - cw[0]].copy_(xl[b])
        fetch1 = [[iv for iv in ((cwins[s][0], cfg.owns[s][0]), (cfg.owns[s][1], cwins[s][1])) if iv[0] < iv[1]]
                  for s in range(cfg.world)]
        pend = start_exchange(xc, cw, xl, FramePlan(cfg.owns, cwins), fetch1, rank, cfg.group)
        wqkv = torch.cat([wq, wk, wv], 0).to(dt)
        bqkv = torch.cat([bq, bk, bv], 0).to(dt)

        wq_, wkv = wqkv[:C], wqkv[C:]
        bq_, bkv = bqkv[:C], bqkv[C:]

        def kv_window(dmax_: float, kv_rows: Optional[Tensor] = None):
            """K/V window of every rank (deterministic on all ranks) for a largest temporal offset; the
            window buffer with the own K/V rows in place (projected straight into it per sample, or copied
            from `kv_rows` [own rows, 2C]); the frames every rank fetches."""
            if not math.isfinite(dmax_):
                raise FloatingPointError("non-finite offsets: the K/V halo cannot be bounded")
            kw_ = [kv_frame_range(T, W, kt, o, dmax_) for o in cfg.owns]
            kw_ = [(min(a[0], o[0]), max(a[1], o[1])) for a, o in zip(kw_, cfg.owns)]
            buf = torch.empty(B, kw_[rank][1] - kw_[rank][0], HW, 2 * C, dtype=dt, device=x.device)
            own_kv = buf[:, own[0] - kw_[rank][0]:own[1] - kw_[rank][0]]  # sent from here: contiguous per sample
            for b in range(B):
                dst = own_kv[b].view(nown * HW, 2 * C)
                if kv_rows is None:
                    torch.addmm(bkv, xl[b].view(nown * HW, C), wkv.t(), out=dst)
                else:
                    dst.copy_(kv_rows[b * nown * HW:(b + 1) * nown * HW])
            fetch = [[iv for iv in ((kw_[s_][0], cfg.owns[s_][0]), (cfg.owns[s_][1], kw_[s_][1])) if iv[0] < iv[1]]
                     for s_ in range(cfg.world)]
            return kw_, buf, own_kv, fetch

        # the K/V window is known before the offsets when the caller bounds them or when it is planned from
        # the previous step (speculative): then the projected K/V halo rows travel while the offset
        # predictor and the dw_conv term compute
        spec_plan = cfg.spec.plan() if (cfg.spec is not None and cfg.offset_bound is None) else None
        early = float(cfg.offset_bound) * abs(cfg.oscale) if cfg.offset_bound is not None else spec_plan
        kv_pend = None
        if early is not None:
            # q and the own K/V rows (into the window buffer), overlapping the conv-halo exchange
            q = torch.addmm(bq_, xo2, wq_.t())
            dmax = early
            kwins, kvw, kv_own, fetch2 = kv_window(dmax)
            kv_pend = start_exchange(kvw, kwins[rank], kv_own, FramePlan(cfg.owns, kwins), fetch2, rank, cfg.group)
        pend.finish()
        xc2 = xc.view(-1, C)
        # 2. offsets and the dw_conv term of the own frames
        conv3 = ops.ConvShape(B, T, H, W, C, (3, 3, 3), in_frame0=cw[0], in_frames=cw[1] - cw[0],
                              out_frame0=own[0], out_frames=nown)
        convk = ops.ConvShape(B, T, H, W, C, (kt, kh, kw), in_frame0=cw[0], in_frames=cw[1] - cw[0],
                              out_frame0=own[0], out_frames=nown)
        w1_kc = ops.conv_weight_kc(w1)
        b1f = b1.detach().float().contiguous()
        w2m = w2.reshape(w2.shape[0], C)
        if off_in is None:
            hact = ops.dwconv_fwd(conv3, xc2, w1_kc, b1f, epilogue=MSL_EPI_GELU)
            off = _mm_f32(hact, w2m.to(dt).t())  # its bias b2 is added by the kernels as they read it
            b2f = b2.detach().float().contiguous()
        else:  # raw offsets of the own frames given by the caller (the offset predictor does not run)
            hact = None
            off = off_in.reshape(B * nown * HW, -1)
            b2f = None
        wd_kc = ops.conv_weight_kc(wd)
        dwk = (wd_kc, bd.detach().float().contiguous(), bo.detach().float().contiguous())
        if cfg.offset_bound is not None:
            # the caller bounds |raw offset| (e.g. clipped synthetic offsets): the K/V window followed from the
            # bound alone, with no reduction and no host synchronisation
            D = ops.dwconv_fwd(convk, xc2, *dwk, epilogue=MSL_EPI_NONE)
        elif spec_plan is not None:
            # speculative window (planned from the previous step's maximum): this step's maximum is reduced
            # and read back without waiting for the next step's plan; the kernels' halo-miss bit checks the
            # plan exactly
            amax = ops.offsets_absmax(off, nh, kt * kh * kw, cfg.oscale, bias=b2f)
            dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=cfg.group)
            amax_h = torch.empty(3, dtype=torch.float32, pin_memory=True)
            amax_h.copy_(amax, non_blocking=True)
            ready = torch.cuda.Event()
            ready.record()
            cfg.spec.pending = (ready, amax_h)
            D = ops.dwconv_fwd(convk, xc2, *dwk, epilogue=MSL_EPI_NONE)
        else:
            # the largest temporal offset over all ranks sizes every rank's K/V window: it is copied to pinned
            # host memory right after its reduction, and the host waits for that copy only, while the q/k/v
            # projection and the dw_conv term (independent of the window) keep the GPU busy
            amax = ops.offsets_absmax(off, nh, kt * kh * kw, cfg.oscale, bias=b2f)
            dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=cfg.group)
            amax_h = torch.empty(3, dtype=torch.float32, pin_memory=True)
            amax_h.copy_(amax, non_blocking=True)
            ready = torch.cuda.Event()
            ready.record()
            q = torch.addmm(bq_, xo2, wq_.t())  # GPU work while the host waits
            kvo = torch.addmm(bkv, xo2, wkv.t())  # [own rows, 2C]
            D = ops.dwconv_fwd(convk, xc2, *dwk, epilogue=MSL_EPI_NONE)
            ready.synchronize()
            dmax = float(amax_h[2])
            if cfg.spec is not None:
                cfg.spec.known = dmax
            # 3. the K/V window: the own projected rows plus the halo frames' rows from their owners
            kwins, kvw, kv_own, fetch2 = kv_window(dmax, kvo)
            kv_pend = start_exchange(kvw, kwins[rank], kv_own, FramePlan(cfg.owns, kwins), fetch2, rank, cfg.group)
        kv_pend.finish()
        kwin = kwins[rank]
        nkw = kwin[1] - kwin[0]
        kplan = FramePlan(cfg.owns, kwins)
        kv = kvw.view(-1, 2 * C)
        k, v = kv[:, :C], kv[:, C:]
        ek = ev = e2 = None
        if G:
            e2 = extra_kv.reshape(B * G, C).to(dt).contiguous()
            ekv = torch.addmm(torch.cat([bk, bv], 0).to(dt), e2, wkv.t())
            ek, ev = ekv[:, :C], ekv[:, C:]
        sh = ops.DsaShape(B, T, H, W, nh, d, (kt, kh, kw), extra=G, q_frame0=own[0], q_frames=nown,
                          kv_frame0=kwin[0], kv_frames=nkw, offset_scale=cfg.oscale,
                          dropout_p=cfg.dropout_p, dropout_seed=cfg.seed)
        train = any(ctx.needs_input_grad)
        sw = ops.status_word(x.device)
        sw.poll()  # raises if an earlier call produced invalid results (e.g. a halo miss)
        probs = saved = None
        if train and ops.wants_probs(sh, dt):
            probs, saved = ops.saved_buffers(sh, dt, x.device)
            try:
                attn, lse = ops.attn_fwd(sh, q, k, v, off, ek, ev, probs=probs, saved=saved, offset_bias=b2f,
                                         status=sw.word)
            except MslError as e:
                if e.code != MSL_ERR_UNSUPPORTED:
                    raise
                probs = saved = None
        if probs is None:
            attn, lse = ops.attn_fwd(sh, q, k, v, off, ek, ev, offset_bias=b2f, status=sw.word)
        sw.post()
        y = D.addmm_(attn, wo.to(dt).t())  # in place: D is not used again
        if cfg.capture is not None:
            cfg.capture.update(xw=xc, xwin=cw, kvwin=kwin, own=own, q=q, kv=kv, hact=hact, off=off, offset_bias=b2f,
                               attn=attn, lse=lse, y=y)
        if train:
            ctx.save_for_backward(xc, xl, q, kv, hact, off, b2f, attn, lse, e2, ek, ev, wqkv, wo, w2m, w1_kc, b1f,
                                  wd_kc, probs, saved)
            ctx.cfg, ctx.sh, ctx.kplan, ctx.cplan = cfg, sh, kplan, FramePlan(cfg.owns, cwins)
            ctx.in_dtype = x.dtype
            ctx.off_dtype = off_in.dtype if off_in is not None else None
            ctx.extra_dtype = extra_kv.dtype if extra_kv is not None else None
        return y.view(B, N, C)

    @staticmethod
    def backward(ctx, dy):
        (xc, xl, q, kv, hact, off, b2f, attn, lse, e2, ek, ev, wqkv, wo, w2m, w1_kc, b1f, wd_kc, probs,
         saved) = ctx.saved_tensors
        cfg: _ShardCfg = ctx.cfg
        sh: ops.DsaShape = ctx.sh
        kplan: FramePlan = ctx.kplan
        cplan: FramePlan = ctx.cplan
        T, H, W, rank = cfg.T, cfg.H, cfg.W, cfg.rank
        HW = H * W
        own, kwin, cw = kplan.owns[rank], kplan.windows[rank], cplan.windows[rank]
        nown, nkw, ncw = own[1] - own[0], kwin[1] - kwin[0], cw[1] - cw[0]
        B = xc.shape[0]
        C = xc.shape[-1]
        dt = cfg.dtype
        kt, kh, kw = cfg.kernel
        G = cfg.G
        xc2 = xc.view(-1, C)
        xo2 = xl.view(-1, C)  # the own frames, contiguous
        with torch.autocast("cuda", enabled=False):
            dy2 = dy.reshape(-1, C).to(dt).contiguous()
            dattn = torch.mm(dy2, wo.to(dt))
            # attention core: dq on the own rows into the [own rows, 3C] gradient buffer, dK / dV accumulated
            # in float32 over the K/V window; the window's halo rows go back to their owners while the
            # out_proj and dw_conv gradients run
            dqkv = torch.empty(q.shape[0], 3 * C, dtype=q.dtype, device=q.device)
            dkv_acc = torch.zeros(B * nkw * HW, 2 * C, dtype=torch.float32, device=xc.device)
            k, v = kv[:, :C], kv[:, C:]
            sw = ops.status_word(xc.device)
            _, _, _, doff, dek, dev = ops.attn_bwd(sh, q, k, v, off, attn, lse, dattn, ek=ek, ev=ev,
                                                   dq=dqkv[:, :C], dk_acc=dkv_acc[:, :C], dv_acc=dkv_acc[:, C:],
                                                   probs=probs, saved=saved, doff_dtype=dt, offset_bias=b2f,
                                                   status=sw.word)
            sw.post()
            if cfg.capture is not None:
                cfg.capture.update(dy2=dy2, dattn=dattn, dq=dqkv[:, :C], dkv=dkv_acc.clone(), doff=doff)
            kv_ret = start_halo_return(dkv_acc.view(B, nkw, HW, 2 * C), kplan, rank, cfg.group)
            g_wo = _mm_f32(dy2.t(), attn)
            g_bo = dy2.sum(0, dtype=torch.float32)
            convk = ops.ConvShape(B, T, H, W, C, (kt, kh, kw), in_frame0=cw[0], in_frames=ncw,
                                  out_frame0=own[0], out_frames=nown)
            g_wd = torch.zeros_like(wd_kc)
            g_bd = torch.zeros(C, device=xc.device, dtype=torch.float32)
            ops.dwconv_bwd_weight(convk, dy2, xc2, g_wd, g_bd)
            # parameter gradients are summed over the ranks bucket by bucket, overlapping the backward
            buckets = _GradBuckets(cfg.group)
            buckets.add([g_wo, g_bo, g_wd, g_bd])
            # transposed convs: the dw_conv term and the offset predictor spread into the conv halo
            dxc = torch.zeros(B * ncw * HW, C, dtype=torch.float32, device=xc.device)
            convk_t = ops.ConvShape(B, T, H, W, C, (kt, kh, kw), in_frame0=own[0], in_frames=nown,
                                    out_frame0=cw[0], out_frames=ncw, zero_outside=True)
            ops.dwconv_bwd_data(convk_t, dy2, wd_kc, out=dxc, accumulate=True)
            predictor = hact is not None
            d_off_in = None
            if predictor:
                dh = _mm_f32(doff, w2m.to(dt))
                g_w2 = _mm_f32(doff.t(), hact)
                g_b2 = doff.sum(0, dtype=torch.float32)
                conv3 = ops.ConvShape(B, T, H, W, C, (3, 3, 3), in_frame0=cw[0], in_frames=ncw, out_frame0=own[0],
                                      out_frames=nown)
                du = ops.dwconv_fwd(conv3, xc2, w1_kc, b1f, epilogue=MSL_EPI_GELU_GRAD, aux=dh,
                                    out_dtype=torch.float32)
                conv3_t = ops.ConvShape(B, T, H, W, C, (3, 3, 3), in_frame0=own[0], in_frames=nown, out_frame0=cw[0],
                                        out_frames=ncw, zero_outside=True)
                ops.dwconv_bwd_data(conv3_t, du, w1_kc, out=dxc, accumulate=True)
                g_w1 = torch.zeros_like(w1_kc)
                g_b1 = torch.zeros(C, device=xc.device, dtype=torch.float32)
                ops.dwconv_bwd_weight(conv3, du, xc2, g_w1, g_b1)
                buckets.add([g_w1, g_b1, g_w2, g_b2])
            elif ctx.needs_input_grad[3]:
                d_off_in = doff.view(B, nown * HW, -1).to(ctx.off_dtype)
            conv_ret = start_halo_return(dxc.view(B, ncw, HW, C), cplan, rank, cfg.group)
            # the own K/V rows, with every rank's contributions, in the compute dtype next to dq
            dkv_own = kv_ret.finish()  # [B, nown, HW, 2C] float32 view of the window accumulator
            rows_s = nown * HW
            for b in range(B):
                ops.convert_f32(dkv_own[b].reshape(rows_s, 2 * C), dqkv[b * rows_s:(b + 1) * rows_s, C:])
            d_extra = None
            g_ekv = sums = None
            if G:
                dekv = torch.cat([dek, dev], 1)
                d_extra = torch.mm(dekv, wqkv[C:].float()).view(B, G, C)
                g_ekv = torch.mm(dekv.t(), e2.float())
                sums = dekv.sum(0)
            g_wqkv = _mm_f32(dqkv.t(), xo2)
            g_bqkv = dqkv.sum(0, dtype=torch.float32)
            if G:
                g_wqkv[C:] += g_ekv
                g_bqkv[C:] += sums
            buckets.add([g_wqkv, g_bqkv] + ([d_extra] if d_extra is not None else []))
            dx = _mm_f32(dqkv, wqkv)  # [own rows, C] float32
            dx_conv = conv_ret.finish()  # [B, nown, HW, C] float32
            dx = dx.view(B, nown, HW, C)
            for b in range(B):  # per sample: contiguous blocks (vectorised adds)
                dx[b].add_(dx_conv[b])
            summed = buckets.wait()
        g_wo, g_bo, g_wd, g_bd = summed[0]
        i = 1
        if predictor:
            g_w1, g_b1, g_w2, g_b2 = summed[1]
            i = 2
        g_wqkv, g_bqkv = summed[i][:2]
        d_extra = summed[i][2] if G else None
        g_wq, g_wk, g_wv = g_wqkv[:C], g_wqkv[C:2 * C], g_wqkv[2 * C:]
        g_bq, g_bk, g_bv = g_bqkv[:C], g_bqkv[C:2 * C], g_bqkv[2 * C:]
        pd = cfg.param_dtypes

        def conv_w(gkc, k3):
            return gkc.t().reshape(C, 1, *k3)

        grads = (
            g_wq.to(pd[0]), g_bq.to(pd[1]), g_wk.to(pd[2]), g_bk.to(pd[3]), g_wv.to(pd[4]), g_bv.to(pd[5]),
            g_wo.to(pd[6]), g_bo.to(pd[7]), conv_w(g_wd, (kt, kh, kw)).to(pd[8]), g_bd.to(pd[9]),
        )
        if predictor:
            grads += (conv_w(g_w1, (3, 3, 3)).to(pd[10]), g_b1.to(pd[11]),
                      g_w2.reshape(w2m.shape[0], C, 1, 1, 1).to(pd[12]), g_b2.to(pd[13]))
        else:
            grads += (None, None, None, None)
        dx_out = dx.reshape(B, nown * HW, C).to(ctx.in_dtype)
        de = d_extra.to(ctx.extra_dtype) if d_extra is not None else None
        return (None, dx_out, de, d_off_in) + grads


class TimeShardedDSA3D(nn.Module):
    """Runs a DeformableSlideAttention3D (whose parameters it shares) on this rank's frames of a
    volume sharded along time.

    forward(x_local [B, own_frames*H*W, D], video_shape = GLOBAL (T, H, W), extra_kv=None) returns
    the module output for the own frames; gradients w.r.t. x_local and the (replicated) parameters
    equal those of the unsharded module (parameter gradients are summed over the ranks inside the
    backward, so every rank ends with the full gradient).  Frame ranges: `shard_ranges(T, world)`
    unless `frame_ranges` is given (the same list on every rank).

    forward_with_offsets(x_local, video_shape, offsets_local, offset_bound=None) runs the op on given
    raw offsets of the own frames (float32 [B, own_frames*H*W, nh*K*3]; the offset predictor does not
    run).  With `offset_bound` (a bound on |raw offset| that the caller guarantees, e.g. for offsets
    clipped to +-3) the K/V window of every rank follows from the bound: no reduction of the largest
    offset and no host synchronisation.  ``capture``: as DeformableSlideAttention3D.capture.

    speculative_window=True (learned offsets): from the second step on, the K/V window is planned from
    the previous step's largest temporal offset (times 1.05, plus 0.1) instead of waiting for this
    step's; this step's maximum is still reduced on the device and read back for the next plan.  The
    plan is checked exactly: a sample corner outside the window sets MSL_STATUS_HALO_MISS, and the
    next call (or megaslide_b200.check_status()) raises MslError - a step whose offsets jumped past the
    margin is reported, never silently wrong."""

    def __init__(self, module: DeformableSlideAttention3D, group=None,
                 frame_ranges: Optional[Sequence[Range]] = None, speculative_window: bool = False):
        super().__init__()
        self.module = module
        self.group = group
        self.frame_ranges = list(frame_ranges) if frame_ranges is not None else None
        self._joined = False
        self.capture: Optional[dict] = None
        # learned offsets: plan the K/V window from the previous step's largest offset (no host wait;
        # the kernels' halo-miss bit verifies the plan and the next call raises if it did not hold)
        self._spec = _SpeculativeWindow() if speculative_window else None

    def forward(self, x: Tensor, video_shape: Tuple[int, int, int], extra_kv: Optional[Tensor] = None) -> Tensor:
        return self._run(x, video_shape, extra_kv, None, None)

    def forward_with_offsets(self, x: Tensor, video_shape: Tuple[int, int, int], offsets: Tensor,
                             offset_bound: Optional[float] = None, extra_kv: Optional[Tensor] = None) -> Tensor:
        m = self.module
        if offsets.dtype != torch.float32:
            raise TypeError("offsets must be float32")
        want = tuple(x.shape[:2]) + (m.num_heads * m.k_t * m.k_h * m.k_w * 3,)
        if tuple(offsets.shape) != want:
            raise ValueError(f"offsets must have shape {want}, got {tuple(offsets.shape)}")
        if offset_bound is not None and not (offset_bound >= 0 and math.isfinite(offset_bound)):
            raise ValueError("offset_bound must be a finite non-negative number")
        return self._run(x, video_shape, extra_kv, offsets.contiguous(), offset_bound)

    def _run(self, x: Tensor, video_shape: Tuple[int, int, int], extra_kv: Optional[Tensor],
             offsets: Optional[Tensor], offset_bound: Optional[float]) -> Tensor:
        m = self.module
        T, H, W = video_shape
        world = dist.get_world_size(self.group)
        rank = dist.get_rank(self.group)
        owns = self.frame_ranges or shard_ranges(T, world)
        if len(owns) != world:
            raise ValueError("frame_ranges must have one range per rank")
        own = owns[rank]
        B, N, D = x.shape
        if N != (own[1] - own[0]) * H * W:
            raise ValueError(f"x holds {N} tokens but the own frames {own} of {H}x{W} need {(own[1] - own[0]) * H * W}")
        if D != m.hidden_size:
            raise ValueError(f"hidden size {D} != {m.hidden_size}")
        if not x.is_cuda:
            raise RuntimeError("TimeShardedDSA3D runs on CUDA tensors only (no CPU fallback)")
        dt = x.dtype
        if torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16:
            dt = torch.bfloat16
        if dt not in (torch.float32, torch.bfloat16):
            raise TypeError(f"megaslide_b200 supports float32 and bfloat16, got {dt}")
        if not self._joined:  # the first NCCL call of the group must involve every rank
            dist.all_reduce(torch.zeros(1, device=x.device), group=self.group)
            self._joined = True
        G = extra_kv.shape[1] if extra_kv is not None else 0
        p = m.dropout.p if m.training else 0.0
        seed = 0
        if p > 0:  # one seed for all ranks: the keep rule is keyed by the global softmax index
            s = torch.randint(0, 2 ** 62, (1,), device=x.device)
            dist.broadcast(s, src=dist.get_global_rank(self.group, 0) if self.group is not None else 0,
                           group=self.group)
            seed = int(s.item())
        cfg = _ShardCfg()
        cfg.T, cfg.H, cfg.W, cfg.rank, cfg.world, cfg.owns, cfg.group = T, H, W, rank, world, owns, self.group
        cfg.heads, cfg.head_dim, cfg.kernel = m.num_heads, m.head_dim, (m.k_t, m.k_h, m.k_w)
        cfg.oscale, cfg.dropout_p, cfg.seed, cfg.dtype = float(m.offset_scale), float(p), seed, dt
        cfg.param_dtypes = tuple(t.dtype for t in m._params())
        cfg.G = G
        cfg.offset_bound = offset_bound
        cfg.capture = self.capture
        cfg.spec = self._spec
        with torch.autocast("cuda", enabled=False):
            return DSA3DShardedFunction.apply(cfg, x, extra_kv, offsets, *m._params())
