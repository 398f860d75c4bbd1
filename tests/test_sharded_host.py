"""Host logic of the time-sharded path (megaslide_b200/sharded.py), on CPU: the frame plan, the K/V
halo bound (against a brute-force float32 evaluation of the reference's coordinate formulas), the
two exchange steps run as 2 and 4 gloo ranks on CPU tensors, the speculative window plan and the
parameter-gradient buckets (3 gloo ranks)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from megaslide_b200.sharded import (FramePlan, _GradBuckets, _SpeculativeWindow, conv_window, exchange_into,
                                    kv_frame_range, return_halo_grads, shard_ranges)


def test_shard_ranges_cover_the_volume():
    for T, world in [(64, 1), (64, 8), (65, 8), (7, 3), (256, 8)]:
        r = shard_ranges(T, world)
        assert r[0][0] == 0 and r[-1][1] == T
        assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
        sizes = [b - a for a, b in r]
        assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_ranges(3, 4)


def _corner_frames_f32(T, W, kt, t, it, o2):
    """Frames of the two trilinear corners of window row `it` of query frame t (float32, in the
    kernels' operation order: attention.py:113-127, 209-236, 262-268)."""
    f = np.float32
    den = f(max(T - 1, 1))
    g = f(f(2 * (t + it - kt // 2)) / den) - f(1.0)
    if W > 1:
        g = f(g + f(f(o2) / f(W - 1)))
    p = f(f(f(f(g + f(1.0)) * f(T)) - f(1.0)) * f(0.5))
    p = min(f(T - 1), max(p, f(0.0)))
    t0 = int(np.floor(p))
    return [c for c in (t0, t0 + 1) if c < T]


@pytest.mark.parametrize("T,W,kt,world,delta", [(64, 32, 3, 8, 2.5), (256, 64, 3, 8, 3.0), (16, 16, 5, 4, 9.0),
                                                (9, 2, 3, 3, 0.7), (4, 1, 3, 2, 5.0), (1, 8, 1, 1, 1.0)])
def test_kv_frame_range_holds_every_corner(T, W, kt, world, delta):
    rng = np.random.default_rng(0)
    for own in shard_ranges(T, world):
        lo, hi = kv_frame_range(T, W, kt, own, delta)
        assert 0 <= lo < hi <= T
        offs = np.concatenate([[-delta, delta, 0.0], rng.uniform(-delta, delta, 64)]).astype(np.float32)
        for t in range(*own):
            for it in range(kt):
                for o in offs:
                    for c in _corner_frames_f32(T, W, kt, t, it, o):
                        assert lo <= c < hi, (own, t, it, o, c, lo, hi)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, T, HW, C, q, strided_local=False):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B = 2
        g = torch.arange(B * T * HW * C, dtype=torch.float32).view(B, T, HW, C)  # the global volume
        owns = shard_ranges(T, world)
        own = owns[rank]
        local = g[:, own[0]:own[1]].contiguous()
        if strided_local:  # the own rows as a column slice of a wider buffer (like q/k/v views of one GEMM)
            local = torch.cat([torch.zeros_like(local), local], dim=-1)[..., C:]
        # forward: windows of different sizes per rank, fetched in two phases as the module does
        cw = [conv_window(T, o, 1) for o in owns]
        wins = [conv_window(T, o, 3 if r % 2 == 0 else 2) for r, o in enumerate(owns)]
        win = wins[rank]
        buf = torch.full((B, win[1] - win[0], HW, C), -1.0)
        buf[:, own[0] - win[0]:own[1] - win[0]] = local
        fetch1 = [[iv for iv in ((cw[s][0], owns[s][0]), (owns[s][1], cw[s][1])) if iv[0] < iv[1]] for s in range(world)]
        fetch2 = [[iv for iv in ((wins[s][0], cw[s][0]), (cw[s][1], wins[s][1])) if iv[0] < iv[1]] for s in range(world)]
        plan = FramePlan(owns, wins)
        exchange_into(buf, win, local, plan, fetch1, rank)
        exchange_into(buf, win, local, plan, fetch2, rank)
        ok_fwd = bool(torch.equal(buf, g[:, win[0]:win[1]]))
        # backward: every rank holds a gradient over its window; the owner must end with the sum
        dwin = torch.ones(B, win[1] - win[0], HW, C) * (rank + 1)
        mine = return_halo_grads(dwin, plan, rank)
        want = torch.zeros(B, own[1] - own[0], HW, C)
        for r, w in enumerate(wins):
            lo, hi = max(w[0], own[0]), min(w[1], own[1])
            if lo < hi:
                want[:, lo - own[0]:hi - own[0]] += r + 1
        ok_bwd = bool(torch.equal(mine, want))
        q.put((rank, ok_fwd, ok_bwd))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,T,strided", [(2, 8, False), (2, 5, True), (4, 12, False), (4, 9, True)])
def test_frame_exchange_gloo_ranks(world, T, strided):
    """Forward window fill and backward halo return on 2 and 4 CPU ranks (4: interior ranks with two
    neighbours; T=9: windows that reach past a neighbour's 2-frame shard), B = 2, contiguous and
    column-strided own rows."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, T, 3, 2, q, strided)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok_fwd, ok_bwd in res:
        assert ok_fwd, f"rank {rank}: forward window differs from the global volume"
        assert ok_bwd, f"rank {rank}: returned halo gradients do not sum up"


class _SlowEvent:
    """An event whose query() says 'not yet' until synchronize() is called (a GPU running behind)."""

    def __init__(self):
        self.done = False

    def query(self):
        return self.done

    def synchronize(self):
        self.done = True


def test_speculative_plan_uses_the_previous_steps_value_on_every_rank():
    """The window plan must not depend on how far a rank's GPU has got: each plan waits for the
    previous step's reduced maximum, so ranks that run at different speeds plan the same window."""
    spec = _SpeculativeWindow()
    assert spec.plan() is None  # no step seen yet: the exact path
    spec.known = 2.0  # the exact path of step 1 stores its reduced value
    assert spec.plan() == pytest.approx(2.0 * 1.05 + 0.1)
    spec.pending = (_SlowEvent(), torch.tensor([0.0, 0.0, 3.0]))  # step 2's value, copy still queued
    assert spec.plan() == pytest.approx(3.0 * 1.05 + 0.1)
    assert spec.pending is None
    spec.pending = (_SlowEvent(), torch.tensor([0.0, 0.0, float("inf")]))  # non-finite: back to the exact path
    assert spec.plan() is None


def _bucket_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        b = _GradBuckets(None)
        parts1 = [torch.full((3, 2), float(rank + 1)), torch.arange(4, dtype=torch.float32) * (rank + 1)]
        parts2 = [torch.full((5,), 0.5 * (rank + 1), dtype=torch.bfloat16)]  # summed in float32
        b.add(parts1)
        b.add(parts2)
        out = b.wait()
        tot = sum(range(1, world + 1))
        ok = (len(out) == 2 and [t.shape for t in out[0]] == [(3, 2), (4,)] and out[1][0].shape == (5,)
              and torch.equal(out[0][0], torch.full((3, 2), float(tot)))
              and torch.equal(out[0][1], torch.arange(4, dtype=torch.float32) * tot)
              and out[1][0].dtype == torch.float32 and torch.allclose(out[1][0], torch.full((5,), 0.5 * tot)))
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_gradient_buckets_sum_over_ranks():
    """Parameter-gradient buckets: each bucket's all-reduce starts when it is added; wait() hands back
    every bucket's float32 sums in the shapes that went in, the same on every rank."""
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_bucket_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok for _, ok in res), res
