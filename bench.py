"""Benchmark of the 3D deformable slide attention hot path (DeformableSlideAttention3D fwd+bwd).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl ours|reference]

A "step" is one forward + backward of the module over one batch of synthetic tokens (loss =
sum(y * G) with a fixed G).  The default workload is BASELINE config 2: B=2, T=64, H=W=32
(131,072 tokens), C=1152, 16 heads x 72, window (3,7,7), bf16 activations with float32
accumulation, offset-conv weights ~N(0, 0.05).  Under torchrun the same volume is split along time
into one frame shard per rank (TimeShardedDSA3D: K/V halo exchange over NCCL; strong scaling); the
time is the max over ranks.  Inputs are seeded per global frame, so every N sees the same tokens.

Prints one JSON line (rank 0): value = Mtokens/s with inputs resident in HBM; e2e = the same
through the module's public API with the input copied from pinned host memory and the loss read
back every step (the next step's copy runs on a side stream, double-buffered, while a step
computes); roofline of the dominant kernel timed live with CUDA events, with the op's binding roof;
clocks sampled by nvidia-smi during the timed region; cpu_baseline = the CPU oracle (oracle/) on a
bounded sample; parity = one more step after the timed region checked against the oracle at
sampled rows on every rank (oracle/sampled.py); c4 = the 1M-token config (raw offsets ~N(0,1)
clipped to +-3, injected) at the same N, timed and checked the same way (on one GPU only when it fits).

``--impl reference`` times the reference algorithm's CPU implementation instead (the oracle port,
all host threads) on a bounded sample of the same workload; under torchrun only rank 0 works.
``--config c3`` times the DiT step of the CPU-master streaming trainer instead.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIGS = {
    # name: B, T, H, W, C, nh, kernel, dtype, offset weight std (learned offsets) or clip (injected offsets)
    "c1": dict(B=1, T=8, H=16, W=16, C=256, nh=4, kernel=(3, 7, 7), dtype="float32", ostd=1e-2),
    "c2": dict(B=2, T=64, H=32, W=32, C=1152, nh=16, kernel=(3, 7, 7), dtype="bfloat16", ostd=0.05),
    # config-2 widths on 16 frames: the case profiled with ncu (inputs > L2, a few GB on the device)
    "c2_prof": dict(B=1, T=16, H=32, W=32, C=1152, nh=16, kernel=(3, 7, 7), dtype="bfloat16", ostd=0.05),
    # the 1M-token long-sequence config: raw offsets ~N(0,1) clipped to +-3 injected in place of the
    # offset predictor's output (seeded per global frame, identical for every GPU count)
    "c4": dict(B=1, T=256, H=64, W=64, C=1536, nh=24, kernel=(3, 7, 7), dtype="bfloat16", clip=3.0),
    # c4's widths and offsets on 16 frames (timing probes) and on 8 frames (ncu captures: a few GB).  The
    # reference divides the offset that moves the time axis by W-1 and the one that moves the width axis
    # by T-1, so fewer frames turn c4's +-6.1-frame temporal spread into a +-6.4 (T=16) or +-13.7 (T=8)
    # column spread: these two cases have other envelopes than c4
    "c4_prof": dict(B=1, T=16, H=64, W=64, C=1536, nh=24, kernel=(3, 7, 7), dtype="bfloat16", clip=3.0),
    "c4_ncu": dict(B=1, T=8, H=64, W=64, C=1536, nh=24, kernel=(3, 7, 7), dtype="bfloat16", clip=3.0),
    # bands of fewer rows keep T and W and so the sample spread of c2 / c4 (the height offsets do not depend
    # on T or W; more samples clamp at the upper and lower border): the reduced cases that stand for them
    "c2_band": dict(B=1, T=64, H=8, W=32, C=1152, nh=16, kernel=(3, 7, 7), dtype="bfloat16", ostd=0.05),
    "c4_band": dict(B=1, T=256, H=8, W=64, C=1536, nh=24, kernel=(3, 7, 7), dtype="bfloat16", clip=3.0),
}
METRIC = "3D-DSA fwd+bwd Mtokens/s"
# reduced-volume sample of a config timed on the CPU (same C, heads, window; fewer frames)
CPU_SAMPLE = {"c1": dict(B=1, T=8, H=16, W=16), "c2": dict(B=1, T=8, H=16, W=16),
              "c2_prof": dict(B=1, T=8, H=16, W=16), "c4": dict(B=1, T=8, H=16, W=16),
              "c4_prof": dict(B=1, T=8, H=16, W=16), "c4_ncu": dict(B=1, T=8, H=16, W=16),
              "c2_band": dict(B=1, T=8, H=16, W=16), "c4_band": dict(B=1, T=8, H=16, W=16)}


# DiT step time with CPU-master streaming (the reference's MegaSlideDiT architecture:
# additive timestep embedding, no adaLN).  Not the default workload: python bench.py --config c3
DIT_CONFIGS = {
    "c3": dict(frames=32, in_channels=4, height=64, width=64, patch_size=2, hidden_size=1152, num_heads=16,
               num_layers=28, mlp_ratio=4.0, dsa_kernel_size=(3, 7, 7), learning_rate=1e-4, dtype="bfloat16",
               checkpoint_interval=4, num_grad_slabs=4, log_interval=0),
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS) + sorted(DIT_CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the sampled-row oracle check after timing")
    ap.add_argument("--no-c4", action="store_true", help="skip the extra c4 (1M-token) measurement")
    ap.add_argument("--parity-rows", type=int, default=2048)
    ap.add_argument("--resident", action="store_true", help="c3: force resident mode (weights kept in HBM)")
    ap.add_argument("--streamed", action="store_true", help="c3: force streamed mode (weights streamed per block)")
    return ap.parse_args()


def _host_threads():
    """Every host thread for the CPU arms: OpenMP (the C oracle) and the BLAS pool numpy uses.  torchrun
    sets OMP_NUM_THREADS=1 in every rank, which would otherwise make the CPU figures depend on N."""
    n = os.cpu_count() or 1
    for var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[var] = str(n)
    blas = None
    try:
        from threadpoolctl import threadpool_info, threadpool_limits

        threadpool_limits(limits=n)
        blas = max((i.get("num_threads", 0) for i in threadpool_info()), default=None)
    except Exception:
        pass
    return n, blas


# ----------------------------------------------------------------------------- CPU (oracle)
def cpu_sample_step(cfg_name: str, threads: int):
    """One fwd+bwd of the CPU oracle on the config's reduced-volume sample; returns (seconds, tokens)."""
    import numpy as np

    from oracle import dsa_oracle as O

    O.set_num_threads(threads)
    c = CONFIGS[cfg_name]
    s = CPU_SAMPLE[cfg_name]
    B, T, H, W = s["B"], s["T"], s["H"], s["W"]
    C, nh, ks = c["C"], c["nh"], c["kernel"]
    rng = np.random.default_rng(0)
    K = ks[0] * ks[1] * ks[2]
    lim = math.sqrt(6.0 / (2 * C))
    params = {}
    for nm in ("q_proj", "k_proj", "v_proj", "out_proj"):
        params[nm + ".weight"] = rng.uniform(-lim, lim, (C, C))
        params[nm + ".bias"] = np.zeros(C)
    params["dw_conv.weight"] = rng.normal(0, 1 / math.sqrt(K), (C, 1, *ks))
    params["dw_conv.bias"] = np.zeros(C)
    params["offset_net.0.weight"] = rng.normal(0, 1 / math.sqrt(27), (C, 1, 3, 3, 3))
    params["offset_net.0.bias"] = np.zeros(C)
    params["offset_net.2.weight"] = rng.normal(0, c.get("ostd") or 0.0, (nh * K * 3, C, 1, 1, 1))
    params["offset_net.2.bias"] = np.zeros(nh * K * 3)
    x = rng.normal(size=(B, T * H * W, C))
    g = rng.normal(size=(B, T * H * W, C))
    off = None
    if c.get("clip"):
        off = np.clip(rng.normal(size=(B, T * H * W, nh * K * 3)), -c["clip"], c["clip"]).astype(np.float32)
    t0 = time.perf_counter()
    _, cache = O.module_forward(params, x, (T, H, W), heads=nh, kernel_size=ks, offsets=off)
    O.module_backward(cache, g)
    return time.perf_counter() - t0, B * T * H * W


def _cpu_sample_desc(cfg_name, tok):
    s = CPU_SAMPLE[cfg_name]
    inj = " with injected offsets (clip {})".format(CONFIGS[cfg_name]["clip"]) if CONFIGS[cfg_name].get("clip") else ""
    return (f"oracle/ (C + numpy float64) fwd+bwd of {cfg_name}'s C/heads/window{inj} on a reduced volume "
            f"B={s['B']} T={s['T']} H={s['H']} W={s['W']} ({tok} tokens)")


def cpu_baseline(cfg_name: str, reps: int = 3):
    threads, blas = _host_threads()
    cpu_sample_step(cfg_name, threads)  # warm-up (page-in, thread pool)
    times = []
    tok = 0
    for _ in range(reps):
        dt, tok = cpu_sample_step(cfg_name, threads)
        times.append(dt)
    med = statistics.median(times)
    return {"value": tok / med / 1e6, "unit": "Mtokens/s", "cores": threads, "kind": "port",
            "sample": _cpu_sample_desc(cfg_name, tok) + f", median of {reps} after 1 warm-up",
            "seconds_per_sample": med, "threads": {"openmp": threads, "blas": blas}}


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads, blas = _host_threads()
    for _ in range(args.warmup):
        cpu_sample_step(args.config, threads)
    times = []
    tok = 0
    for _ in range(args.steps):
        dt, tok = cpu_sample_step(args.config, threads)
        times.append(dt)
    total = sum(times)
    value = tok * args.steps / total / 1e6
    s = CPU_SAMPLE[args.config]
    c = CONFIGS[args.config]
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "Mtokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": _workload_name(args.config, c), "sample": f"B={s['B']} T={s['T']} H={s['H']} W={s['W']}"},
        "cpu_baseline": {"value": value, "unit": "Mtokens/s", "cores": threads, "kind": "port",
                         "sample": _cpu_sample_desc(args.config, tok) + " per step",
                         "threads": {"openmp": threads, "blas": blas}},
        "e2e": {"value": value, "unit": "Mtokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def _workload_name(name, c):
    offs = (f"raw offsets ~N(0,1) clipped to +-{c['clip']} injected" if c.get("clip")
            else f"learned offsets (offset-conv weights ~N(0,{c['ostd']}))")
    return (f"{name}: DeformableSlideAttention3D fwd+bwd B={c['B']} T={c['T']} H={c['H']} W={c['W']} "
            f"C={c['C']} heads={c['nh']}x{c['C'] // c['nh']} window={c['kernel']} {c['dtype']}, {offs}")


# ----------------------------------------------------------------------------- GPU
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.file = None

    def start(self):
        """Starts nvidia-smi and returns once it has written its first sample (its start-up queries the
        driver and must not overlap a timed region), or after 10 s."""
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.file, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return
        t0 = time.time()
        while time.time() - t0 < 10.0 and self.proc.poll() is None:
            if os.path.getsize(self.file.name) > 0:
                break
            time.sleep(0.05)
        time.sleep(0.25)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.seek(0)
        rows = [r.split(",") for r in self.file.read().strip().splitlines() if r.count(",") >= 8]
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if "Active" in v and "Not" not in v})
        pw = [float(r[3]) for r in rows if r[3].strip().replace(".", "").isdigit()]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "power_w_max": max(pw) if pw else None}


def _peaks():
    """(hbm GB/s, bf16 TFLOP/s burst, bf16 TFLOP/s sustained, source) from MEASURED_PEAKS.json."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return (float(d["hbm_gbs"]), float(d["bf16_tflops"]),
                float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured")
    return 6650.0, 1590.0, 1400.0, "fallback"


def _op_bytes_per_token(C, nh, es):
    """The op's algorithmic HBM bytes per token (a token = one query position of one sample through
    fwd+bwd): every activation crosses the op boundary once at the compute dtype, Q/K/V saved for the
    backward, one float32 log-sum-exp per head saved and re-read; offsets never reach HBM.
    forward: read x, write y, write Q, K, V            = 5 C es + 4 nh
    backward: read x, dy, Q, K, V, write dx            = 6 C es + 4 nh
    (22 C + 8 nh at bf16)."""
    return {"msl_dsa_attn_fwd": 5 * C * es + 4 * nh, "msl_dsa_attn_bwd": 6 * C * es + 4 * nh,
            "op": 11 * C * es + 8 * nh}


def _kernel_io_bytes_per_token(name, C, nh, K, es, probs=False):
    """Bytes each attention entry point of THIS build reads and writes per token (operands crossing the
    entry point once; float32 dK/dV accumulators are scratch, not counted): besides q/k/v/out/lse it
    materialises the float32 offsets, and on the tensor-core path the per-sample softmax weights
    (float32 [nh, K]) and 8-byte records that the backward reads instead of the offsets; the backward
    writes the offset gradients in the compute dtype."""
    off = 4 * nh * K * 3
    doff = es * nh * K * 3
    pr = 4 * nh * K if probs else 0
    rec = 8 * nh * K if probs else 0
    if name == "msl_dsa_attn_bwd":  # read q k v out dout lse, offsets or (probs, records); write dq dk dv doffsets
        return 5 * C * es + (pr + rec if probs else off) + 4 * nh + 3 * C * es + doff
    if name == "msl_dsa_attn_fwd":  # read q k v offsets, write out lse (probs, records)
        return 3 * C * es + off + C * es + 4 * nh + pr + rec
    if name == "msl_dwconv3d_bwd_weight":  # read dy, x
        return 2 * C * es
    return 2 * C * es  # read x, write y


def _frames_randn(seed, B, frames, HW, cols, dev, dtype, clip=None):
    """[B, len(frames)*HW, cols] standard normals, one generator per global (sample, frame): every GPU
    count sees the same values for a given global token."""
    import torch

    out = torch.empty(B, len(frames) * HW, cols, device=dev, dtype=dtype)
    g = torch.Generator(device=dev)
    for b in range(B):
        for i, t in enumerate(frames):
            g.manual_seed(seed * 1_000_003 + b * 65_537 + t)
            blk = out[b, i * HW:(i + 1) * HW]
            blk.copy_(torch.randn(HW, cols, device=dev, dtype=torch.float32, generator=g))
            if clip is not None:
                blk.clamp_(-clip, clip)
    return out


class Workload:
    """One config's module, inputs and step on this rank (time-sharded over the ranks when world > 1)."""

    def __init__(self, name, dev, world, rank):
        import torch

        import megaslide_b200 as msl

        c = CONFIGS[name]
        self.name, self.c, self.world, self.rank = name, c, world, rank
        self.B, self.T, self.H, self.W, self.C, self.nh, self.ks = (c["B"], c["T"], c["H"], c["W"], c["C"], c["nh"],
                                                                    c["kernel"])
        self.dt = getattr(torch, c["dtype"])
        self.K = self.ks[0] * self.ks[1] * self.ks[2]
        self.d = self.C // self.nh
        self.es = 2 if self.dt == torch.bfloat16 else 4
        self.clip = c.get("clip")
        HW = self.H * self.W
        torch.manual_seed(1234)  # the same parameters on every rank (one module, sharded along time)
        mod = msl.DeformableSlideAttention3D(self.C, self.nh, self.ks)
        if c.get("ostd"):
            with torch.no_grad():
                for p in (mod.offset_net[2].weight, mod.offset_net[2].bias):
                    p.normal_(0, c["ostd"])
        self.mod = mod.to(dev, self.dt)
        self.params = list(self.mod.parameters())
        if world > 1:
            from megaslide_b200.sharded import TimeShardedDSA3D, shard_ranges

            self.owns = shard_ranges(self.T, world)
            # learned offsets: the K/V window of a step is planned from the previous step's largest offset
            # (checked exactly by the kernels' halo-miss bit, reported by the status word after the run)
            self.fwd = TimeShardedDSA3D(self.mod, frame_ranges=self.owns, speculative_window=not self.clip)
        else:
            self.owns = [(0, self.T)]
            self.fwd = self.mod
        own = self.owns[rank]
        frames = range(own[0], own[1])
        # the same global volume on every rank and for every N (seeded per global frame)
        self.x = _frames_randn(4321, self.B, frames, HW, self.C, dev, self.dt)
        self.G = _frames_randn(8765, self.B, frames, HW, self.C, dev, self.dt)
        self.off = (_frames_randn(2468, self.B, frames, HW, self.nh * self.K * 3, dev, torch.float32, clip=self.clip)
                    if self.clip else None)
        self.vshape = (self.T, self.H, self.W)
        self.tokens = self.B * self.T * HW  # the whole (sharded) volume
        self.n_local = self.x.shape[1]

    def run(self, inp):
        if self.off is None:
            return self.fwd(inp, self.vshape)
        if self.world > 1:
            return self.fwd.forward_with_offsets(inp, self.vshape, self.off, offset_bound=self.clip)
        return self.fwd.forward_with_offsets(inp, self.vshape, self.off)

    def step(self, inp, keep_grads=False):
        y = self.run(inp)
        y.backward(self.G)
        if not keep_grads:
            for p in self.params:
                p.grad = None
        return y

    def parity(self, n_rows, seed=0):
        """One more step with the intermediates captured, checked against the oracle at sampled rows."""
        import torch
        import torch.distributed as dist

        from oracle import sampled

        cap: dict = {}
        self.fwd.capture = cap
        try:
            self.step(self.x, keep_grads=True)
        finally:
            self.fwd.capture = None
        torch.cuda.synchronize()
        kw = {}
        if self.world > 1:
            own, win = cap["own"], cap["kvwin"]
            kw = dict(q_frame0=own[0], q_frames=own[1] - own[0], kv_frame0=win[0], kv_frames=win[1] - win[0],
                      world=self.world)
        t0 = time.perf_counter()
        res = sampled.check(self.mod, cap, self.vshape, batch=self.B, dtype=self.dt,
                            n_rows=max(64, n_rows // self.world), seed=seed + self.rank,
                            injected=self.off is not None, **kw)
        res["seconds"] = time.perf_counter() - t0
        halo = [cap["own"][0] - cap["kvwin"][0], cap["kvwin"][1] - cap["own"][1]] if self.world > 1 else [0, 0]
        for p in self.params:
            p.grad = None
        del cap
        if self.world > 1:
            allr = [None] * self.world
            dist.all_gather_object(allr, (res, halo))
        else:
            allr = [(res, halo)]
        return _merge_parity(allr)


def _merge_parity(allr):
    """Per entry: the worst error over ranks; ok when every rank's entry is."""
    out = {}
    for res, _ in allr:
        for k, v in res.items():
            if isinstance(v, dict):
                o = out.setdefault(k, {"err": v["err"], "tol": v["tol"], "ok": True})
                o["err"] = max(o["err"], v["err"])
                o["ok"] = o["ok"] and v["ok"]
    out["ok"] = all(v["ok"] for v in out.values() if isinstance(v, dict))
    out["n_rows"] = sum(r["n_rows"] for r, _ in allr)
    out["ranks"] = len(allr)
    out["seconds_max"] = max(r["seconds"] for r, _ in allr)
    out["halo_frames_max"] = [max(h[0] for _, h in allr), max(h[1] for _, h in allr)]
    return out


def time_steps(wl, steps, warmup, barrier, local, world, dev):
    """W warm-up steps, then K steps bracketed by barrier + synchronize, CUDA events on the launching
    stream, max over ranks.  Returns (ms total, library launches, per-entry-point device times, clocks)."""
    import torch
    import torch.distributed as dist

    import megaslide_b200 as msl
    from megaslide_b200 import ops

    for _ in range(warmup):
        wl.step(wl.x)
    barrier()
    sampler = ClockSampler(local)
    sampler.start()
    if world > 1:
        dist.barrier()  # every rank's sampler is up before the timed region
    torch.cuda.synchronize()
    n0 = msl.launch_count()
    stream = torch.cuda.current_stream()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with ops.kernel_timer() as rec:
        e0.record(stream)
        for _ in range(steps):
            wl.step(wl.x)
        e1.record(stream)
    launches = msl.launch_count() - n0
    barrier()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    per = {}
    for name, s, e in rec:
        tot, cnt = per.get(name, (0.0, 0))
        per[name] = (tot + s.elapsed_time(e), cnt + 1)
    return ms, launches, per, clocks


def roofline(wl, per, ms_step, clocks):
    """Roofline of the dominant entry point (section 8(d) bytes) plus the op's binding roof."""
    hbm_peak, tc_burst, tc_sust, peak_kind = _peaks()
    dom = max(per, key=lambda n: per[n][0])
    dom_ms = per[dom][0] / per[dom][1]
    C, nh, K, es = wl.C, wl.nh, wl.K, wl.es
    rows = wl.B * wl.n_local  # tokens one launch of the attention kernels processes on this rank
    opb = _op_bytes_per_token(C, nh, es)
    alg = opb.get(dom, 2 * C * es) * rows
    achieved = alg / (dom_ms / 1e3) / 1e9
    tc_path = wl.es == 2 and wl.d % 8 == 0 and 16 <= wl.d <= 128
    io = _kernel_io_bytes_per_token(dom, C, nh, K, es, probs=tc_path) * rows
    traffic = None
    tfile = ROOT / "profiles" / "traffic.json"
    if tfile.exists():
        tj = json.loads(tfile.read_text()).get(dom, {}).get(wl.name)
        if tj:
            traffic = float(tj["bytes_per_token"]) * rows
    roof = {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
            "traffic": traffic, "kernel": dom, "launch_ms": dom_ms,
            "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})",
            "algorithmic_bytes_per_launch": alg,
            "algorithmic_bytes_per_token": opb.get(dom),
            "kernel_io_bytes_per_launch": io,
            "materialised_bytes_per_launch": io - alg,
            "waste_ratio": (traffic / alg) if traffic else None}
    # the op's floors per step: HBM (22C+8nh bytes/token at bf16), the FP32 gather formulation
    # (140 K C flops/token) and the dense GEMMs on the tensor cores (24 C^2 + 6 C O flops/token, no
    # offset GEMM when offsets are injected)
    clk = clocks.get("sm_mhz") or 1965.0
    fp32_peak = 148 * 128 * 2 * clk * 1e6
    O = nh * K * 3
    tok = wl.tokens / wl.world  # per GPU
    floors = {
        "hbm_ms": tok * opb["op"] / (hbm_peak * 1e9) * 1e3,
        "fp32_gather_ms": tok * 140 * K * C / fp32_peak * 1e3,
        "tensor_gemm_ms": tok * (24 * C * C + (0 if wl.clip else 6 * C * O)) / (tc_sust * 1e12) * 1e3,
    }
    bind = max(floors, key=floors.get)
    roof["binding_roof"] = {
        "floors_ms_per_step": floors, "binding": bind, "ms_per_step": ms_step,
        "frac": floors[bind] / ms_step, "hbm_frac": floors["hbm_ms"] / ms_step,
        "peaks": {"hbm_gbs": hbm_peak, "fp32_tflops": fp32_peak / 1e12, "bf16_tflops_sustained": tc_sust},
        "note": "per GPU; fp32 peak = 148 SMs x 128 FMA/clk at the sampled median SM clock; "
                "bf16 = MEASURED_PEAKS.json sustained (a whole step under the power cap)"}
    return roof


def measure_e2e(wl, steps, warmup, barrier, world, dev):
    """End to end through the module: every step copies its input from pinned host memory and reads
    its loss back.  As in a training input pipeline, step i+1's input is copied on a side stream into
    the other of two device buffers while step i computes (the copy waits until the step before has
    finished with that buffer); every step's copy and read-back lie inside the timed region."""
    import torch
    import torch.distributed as dist

    stream = torch.cuda.current_stream()
    xh = wl.x.detach().cpu().pin_memory()
    xd = [torch.empty_like(wl.x), torch.empty_like(wl.x)]
    copy_stream = torch.cuda.Stream()
    copied = [torch.cuda.Event(), torch.cuda.Event()]
    freed = [torch.cuda.Event(), torch.cuda.Event()]
    loss_h = torch.empty(1, dtype=torch.float32).pin_memory()

    def issue_copy(i):
        b = i % 2
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(freed[b])
            xd[b].copy_(xh, non_blocking=True)
            copied[b].record(copy_stream)

    def e2e_run(n):
        copy_stream.wait_stream(stream)  # the first copy starts inside the caller's timed region
        issue_copy(0)
        for i in range(n):
            b = i % 2
            stream.wait_event(copied[b])
            if i + 1 < n:
                issue_copy(i + 1)
            y = wl.step(xd[b])
            freed[b].record(stream)
            loss = (y * wl.G).sum(dtype=torch.float32)
            loss_h.copy_(loss.view(1), non_blocking=True)

    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e2e_run(max(1, warmup))
    barrier()
    e0.record(stream)
    e2e_run(steps)
    e1.record(stream)
    barrier()
    ms2 = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms2], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms2 = float(t.item())
    return {"value": wl.tokens * steps / (ms2 / 1e3) / 1e6, "unit": "Mtokens/s",
            "h2d_bytes_per_step": xh.numel() * xh.element_size(), "d2h_bytes_per_step": 4,
            "ms_per_step": ms2 / steps,
            "h2d": "pinned host -> device on a copy stream, double-buffered: step i+1's input copies while step i runs"}


def msl_status_bits():
    """Synchronous read of this GPU's attention status word: raises MslError if any call of the run
    reported invalid results (a halo miss of the K/V window, a timed-out TMA wait); returns the
    informational bits (MSL_STATUS_TC_RANGE: tiles computed by the CUDA-core fallback)."""
    import megaslide_b200 as msl

    return int(msl.check_status())


def _c4_bytes_estimate(world):
    """Device bytes a c4 fwd+bwd needs on one rank (inputs, saved forward state, backward buffers)."""
    c = CONFIGS["c4"]
    C, nh, K = c["C"], c["nh"], 147
    frames = c["T"] / world + (16 if world > 1 else 0)  # own frames + the widest halo (+-3 offsets)
    rows = frames * c["H"] * c["W"]
    per_row = (2 * C * 3  # x, G, y
               + 4 * nh * K * 3  # injected float32 offsets
               + 2 * 3 * C + 2 * C + 2 * C  # qkv, attn, dw term
               + 4 * nh * K + 8 * nh * K  # probs, records
               + 2 * C + 2 * 3 * C + 8 * C + 2 * nh * K * 3 + 4 * C)  # dattn, dqkv, dK/dV accumulators, doff, dx
    return rows * per_row


def run_gpu(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    wl = Workload(args.config, dev, world, rank)
    ms, launches, per, clocks = time_steps(wl, args.steps, args.warmup, barrier, local, world, dev)
    value = wl.tokens * args.steps / (ms / 1e3) / 1e6
    roof = roofline(wl, per, ms / args.steps, clocks)
    kernels = {n: {"ms_per_launch": v[0] / v[1], "launches": v[1], "share": v[0] / sum(t for t, _ in per.values())}
               for n, v in sorted(per.items(), key=lambda kv: -kv[1][0])}
    e2e = None if args.no_e2e else measure_e2e(wl, args.steps, args.warmup, barrier, world, dev)
    parity = None if args.no_parity else wl.parity(args.parity_rows)
    x_mb = wl.x.numel() * wl.x.element_size() / 1e6
    main_cfg = {"workload": _workload_name(args.config, wl.c), "tokens_per_step": wl.tokens,
                "parallelism": (f"time-sharded x{world}: {wl.T}-frame volume split into {wl.T // world}-frame shards, "
                                "projected K/V halo rows exchanged over NCCL, K/V window planned from the previous "
                                "step's largest offset (verified by the kernels' halo-miss bit: status_ok)")
                               if world > 1 else "single GPU",
                "l2": f"inputs larger than L2 (x = {x_mb:.0f} MB per GPU)" if x_mb > 126 else
                      f"x = {x_mb:.0f} MB per GPU (below L2)"}
    del wl
    torch.cuda.empty_cache()

    c4 = None
    if not args.no_c4 and args.config != "c4" and not args.config.endswith(("_prof", "_ncu", "_band")):
        c4 = run_c4_leg(args, world, rank, dev, barrier, local)

    status_bits = msl_status_bits()  # raises if any step of the run (c4 included) reported invalid results

    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.config)

    if rank == 0:
        dt = CONFIGS[args.config]["dtype"]
        line = {
            "metric": METRIC, "value": value, "unit": "Mtokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak",
            "vs_baseline": None, "dtype": "bf16" if dt == "bfloat16" else "f32",
            "data": "synthetic (seeded torch.randn tokens per global frame; random-init weights)",
            "config": main_cfg,
            "e2e": e2e, "roofline": roof, "cpu_baseline": cpu, "clocks": clocks, "gpu_launches": launches,
            "kernels": kernels, "parity": parity, "c4": c4,
            "status_ok": True, "status_bits": status_bits,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


def run_c4_leg(args, world, rank, dev, barrier, local):
    """The 1M-token config c4 (raw offsets ~N(0,1) clipped to +-3) at this N: Mtok/s, ms/step, the K/V
    halo per side and a sampled-row parity check.  On one GPU it runs only when its estimated memory fits."""
    import torch

    need = _c4_bytes_estimate(world)
    free, total = torch.cuda.mem_get_info(dev)
    info = {"workload": _workload_name("c4", CONFIGS["c4"]), "n_gpus": world, "estimated_gb_per_gpu": need / 1e9,
            "device_gb": total / 1e9}
    if world == 1 and need > 0.92 * free:
        info.update(fits_one_gpu=False, reason=f"estimated {need / 1e9:.0f} GB > 92% of {free / 1e9:.0f} GB free")
        return info
    steps, warmup = max(3, min(args.steps, 5)), 2
    try:
        torch.cuda.reset_peak_memory_stats(dev)
        wl = Workload("c4", dev, world, rank)
        ms, launches, per, clocks = time_steps(wl, steps, warmup, barrier, local, world, dev)
        roof = roofline(wl, per, ms / steps, clocks)
        parity = None if args.no_parity else wl.parity(min(args.parity_rows, 1024))
        peak = torch.cuda.max_memory_allocated(dev)
        info.update(value=wl.tokens * steps / (ms / 1e3) / 1e6, unit="Mtokens/s", ms_per_step=ms / steps,
                    steps=steps, warmup=warmup, peak_mem_gb=peak / 1e9, fits_one_gpu=(world == 1) or None,
                    halo_frames_per_side=parity["halo_frames_max"] if parity else None,
                    kernels={n: {"ms_per_launch": v[0] / v[1], "launches": v[1]} for n, v in per.items()},
                    roofline={k: roof[k] for k in ("kernel", "launch_ms", "achieved", "frac", "traffic",
                                                   "waste_ratio", "binding_roof")},
                    clocks=clocks, gpu_launches=launches, parity=parity)
        del wl
    except torch.OutOfMemoryError as e:
        if world > 1:
            raise
        info.update(fits_one_gpu=False, reason=f"out of memory: {str(e).splitlines()[0][:200]}")
    torch.cuda.empty_cache()
    return info


def _host_memory():
    """Host RAM and cores of this box, and whether config 5's host state would fit: 33e9 parameters
    as an fp32 master, two fp32 AdamW moments, an fp32 gradient accumulator and a bf16 staging copy
    (18 bytes per parameter, ~594 GB) plus the fp32 model the trainer is built from (~132 GB)."""
    try:
        import psutil

        vm = psutil.virtual_memory()
        need = 33e9 * (18 + 4)
        return {"ram_total_gb": vm.total / 1e9, "ram_available_gb": vm.available / 1e9, "cores": os.cpu_count(),
                "c5_host_state_gb": need / 1e9, "c5_fits_host_ram": bool(vm.available > 1.15 * need)}
    except Exception as e:  # pragma: no cover
        return {"error": repr(e)}


def run_dit(args):
    """DiT step time (fwd + bwd + AdamW) of the streaming CPU-master trainer on one GPU."""
    import torch

    import megaslide_b200 as msl
    from megaslide_b200.dit import MegaSlideDiT, VideoDiTConfig
    from megaslide_b200.stream import CPUMasterVideoDiT

    if args.gpus != 1 or int(os.environ.get("WORLD_SIZE", "1")) != 1:
        raise SystemExit("--config c3 runs on one GPU (the CPU-master trainer is single-device)")
    mode = True if args.resident else (False if args.streamed else None)
    cfg = VideoDiTConfig(**DIT_CONFIGS[args.config], device=0, resident_blocks=mode)
    torch.manual_seed(1234)
    model = MegaSlideDiT(cfg)
    with torch.no_grad():  # learned offsets of the size the op benchmark uses (config 2)
        for b in model.blocks:
            b.attn.offset_net[2].weight.normal_(0, 0.05)
    trainer = CPUMasterVideoDiT(model, cfg)
    g = torch.Generator().manual_seed(4321)
    shape = (1, cfg.in_channels, cfg.frames, cfg.height, cfg.width)
    lat = torch.randn(shape, generator=g).pin_memory()
    noise = torch.randn(shape, generator=g).pin_memory()
    ts = torch.randint(0, 1000, (1,), generator=g)

    phases = {"fwd_bwd_wall_s": 0.0, "gpu_fwd_s": 0.0, "gpu_bwd_s": 0.0, "optimizer_call_s": 0.0}

    def step(record=False):
        trainer.zero_grad()
        t0 = time.perf_counter()
        loss, tm = trainer.forward_and_backward(lat, ts, noise)
        t1 = time.perf_counter()
        trainer.optimizer_step()
        t2 = time.perf_counter()
        if record:
            phases["fwd_bwd_wall_s"] += t1 - t0
            phases["gpu_fwd_s"] += tm["forward"]
            phases["gpu_bwd_s"] += tm["backward"]
            phases["optimizer_call_s"] += t2 - t1
        return loss

    for _ in range(args.warmup):
        step()
    trainer.get_parameters()  # host optimizer drained
    torch.cuda.synchronize()
    sampler = ClockSampler(0)
    sampler.start()
    time.sleep(0.3)
    n0, h0, d0 = msl.launch_count(), trainer.h2d_bytes, trainer.d2h_bytes
    from megaslide_b200 import ops

    t0 = time.perf_counter()
    with ops.kernel_timer() as rec:  # device time of this library's entry points inside the steps
        for _ in range(args.steps):
            loss = step(record=True)
    t_drain = time.perf_counter()
    trainer.get_parameters()  # the last step's host AdamW is part of the step
    phases["final_drain_s"] = time.perf_counter() - t_drain
    torch.cuda.synchronize()
    sec = (time.perf_counter() - t0) / args.steps
    clocks = sampler.stop()
    launches = msl.launch_count() - n0
    per = {}
    for name, s_ev, e_ev in rec:
        tot, cnt = per.get(name, (0.0, 0))
        per[name] = (tot + s_ev.elapsed_time(e_ev), cnt + 1)
    kernels = {n: {"ms_per_step": t / args.steps, "launches_per_step": c / args.steps}
               for n, (t, c) in sorted(per.items(), key=lambda kv: -kv[1][0])}
    h2d = (trainer.h2d_bytes - h0) / args.steps
    d2h = (trainer.d2h_bytes - d0) / args.steps
    tokens = cfg.num_patches
    resident = bool(trainer.resident)
    # one more step with the per-block event timeline (weight H2D / gradient D2H on their side streams
    # against block compute), after the timed region
    trainer.timeline = []
    origin = torch.cuda.Event(enable_timing=True)
    origin.record(torch.cuda.current_stream())
    step()
    trainer.get_parameters()
    torch.cuda.synchronize()
    from megaslide_b200.stream import timeline_summary

    timeline = timeline_summary(trainer.timeline, origin)
    trainer.timeline = None
    trainer.cleanup()
    line = {
        "metric": "DiT step time (fwd+bwd+AdamW, CPU-master streaming)", "value": sec, "unit": "s/step",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded latents / noise; random init)",
        "config": {"workload": f"{args.config}: MegaSlideDiT {cfg.num_layers} blocks, hidden {cfg.hidden_size}, "
                               f"{cfg.num_heads} heads, MLP x{cfg.mlp_ratio}, latent {cfg.in_channels}x{cfg.frames}x"
                               f"{cfg.height}x{cfg.width}, patch {cfg.patch_size} ({tokens} tokens), window "
                               f"{tuple(cfg.dsa_kernel_size)}, checkpoint every {cfg.checkpoint_interval} blocks",
                   "tokens_per_step": tokens,
                   "parallelism": ("single GPU, resident mode: every block's bf16 weights and activations kept "
                                   "in HBM, updated weights copied once per step" if resident else
                                   "single GPU, streamed mode: blocks streamed through 2 slots"),
                   "timing": "wall clock per step including the host AdamW (synchronised at both ends)"},
        "e2e": {"value": sec, "unit": "s/step", "h2d_bytes_per_step": int(h2d + 2 * lat.numel() * 4 + 8),
                "d2h_bytes_per_step": int(d2h + 4)},
        "stream": {"weight_h2d_gbs": h2d / sec / 1e9, "grad_d2h_gbs": d2h / sec / 1e9,
                   "weight_bytes_per_step": h2d, "grad_bytes_per_step": d2h, "loss": loss,
                   "timeline": timeline},
        "phases_per_step": {k: v / (1 if k == "final_drain_s" else args.steps) for k, v in phases.items()},
        "kernels": kernels,
        "host": _host_memory(),
        "clocks": clocks, "gpu_launches": launches,
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse()
    if args.config in DIT_CONFIGS:
        return run_dit(args)
    if args.impl == "reference":
        return run_reference_arm(args)
    return run_gpu(args)


if __name__ == "__main__":
    sys.exit(main())
