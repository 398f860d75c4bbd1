"""Benchmark of the 3D deformable slide attention hot path (DeformableSlideAttention3D fwd+bwd).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl ours|reference]

A "step" is one forward + backward of the module over one batch of synthetic tokens (loss =
sum(y * G) with a fixed G).  The default workload is BASELINE config 2: B=2, T=64, H=W=32
(131,072 tokens), C=1152, 16 heads x 72, window (3,7,7), bf16 activations with float32
accumulation, offset-conv weights ~N(0, 0.05).  Under torchrun the same volume is split along time
into one frame shard per rank (TimeShardedDSA3D: K/V halo exchange over NCCL; strong scaling); the
time is the max over ranks.

Prints one JSON line (rank 0): value = Mtokens/s with inputs resident in HBM; e2e = the same
through the module's public API with the input copied from pinned host memory and the loss read
back every step (the next step's copy runs on a side stream, double-buffered, while a step computes); roofline of the dominant kernel timed live with CUDA events; clocks sampled by
nvidia-smi during the timed region; cpu_baseline = the CPU oracle (oracle/) on a bounded sample.

``--impl reference`` times the reference algorithm's CPU implementation instead (the oracle port,
all host threads) on a bounded sample of the same workload; under torchrun only rank 0 works.
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
    # name: B, T, H, W, C, nh, kernel, dtype, offset weight std
    "c1": dict(B=1, T=8, H=16, W=16, C=256, nh=4, kernel=(3, 7, 7), dtype="float32", ostd=1e-2),
    "c2": dict(B=2, T=64, H=32, W=32, C=1152, nh=16, kernel=(3, 7, 7), dtype="bfloat16", ostd=0.05),
    # config-2 widths on 16 frames: the case profiled with ncu (inputs > L2, a few GB on the device)
    "c2_prof": dict(B=1, T=16, H=32, W=32, C=1152, nh=16, kernel=(3, 7, 7), dtype="bfloat16", ostd=0.05),
}
METRIC = "3D-DSA fwd+bwd Mtokens/s"
# reduced-volume sample of a config timed on the CPU (same C, heads, window; fewer frames)
CPU_SAMPLE = {"c1": dict(B=1, T=8, H=16, W=16), "c2": dict(B=1, T=8, H=16, W=16),
              "c2_prof": dict(B=1, T=8, H=16, W=16)}


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
    return ap.parse_args()


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
    params["offset_net.2.weight"] = rng.normal(0, c["ostd"], (nh * K * 3, C, 1, 1, 1))
    params["offset_net.2.bias"] = np.zeros(nh * K * 3)
    x = rng.normal(size=(B, T * H * W, C))
    g = rng.normal(size=(B, T * H * W, C))
    t0 = time.perf_counter()
    _, cache = O.module_forward(params, x, (T, H, W), heads=nh, kernel_size=ks)
    O.module_backward(cache, g)
    return time.perf_counter() - t0, B * T * H * W


def cpu_baseline(cfg_name: str, reps: int = 3):
    threads = os.cpu_count() or 1
    cpu_sample_step(cfg_name, threads)  # warm-up (page-in, thread pool)
    times = []
    for _ in range(reps):
        dt, tok = cpu_sample_step(cfg_name, threads)
        times.append(dt)
    med = statistics.median(times)
    s = CPU_SAMPLE[cfg_name]
    return {"value": tok / med / 1e6, "unit": "Mtokens/s", "cores": threads, "kind": "port",
            "sample": f"oracle/ (C + numpy float64) fwd+bwd of {cfg_name}'s C/heads/window on a reduced volume "
                      f"B={s['B']} T={s['T']} H={s['H']} W={s['W']} ({tok} tokens), median of {reps} after 1 warm-up",
            "seconds_per_sample": med}


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
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
                         "sample": f"oracle/ fwd+bwd on {tok} tokens of {args.config}'s C/heads/window per step"},
        "e2e": {"value": value, "unit": "Mtokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def _workload_name(name, c):
    return (f"{name}: DeformableSlideAttention3D fwd+bwd B={c['B']} T={c['T']} H={c['H']} W={c['W']} "
            f"C={c['C']} heads={c['nh']}x{c['C'] // c['nh']} window={c['kernel']} {c['dtype']}")


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
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.file, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

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
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def _alg_bytes_per_token(name, C, nh, K, es, probs=False):
    """Algorithmic HBM bytes per token of one launch of each entry point (operands crossing the
    entry point once; float32 accumulators inside msl_dsa_attn_bwd are scratch, not counted).
    probs: the tensor-core path, whose forward also writes the per-sample softmax weights (float32
    [nh, K] per token) and records (8 bytes per sample, `saved`) that its backward reads instead of
    the offsets.  The backward writes the offset gradients in the compute dtype (es bytes)."""
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


def _flops_per_token(name, C, nh, K, d):
    """CUDA-core float32 FLOPs per token of the gather kernels (corner dot products and value
    interpolation: 8 corners x d MACs per K/V use)."""
    if name == "msl_dsa_attn_fwd":
        return nh * K * 8 * d * 2 * 2  # q.k_c and p*w*v_c
    if name == "msl_dsa_attn_bwd":
        return nh * K * 8 * d * 2 * 5  # q.k_c, dout.v_c, dq, dk, dv
    return None


def run_gpu(args):
    import torch
    import torch.distributed as dist

    import megaslide_b200 as msl
    from megaslide_b200 import ops

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    c = CONFIGS[args.config]
    B, T, H, W, C, nh, ks = c["B"], c["T"], c["H"], c["W"], c["C"], c["nh"], c["kernel"]
    dt = getattr(torch, c["dtype"])
    N = T * H * W
    K = ks[0] * ks[1] * ks[2]
    d = C // nh
    es = 2 if dt == torch.bfloat16 else 4

    torch.manual_seed(1234)  # the same parameters on every rank (one module, sharded along time)
    mod = msl.DeformableSlideAttention3D(C, nh, ks)
    with torch.no_grad():
        for p in (mod.offset_net[2].weight, mod.offset_net[2].bias):
            p.normal_(0, c["ostd"])
    mod = mod.to(dev, dt)
    gen = torch.Generator(device=dev)
    gen.manual_seed(4321)  # the same global volume on every rank and for every N
    x = torch.randn(B, N, C, device=dev, dtype=dt, generator=gen)
    G = torch.randn(B, N, C, device=dev, dtype=dt, generator=gen)
    params = list(mod.parameters())

    if world > 1:
        # strong scaling: the config's volume is sharded along time (every N sees the same seeded
        # tokens and offsets); each rank exchanges the halo frames its samples reach over NCCL
        from megaslide_b200.sharded import TimeShardedDSA3D, shard_ranges

        owns = shard_ranges(T, world)
        fwd = TimeShardedDSA3D(mod, frame_ranges=owns)
        rows = slice(owns[rank][0] * H * W, owns[rank][1] * H * W)
        x = x[:, rows].contiguous()
        G = G[:, rows].contiguous()
    else:
        fwd = mod
    vshape = (T, H, W)

    def step(inp):
        y = fwd(inp, vshape)
        y.backward(G)
        for p in params:
            p.grad = None
        return y

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step(x)
    barrier()

    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    n0 = msl.launch_count()
    stream = torch.cuda.current_stream()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with ops.kernel_timer() as rec:
        e0.record(stream)
        for _ in range(args.steps):
            step(x)
        e1.record(stream)
    launches = msl.launch_count() - n0
    barrier()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    tokens = B * N  # the whole (sharded) volume
    value = tokens * args.steps / (ms / 1e3) / 1e6

    # per entry point device time inside the timed region
    per = {}
    for name, s, e in rec:
        tot, cnt = per.get(name, (0.0, 0))
        per[name] = (tot + s.elapsed_time(e), cnt + 1)
    dom = max(per, key=lambda n: per[n][0])
    dom_ms = per[dom][0] / per[dom][1]
    hbm_peak, tc_peak, peak_kind = _peaks()
    tc_path = dt == torch.bfloat16 and d % 8 == 0 and 16 <= d <= 128  # tensor-core kernels, probs saved
    n_local = x.shape[1]  # this rank's tokens per sample (the kernels' launch size)
    alg_bytes = _alg_bytes_per_token(dom, C, nh, K, es, probs=tc_path) * B * n_local
    achieved = alg_bytes / (dom_ms / 1e3) / 1e9
    traffic = None
    tfile = ROOT / "profiles" / "traffic.json"
    if tfile.exists():
        tj = json.loads(tfile.read_text()).get(dom, {}).get(args.config)
        if tj:
            traffic = float(tj["bytes_per_token"]) * B * n_local
    roof = {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
            "traffic": traffic, "kernel": dom, "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})",
            "algorithmic_bytes_per_launch": alg_bytes, "launch_ms": dom_ms}
    fl = _flops_per_token(dom, C, nh, K, d)
    if fl:
        clk = clocks.get("sm_mhz") or 1965.0
        fp32_peak = 148 * 128 * 2 * clk * 1e6 / 1e12
        ach = fl * B * n_local / (dom_ms / 1e3) / 1e12
        roof["fp32_cuda_core"] = {"achieved": ach, "peak": fp32_peak, "unit": "TFLOP/s", "frac": ach / fp32_peak,
                                  "peak_source": "nominal 148 SMs x 128 FMA/clk at the sampled median SM clock"}
    kernels = {n: {"ms_per_launch": v[0] / v[1], "launches": v[1], "share": v[0] / sum(t for t, _ in per.values())}
               for n, v in sorted(per.items(), key=lambda kv: -kv[1][0])}

    e2e = None
    if not args.no_e2e:
        # End to end through the module: every step copies its input from pinned host memory and reads its
        # loss back.  As in a training input pipeline, step i+1's input is copied on a side stream into the
        # other of two device buffers while step i computes (the copy waits until the step before has
        # finished with that buffer); every step's copy and read-back lie inside the timed region.
        xh = x.detach().cpu().pin_memory()
        xd = [torch.empty_like(x), torch.empty_like(x)]
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
                y = step(xd[b])
                freed[b].record(stream)
                loss = (y * G).sum(dtype=torch.float32)
                loss_h.copy_(loss.view(1), non_blocking=True)

        e2e_run(max(1, args.warmup))
        barrier()
        e0.record(stream)
        e2e_run(args.steps)
        e1.record(stream)
        barrier()
        ms2 = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms2], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms2 = float(t.item())
        e2e = {"value": tokens * args.steps / (ms2 / 1e3) / 1e6, "unit": "Mtokens/s",
               "h2d_bytes_per_step": xh.numel() * xh.element_size(), "d2h_bytes_per_step": 4,
               "ms_per_step": ms2 / args.steps,
               "h2d": "pinned host -> device on a copy stream, double-buffered: step i+1's input copies while step i runs"}

    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.config)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "Mtokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak",
            "vs_baseline": None, "dtype": "bf16" if dt == torch.bfloat16 else "f32",
            "data": "synthetic (seeded torch.randn tokens; random-init weights)",
            "config": {"workload": _workload_name(args.config, c), "tokens_per_step": tokens,
                       "parallelism": (f"time-sharded x{world}: {T}-frame volume split into {T // world}-frame shards, "
                                       "K/V halo exchange over NCCL") if world > 1 else "single GPU",
                       "l2": f"inputs larger than L2 (x = {x.numel() * x.element_size() / 1e6:.0f} MB per GPU)"},
            "e2e": e2e, "roofline": roof, "cpu_baseline": cpu, "clocks": clocks, "gpu_launches": launches,
            "kernels": kernels,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


def run_dit(args):
    """DiT step time (fwd + bwd + AdamW) of the streaming CPU-master trainer on one GPU."""
    import torch

    import megaslide_b200 as msl
    from megaslide_b200.dit import MegaSlideDiT, VideoDiTConfig
    from megaslide_b200.stream import CPUMasterVideoDiT

    if args.gpus != 1 or int(os.environ.get("WORLD_SIZE", "1")) != 1:
        raise SystemExit("--config c3 runs on one GPU (the CPU-master trainer is single-device)")
    cfg = VideoDiTConfig(**DIT_CONFIGS[args.config], device=0)
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
    t0 = time.perf_counter()
    for _ in range(args.steps):
        loss = step(record=True)
    t_drain = time.perf_counter()
    trainer.get_parameters()  # the last step's host AdamW is part of the step
    phases["final_drain_s"] = time.perf_counter() - t_drain
    torch.cuda.synchronize()
    sec = (time.perf_counter() - t0) / args.steps
    clocks = sampler.stop()
    launches = msl.launch_count() - n0
    h2d = (trainer.h2d_bytes - h0) / args.steps
    d2h = (trainer.d2h_bytes - d0) / args.steps
    tokens = cfg.num_patches
    trainer.cleanup()
    line = {
        "metric": "DiT step time (fwd+bwd+AdamW, CPU-master streaming)", "value": sec, "unit": "s/step",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded latents / noise; random init)",
        "config": {"workload": f"{args.config}: MegaSlideDiT {cfg.num_layers} blocks, hidden {cfg.hidden_size}, "
                               f"{cfg.num_heads} heads, MLP x{cfg.mlp_ratio}, latent {cfg.in_channels}x{cfg.frames}x"
                               f"{cfg.height}x{cfg.width}, patch {cfg.patch_size} ({tokens} tokens), window "
                               f"{tuple(cfg.dsa_kernel_size)}, checkpoint every {cfg.checkpoint_interval} blocks",
                   "tokens_per_step": tokens, "parallelism": "single GPU, blocks streamed through 2 slots",
                   "timing": "wall clock per step including the host AdamW (synchronised at both ends)"},
        "e2e": {"value": sec, "unit": "s/step", "h2d_bytes_per_step": int(h2d + 2 * lat.numel() * 4 + 8),
                "d2h_bytes_per_step": int(d2h + 4)},
        "stream": {"weight_h2d_gbs": h2d / sec / 1e9, "grad_d2h_gbs": d2h / sec / 1e9,
                   "weight_bytes_per_step": h2d, "grad_bytes_per_step": d2h, "loss": loss},
        "phases_per_step": {k: v / (1 if k == "final_drain_s" else args.steps) for k, v in phases.items()},
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
