"""Generates the golden fixtures in tests/golden/*.npz by running the REFERENCE module.

Run in a container that has the reference checkout (jasonliu0704/megaslide) mounted:

    python tests/golden/make_golden.py --reference /path/to/megaslide

It imports ``infinity.video.attention.DeformableSlideAttention3D`` from that checkout, loads
parameters and inputs drawn from numpy's PCG64 generator (so every platform regenerates the same
values), runs forward + backward in float32 on CPU with loss = sum(y * dy), and stores inputs,
parameters, the output, every gradient and the intermediate raw offsets.  The tests only read the
.npz files; they never import the reference.

Cases cover: large offsets that hit the border clamp, zero offsets on odd sizes (sample
coordinates land exactly on voxel centres), the (3,7,7) window of BASELINE config 1, head_dim 72
(config 2's), extra keys/values, T=1 / W=1 / T=H=W=1 volumes, offset_scale != 1, the
reference's own non-causality construction, and BASELINE config 1 itself (stored as selected rows
plus full small gradients, since its inputs regenerate from the seed).
"""

from __future__ import annotations

import argparse
import math
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

CASES = {
    # name: (B, T, H, W, C, nh, kernel, offset_std, offset_scale, G, seed, note)
    "tiny_large_offsets": (1, 3, 4, 5, 8, 2, (3, 3, 3), 0.5, 1.0, 0, 11, "offsets of several voxels: border clamps"),
    "zero_offsets_odd": (2, 5, 3, 7, 12, 3, (3, 3, 3), 0.0, 1.0, 0, 12, "zero offset head, odd sizes: exact voxel centres"),
    "c1_window_small": (1, 4, 6, 6, 32, 4, (3, 7, 7), 1e-2, 1.0, 0, 13, "config-1 window/std on a small volume"),
    "extra_kv": (2, 2, 3, 4, 16, 4, (1, 3, 3), 0.3, 1.0, 4, 14, "G=4 extra keys/values"),
    "degenerate_111": (1, 1, 1, 1, 4, 2, (3, 3, 3), 0.0, 1.0, 0, 15, "T=H=W=1 (reference test)"),
    "t1_plane": (1, 1, 5, 6, 8, 2, (1, 3, 3), 0.5, 1.0, 0, 16, "T=1: channel-0 offsets unused"),
    "w1_column": (1, 4, 3, 1, 8, 1, (3, 3, 1), 0.5, 1.0, 0, 17, "W=1: channel-2 offsets unused"),
    "head_dim_72": (1, 3, 4, 4, 72, 1, (3, 7, 7), 0.05, 1.0, 0, 18, "config-2 head_dim 72"),
    "offset_scale_2": (1, 3, 4, 4, 16, 2, (3, 3, 3), 0.3, 2.0, 0, 19, "offset_scale = 2"),
    "c1_full": (1, 8, 16, 16, 256, 4, (3, 7, 7), 1e-2, 1.0, 0, 1234, "BASELINE config 1"),
}

# rows of y / dx kept for the large case (its inputs regenerate from the seed)
C1_ROWS = 96


def xavier(rng, fan_out, fan_in, shape):
    a = math.sqrt(6.0 / (fan_in + fan_out))
    return rng.uniform(-a, a, size=shape).astype(np.float32)


def make_inputs(name):
    """Parameters and inputs of a case, deterministic from its seed (numpy PCG64)."""
    B, T, H, W, C, nh, ks, ostd, oscale, G, seed, _ = CASES[name]
    rng = np.random.default_rng(seed)
    kt, kh, kw = ks
    K = kt * kh * kw
    O = nh * K * 3
    p = {}
    for nm in ("q_proj", "k_proj", "v_proj", "out_proj"):
        p[f"{nm}.weight"] = xavier(rng, C, C, (C, C))
        p[f"{nm}.bias"] = rng.normal(0, 0.02, size=(C,)).astype(np.float32)
    p["dw_conv.weight"] = rng.normal(0, 1.0 / math.sqrt(K), size=(C, 1, kt, kh, kw)).astype(np.float32)
    p["dw_conv.bias"] = rng.normal(0, 0.02, size=(C,)).astype(np.float32)
    p["offset_net.0.weight"] = rng.normal(0, 1.0 / math.sqrt(27), size=(C, 1, 3, 3, 3)).astype(np.float32)
    p["offset_net.0.bias"] = rng.normal(0, 0.02, size=(C,)).astype(np.float32)
    p["offset_net.2.weight"] = rng.normal(0, ostd, size=(O, C, 1, 1, 1)).astype(np.float32)
    p["offset_net.2.bias"] = rng.normal(0, ostd, size=(O,)).astype(np.float32)
    x = rng.normal(0, 1, size=(B, T * H * W, C)).astype(np.float32)
    dy = rng.normal(0, 1, size=(B, T * H * W, C)).astype(np.float32)
    extra = rng.normal(0, 1, size=(B, G, C)).astype(np.float32) if G else None
    return dict(params=p, x=x, dy=dy, extra=extra, video_shape=(T, H, W), heads=nh, kernel=ks,
                offset_scale=oscale)


def noncausal_inputs():
    """The reference's own construction (tests/test_megaslide_video.py:52-69): V and out_proj
    identity, everything else zero, kernel (3,1,1), video (2,1,1)."""
    C, nh, ks = 2, 1, (3, 1, 1)
    p = {}
    for nm in ("q_proj", "k_proj", "v_proj", "out_proj"):
        p[f"{nm}.weight"] = np.zeros((C, C), np.float32)
        p[f"{nm}.bias"] = np.zeros((C,), np.float32)
    p["v_proj.weight"] = np.eye(C, dtype=np.float32)
    p["out_proj.weight"] = np.eye(C, dtype=np.float32)
    p["dw_conv.weight"] = np.zeros((C, 1, *ks), np.float32)
    p["dw_conv.bias"] = np.zeros((C,), np.float32)
    p["offset_net.0.weight"] = np.zeros((C, 1, 3, 3, 3), np.float32)
    p["offset_net.0.bias"] = np.zeros((C,), np.float32)
    p["offset_net.2.weight"] = np.zeros((nh * 3 * 3, C, 1, 1, 1), np.float32)
    p["offset_net.2.bias"] = np.zeros((nh * 3 * 3,), np.float32)
    x = np.zeros((1, 2, 2), np.float32)
    x[:, 1, :] = [3.0, -2.0]
    dy = np.ones((1, 2, 2), np.float32)
    return dict(params=p, x=x, dy=dy, extra=None, video_shape=(2, 1, 1), heads=nh, kernel=ks, offset_scale=1.0)


def run_reference(ref_cls, torch, inp):
    C = inp["x"].shape[-1]
    m = ref_cls(hidden_size=C, num_heads=inp["heads"], kernel_size=tuple(inp["kernel"]),
                offset_scale=inp["offset_scale"], dropout=0.0)
    sd = {k: torch.from_numpy(v.copy()) for k, v in inp["params"].items()}
    m.load_state_dict(sd)
    offsets = {}

    def hook(_mod, _inp, out):
        B, O = out.shape[:2]
        offsets["raw"] = out.detach().reshape(B, O, -1).transpose(1, 2).contiguous().numpy()

    m.offset_net.register_forward_hook(hook)
    x = torch.from_numpy(inp["x"].copy()).requires_grad_(True)
    extra = None
    if inp["extra"] is not None:
        extra = torch.from_numpy(inp["extra"].copy()).requires_grad_(True)
    y = m(x, tuple(inp["video_shape"]), extra_kv=extra)
    (y * torch.from_numpy(inp["dy"])).sum().backward()
    out = dict(y=y.detach().numpy(), dx=x.grad.numpy(), offsets=offsets["raw"])
    for k, v in m.named_parameters():
        # parameters the graph does not reach (offset net when T=H=W=1) get no .grad
        out["grad." + k] = np.zeros(tuple(v.shape), np.float32) if v.grad is None else v.grad.numpy().copy()
    if extra is not None:
        out["d_extra"] = extra.grad.numpy()
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the jasonliu0704/megaslide checkout")
    ap.add_argument("--only", default=None)
    args = ap.parse_args(argv)
    sys.path.insert(0, args.reference)
    import torch

    torch.set_num_threads(8)
    from infinity.video.attention import DeformableSlideAttention3D as Ref

    names = list(CASES) + ["noncausal_211"]
    if args.only:
        names = [n for n in names if n == args.only]
    for name in names:
        inp = noncausal_inputs() if name == "noncausal_211" else make_inputs(name)
        res = run_reference(Ref, torch, inp)
        meta = dict(video_shape=np.array(inp["video_shape"]), heads=np.array(inp["heads"]),
                    kernel=np.array(inp["kernel"]), offset_scale=np.array(inp["offset_scale"]))
        arrays = {}
        if name == "c1_full":
            # inputs regenerate from the seed; keep selected rows of the big outputs
            rng = np.random.default_rng(99)
            rows = np.sort(rng.choice(inp["x"].shape[1], size=C1_ROWS, replace=False))
            arrays["rows"] = rows
            arrays["y_rows"] = res["y"][:, rows]
            arrays["dx_rows"] = res["dx"][:, rows]
            arrays["offsets_rows"] = res["offsets"][:, rows]
            for k, v in res.items():
                if k.startswith("grad.") and v.size <= 300_000:
                    arrays[k] = v
                elif k.startswith("grad."):
                    step = -(-v.shape[0] // 48)
                    arrays[k + ".rowstep"] = np.array(step)
                    arrays[k + ".rows"] = v.reshape(v.shape[0], -1)[::step]
            arrays["regenerate"] = np.array(1)
        else:
            arrays.update({"in." + k: v for k, v in inp["params"].items()})
            arrays["in.x"] = inp["x"]
            arrays["in.dy"] = inp["dy"]
            if inp["extra"] is not None:
                arrays["in.extra"] = inp["extra"]
            res = dict(res)
            off = res.pop("offsets")
            if off.size > 60_000:  # keep every few rows of large raw-offset tensors
                step = -(-off.shape[1] // 24)
                arrays["offsets_rows"] = np.arange(0, off.shape[1], step)
                off = off[:, ::step]
            arrays["offsets"] = off
            arrays.update(res)
            arrays["regenerate"] = np.array(0)
        out = HERE / f"{name}.npz"
        np.savez_compressed(out, **meta, **arrays)
        print(f"{name}: {out.stat().st_size / 1024:.0f} KiB")


if __name__ == "__main__":
    main()
