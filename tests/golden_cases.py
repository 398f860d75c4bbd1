"""Loads the golden fixtures of tests/golden (made by tests/golden/make_golden.py from the
reference module) and runs the CPU oracle on the same inputs."""

from __future__ import annotations

import importlib.util
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"
NAMES = sorted(p.stem for p in GOLDEN.glob("*.npz"))


def _make_golden():
    spec = importlib.util.spec_from_file_location("make_golden", GOLDEN / "make_golden.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def load(name: str) -> dict:
    """Fixture as a dict with keys: params, x, dy, extra, video_shape, heads, kernel, offset_scale and
    the reference outputs (y / dx / grad.* / offsets, or their stored row subsets)."""
    z = np.load(GOLDEN / f"{name}.npz")
    f = {k: z[k] for k in z.files}
    case = dict(video_shape=tuple(int(v) for v in f["video_shape"]), heads=int(f["heads"]),
                kernel=tuple(int(v) for v in f["kernel"]), offset_scale=float(f["offset_scale"]),
                regenerate=bool(int(f["regenerate"])), ref=f)
    if case["regenerate"]:
        inp = _make_golden().make_inputs(name)
        case.update(params=inp["params"], x=inp["x"], dy=inp["dy"], extra=inp["extra"])
    else:
        case.update(params={k[3:]: v for k, v in f.items() if k.startswith("in.") and "." in k[3:]},
                    x=f["in.x"], dy=f["in.dy"], extra=f.get("in.extra"))
    return case


def run_oracle(case: dict):
    from oracle import dsa_oracle as O

    y, cache = O.module_forward(case["params"], case["x"], case["video_shape"], case["extra"],
                                heads=case["heads"], kernel_size=case["kernel"], offset_scale=case["offset_scale"])
    dx, grads, dextra = O.module_backward(cache, case["dy"])
    return dict(y=y, dx=dx, grads=grads, d_extra=dextra, offsets=cache["off32"])


def rel_err(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def _grad_err(name: str, a: np.ndarray, b: np.ndarray, ref_grads: dict) -> float:
    """Relative error of one gradient tensor.

    A tensor that is zero in exact arithmetic (|ref| below 1e-6 of the case's largest gradient:
    k_proj.bias always — a key bias shifts every score of a query equally and the trilinear
    weights sum to 1 — and the q/k gradients when every sample of a query coincides, T=H=W=1)
    holds only rounding noise on both sides, so its error is our magnitude over that largest
    gradient.  Otherwise: max |a - b| / max |b|."""
    a = np.asarray(a, np.float64)
    g = max(float(np.abs(v).max()) for v in ref_grads.values())
    mb = float(np.abs(b).max())
    if mb <= 1e-6 * g:
        return float(np.abs(a).max() / max(g, 1e-30))
    return float(np.abs(a - b).max() / mb)


def case_errors(res: dict, case: dict) -> dict:
    """Relative errors of a result dict (y, dx, grads, d_extra, offsets) against the fixture."""
    ref = case["ref"]
    errs = {}
    if case["regenerate"]:
        rows = ref["rows"]
        errs["y"] = rel_err(np.asarray(res["y"])[:, rows], ref["y_rows"])
        errs["dx"] = rel_err(np.asarray(res["dx"])[:, rows], ref["dx_rows"])
        if res.get("offsets") is not None:
            errs["offsets"] = rel_err(np.asarray(res["offsets"])[:, rows], ref["offsets_rows"])
    else:
        errs["y"] = rel_err(res["y"], ref["y"])
        errs["dx"] = rel_err(res["dx"], ref["dx"])
        if res.get("offsets") is not None:
            off = np.asarray(res["offsets"])
            if "offsets_rows" in ref:
                off = off[:, ref["offsets_rows"]]
            errs["offsets"] = float(np.abs(off - ref["offsets"]).max() / max(np.abs(ref["offsets"]).max(), 1e-3))
        if "d_extra" in ref:
            errs["d_extra"] = rel_err(res["d_extra"], ref["d_extra"])
    full = {k[5:]: v for k, v in ref.items() if k.startswith("grad.") and not k.endswith((".rows", ".rowstep"))}
    for k, b in full.items():
        errs["grad." + k] = _grad_err(k, res["grads"][k], b, full)
    for k, b in ref.items():
        if k.startswith("grad.") and k.endswith(".rows"):
            nm = k[5:-5]
            step = int(ref["grad." + nm + ".rowstep"])
            a = np.asarray(res["grads"][nm], np.float64)
            a = a.reshape(a.shape[0], -1)[::step]
            errs["grad." + nm] = float(np.abs(a - b).max() / max(float(np.abs(b).max()), 1e-30))
    return errs
