"""Torch-tensor wrappers over the C ABI (include/megaslide_b200.h).

Each function takes CUDA tensors, checks shapes / dtypes / devices on the host, passes raw
pointers, row strides and the current CUDA stream to libmegaslide_b200.so, and raises
``MslError`` (a RuntimeError) on any error code.  Nothing here computes on the CPU.
"""

from __future__ import annotations

import ctypes
import math
from contextlib import contextmanager
from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch

from . import _lib
from ._lib import DsaBwdIO, DsaFwdIO, DsaGeometry, DwconvGeometry

_DTYPES = {torch.float32: _lib.MSL_DTYPE_F32, torch.bfloat16: _lib.MSL_DTYPE_BF16}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPES[dt]
    except KeyError:
        raise TypeError(f"megaslide_b200 supports float32 and bfloat16 activations, got {dt}") from None


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _rows(t: torch.Tensor, name: str) -> int:
    """Row stride (elements) of a [rows, cols] matrix view with unit column stride."""
    if t.dim() != 2 or (t.stride(1) != 1 and t.size(1) > 1):
        raise ValueError(f"{name} must be a row-major 2-D view, got shape {tuple(t.shape)} strides {t.stride()}")
    return t.stride(0) if t.size(0) > 1 else max(t.stride(0), t.size(1))


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


_TIMER: Optional[List] = None


@contextmanager
def kernel_timer():
    """Records a (entry point name, start event, end event) triple around every C-ABI call made
    inside the block, on the stream the kernels are launched on.  Used by bench.py to time the
    kernels live (synchronise before reading the events)."""
    global _TIMER
    prev, _TIMER = _TIMER, []
    try:
        yield _TIMER
    finally:
        _TIMER = prev


def _call(name: str, dev: torch.device, fn):
    if _TIMER is None:
        return fn()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream(dev)
    s.record(stream)
    rc = fn()
    e.record(stream)
    _TIMER.append((name, s, e))
    return rc


class StatusWord:
    """The per-device status word the attention kernels OR their MSL_STATUS_* bits into (device int32),
    read back without stalling the host: after every call an asynchronous copy into pinned memory is
    enqueued with an event, and the next call (poll) reads that copy once its event has completed.  A
    halo miss or a timed-out TMA wait (results not valid) raises MslError there, at most one call late;
    check() reads the word synchronously.  MSL_STATUS_TC_RANGE is informational (the kernels computed
    such tiles with the CUDA-core gather)."""

    BAD = _lib.MSL_STATUS_HALO_MISS | _lib.MSL_STATUS_TIMEOUT

    def __init__(self, device: torch.device):
        self.word = torch.zeros(1, dtype=torch.int32, device=device)
        self.host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.event: Optional[torch.cuda.Event] = None
        self.seen = 0  # every bit observed so far (TC_RANGE included)

    def post(self) -> None:
        with torch.cuda.device(self.word.device):
            self.host.copy_(self.word, non_blocking=True)
            self.event = torch.cuda.Event()
            self.event.record()

    def _raise_if_bad(self, v: int) -> None:
        self.seen |= v
        if v & self.BAD:
            self.word.zero_()
            what = []
            if v & _lib.MSL_STATUS_HALO_MISS:
                what.append("a sample corner fell outside the K/V frames the call was given (halo miss)")
            if v & _lib.MSL_STATUS_TIMEOUT:
                what.append("a tensor-core CTA's TMA copies did not complete within a second")
            raise _lib.MslError("msl_dsa_attn", _lib.MSL_ERR_CUDA,
                                "a previous attention call produced invalid results: " + "; ".join(what))

    def poll(self) -> None:
        if self.event is not None and self.event.query():
            self.event = None
            self._raise_if_bad(int(self.host[0]))

    def check(self) -> int:
        """Synchronous: raises on a bad bit (and clears the word), else returns the word's bits
        (MSL_STATUS_TC_RANGE once a tile took the CUDA-core fallback)."""
        self.event = None
        v = int(self.word.item())
        self._raise_if_bad(v)
        return v


_STATUS: dict = {}


def status_word(device: torch.device) -> StatusWord:
    """The process-wide StatusWord of a CUDA device."""
    key = torch.device(device).index if torch.device(device).index is not None else torch.cuda.current_device()
    sw = _STATUS.get(key)
    if sw is None:
        sw = _STATUS[key] = StatusWord(torch.device("cuda", key))
    return sw


def check_status(device=None) -> int:
    """Synchronously checks the attention kernels' status word of `device` (default: current): raises
    MslError if a call produced invalid results, else returns the informational bits seen so far."""
    return status_word(device if device is not None else torch.device("cuda", torch.cuda.current_device())).check()


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("megaslide_b200 operands must be CUDA tensors (no CPU fallback)")


@dataclass(frozen=True)
class DsaShape:
    """Geometry of one deformable-attention call (mirrors ``msl_dsa_geometry``)."""

    batch: int
    frames: int
    height: int
    width: int
    heads: int
    head_dim: int
    kernel: Tuple[int, int, int]
    extra: int = 0
    q_frame0: int = 0
    q_frames: Optional[int] = None
    kv_frame0: int = 0
    kv_frames: Optional[int] = None
    softmax_scale: Optional[float] = None
    offset_scale: float = 1.0
    dropout_p: float = 0.0
    dropout_seed: int = 0
    algo: int = 0  # 0 auto, 1 CUDA-core gather, 2 tensor-core envelope

    @property
    def taps(self) -> int:
        return self.kernel[0] * self.kernel[1] * self.kernel[2]

    @property
    def q_rows(self) -> int:
        return (self.q_frames if self.q_frames is not None else self.frames) * self.height * self.width

    @property
    def kv_rows(self) -> int:
        return (self.kv_frames if self.kv_frames is not None else self.frames) * self.height * self.width

    def geometry(self, dtype: torch.dtype) -> DsaGeometry:
        kt, kh, kw = self.kernel
        scale = self.softmax_scale if self.softmax_scale is not None else 1.0 / math.sqrt(self.head_dim)
        return DsaGeometry(
            self.batch, self.frames, self.height, self.width, self.heads, self.head_dim, kt, kh, kw, self.extra,
            self.q_frame0, self.q_frames if self.q_frames is not None else self.frames,
            self.kv_frame0, self.kv_frames if self.kv_frames is not None else self.frames,
            dtype_code(dtype), float(scale), float(self.offset_scale), float(self.dropout_p),
            int(self.dropout_seed) & 0xFFFFFFFFFFFFFFFF, int(self.algo))


def wants_probs(shape: DsaShape, dtype: torch.dtype) -> bool:
    """Host-side pre-check for the tensor-core backward, which needs two outputs of the tensor-core
    forward (``probs``, ``saved``): bf16, at most 256 extra keys, head_dim a multiple of 8 in [16, 128],
    algo not forced to the CUDA-core gather.  The library makes the final decision (alignment,
    shared-memory plan)."""
    return (dtype == torch.bfloat16 and shape.extra <= 256 and shape.algo != _lib.MSL_ALGO_SIMT
            and shape.head_dim % 8 == 0 and 16 <= shape.head_dim <= 128)


def probs_buffer(shape: DsaShape, device) -> torch.Tensor:
    """float32 [B, nh, q_rows, K] buffer for the forward's per-sample softmax weights."""
    return torch.empty(shape.batch, shape.heads, shape.q_rows, shape.taps, device=device, dtype=torch.float32)


def saved_buffer(shape: DsaShape, dtype: torch.dtype, device) -> torch.Tensor:
    """uint8 buffer (msl_dsa_saved_bytes) for the tensor-core forward's per-sample records and tile
    envelopes, which the tensor-core backward reads instead of recomputing the sample coordinates."""
    g = shape.geometry(dtype)
    n = int(_lib.load().msl_dsa_saved_bytes(ctypes.byref(g)))
    if n <= 0:
        raise ValueError("invalid geometry for the saved buffer")
    return torch.empty(n, device=device, dtype=torch.uint8)


def saved_buffers(shape: DsaShape, dtype: torch.dtype, device) -> Tuple[torch.Tensor, torch.Tensor]:
    """(probs, saved): the tensor-core forward's outputs that the tensor-core backward needs."""
    return probs_buffer(shape, device), saved_buffer(shape, dtype, device)


def _check_saved(shape: DsaShape, dtype: torch.dtype, saved: torch.Tensor) -> None:
    g = shape.geometry(dtype)
    n = int(_lib.load().msl_dsa_saved_bytes(ctypes.byref(g)))
    if saved.dtype != torch.uint8 or saved.numel() < n or not saved.is_contiguous():
        raise ValueError(f"saved must be a contiguous uint8 tensor of at least {n} bytes (saved_buffer)")


def _check_probs(shape: DsaShape, probs: torch.Tensor) -> None:
    want = (shape.batch, shape.heads, shape.q_rows, shape.taps)
    if probs.dtype != torch.float32 or tuple(probs.shape) != want or not probs.is_contiguous():
        raise ValueError(f"probs must be a contiguous float32 tensor of shape {want}")


def _check_offset_bias(bias: Optional[torch.Tensor], n: int) -> None:
    if bias is not None and (bias.dtype != torch.float32 or bias.numel() != n or not bias.is_contiguous()):
        raise ValueError(f"offset_bias must be a contiguous float32 tensor of {n} elements")


def attn_fwd(shape: DsaShape, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, offsets: torch.Tensor,
             ek: Optional[torch.Tensor] = None, ev: Optional[torch.Tensor] = None,
             out: Optional[torch.Tensor] = None, lse: Optional[torch.Tensor] = None,
             status: Optional[torch.Tensor] = None,
             probs: Optional[torch.Tensor] = None,
             saved: Optional[torch.Tensor] = None,
             offset_bias: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Deformable gather attention forward.

    q: [B*q_rows, >=C] row view; k, v: [B*kv_rows, >=C]; offsets: float32 [B*q_rows, >=nh*K*3];
    ek, ev: [B*G, >=C] or None.  Returns (out [B*q_rows, C], lse float32 [B, nh, q_rows]).
    probs, saved (optional, see saved_buffers): filled with the per-sample softmax weights and the
    per-sample records for the tensor-core backward; the call raises MslError(MSL_ERR_UNSUPPORTED)
    when the tensor-core forward does not apply to these operands.  offset_bias (float32 [nh*K*3]):
    added to every offsets row before use (offsets + bias, one float32 rounding).
    """
    _need_cuda(q, k, v, offsets, ek, ev, offset_bias)
    _check_offset_bias(offset_bias, shape.heads * shape.taps * 3)
    C = shape.heads * shape.head_dim
    dt = q.dtype
    if offsets.dtype != torch.float32:
        raise TypeError("offsets must be float32")
    if out is None:
        out = torch.empty(shape.batch * shape.q_rows, C, device=q.device, dtype=dt)
    if lse is None:
        lse = torch.empty(shape.batch, shape.heads, shape.q_rows, device=q.device, dtype=torch.float32)
    io = DsaFwdIO(_ptr(q), _rows(q, "q"), _ptr(k), _rows(k, "k"), _ptr(v), _rows(v, "v"),
                  _ptr(offsets), _rows(offsets, "offsets"), _ptr(ek), _ptr(ev),
                  _rows(ek, "ek") if ek is not None else 0, _ptr(out), _rows(out, "out"), _ptr(lse), _ptr(status))
    if probs is not None:
        _need_cuda(probs)
        _check_probs(shape, probs)
        io.probs = _ptr(probs)
    if saved is not None:
        _need_cuda(saved)
        _check_saved(shape, dt, saved)
        io.saved = _ptr(saved)
    io.offset_bias = _ptr(offset_bias)
    g = shape.geometry(dt)
    with torch.cuda.device(q.device):
        rc = _call("msl_dsa_attn_fwd", q.device,
                   lambda: _lib.load().msl_dsa_attn_fwd(ctypes.byref(g), ctypes.byref(io), _stream(q.device)))
    _lib.check("msl_dsa_attn_fwd", rc)
    return out, lse


def attn_bwd(shape: DsaShape, q, k, v, offsets, out, lse, dout, *, ek=None, ev=None, dq=None, dk=None, dv=None,
             dk_acc=None, dv_acc=None, doffsets=None, dek=None, dev=None, workspace=None, status=None, probs=None,
             saved=None, doff_dtype=torch.float32, offset_bias=None):
    """Deformable gather attention backward.

    Without dk_acc: dK/dV are written to dk/dv (allocated if None) in q's dtype, float32
    accumulators live in ``workspace`` (allocated if None).  With dk_acc/dv_acc (float32 views):
    dK/dV are ACCUMULATED there.  Returns (dq, dk, dv, doffsets, dek, dev); dk/dv are the
    accumulators in accumulate mode.  probs, saved: the tensor-core forward's outputs for these operands
    (attn_fwd(probs=..., saved=...)); with both, the tensor-core backward runs where it applies.
    doffsets (or doff_dtype when it is allocated here) is float32 or bf16 (the float32 gradient rounded
    to nearest even).  offset_bias: the forward's.
    """
    _need_cuda(q, k, v, offsets, out, lse, dout, ek, ev, offset_bias)
    _check_offset_bias(offset_bias, shape.heads * shape.taps * 3)
    C = shape.heads * shape.head_dim
    dt = q.dtype
    dev_ = q.device
    rows_q = shape.batch * shape.q_rows
    rows_kv = shape.batch * shape.kv_rows
    if dq is None:
        dq = torch.empty(rows_q, C, device=dev_, dtype=dt)
    accumulate = dk_acc is not None
    if not accumulate:
        if dk is None:
            dk = torch.empty(rows_kv, C, device=dev_, dtype=dt)
        if dv is None:
            dv = torch.empty(rows_kv, C, device=dev_, dtype=dt)
    if doffsets is None:
        doffsets = torch.empty(rows_q, shape.heads * shape.taps * 3, device=dev_, dtype=doff_dtype)
    if doffsets.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError("doffsets must be float32 or bfloat16")
    if shape.extra > 0:
        if dek is None:
            dek = torch.empty(shape.batch * shape.extra, C, device=dev_, dtype=torch.float32)
        if dev is None:
            dev = torch.empty(shape.batch * shape.extra, C, device=dev_, dtype=torch.float32)
    g = shape.geometry(dt)
    lib = _lib.load()
    need = int(lib.msl_dsa_attn_bwd_workspace_bytes(ctypes.byref(g), 1 if accumulate else 0))
    if need and (workspace is None or workspace.numel() < need):
        workspace = torch.empty(need, device=dev_, dtype=torch.uint8)
    io = DsaBwdIO(
        _ptr(q), _rows(q, "q"), _ptr(k), _rows(k, "k"), _ptr(v), _rows(v, "v"),
        _ptr(offsets), _rows(offsets, "offsets"), _ptr(ek), _ptr(ev), _rows(ek, "ek") if ek is not None else 0,
        _ptr(out), _rows(out, "out"), _ptr(lse), _ptr(dout), _rows(dout, "dout"),
        _ptr(dq), _rows(dq, "dq"),
        None if accumulate else _ptr(dk), None if accumulate else _ptr(dv),
        0 if accumulate else _rows(dk, "dk"),
        _ptr(dk_acc), _ptr(dv_acc), _rows(dk_acc, "dk_acc") if accumulate else 0,
        _ptr(doffsets), _rows(doffsets, "doffsets"), _ptr(dek), _ptr(dev), _ptr(status))
    io.doff_dtype = dtype_code(doffsets.dtype)
    io.offset_bias = _ptr(offset_bias)
    if probs is not None:
        _need_cuda(probs)
        _check_probs(shape, probs)
        io.probs = _ptr(probs)
    if saved is not None:
        _need_cuda(saved)
        _check_saved(shape, dt, saved)
        io.saved = _ptr(saved)
    with torch.cuda.device(dev_):
        rc = _call("msl_dsa_attn_bwd", dev_,
                   lambda: lib.msl_dsa_attn_bwd(ctypes.byref(g), ctypes.byref(io), _ptr(workspace) if need else None,
                                                need, _stream(dev_)))
    _lib.check("msl_dsa_attn_bwd", rc)
    if accumulate:
        dk, dv = dk_acc, dv_acc
    return dq, dk, dv, doffsets, dek, dev


@dataclass(frozen=True)
class ConvShape:
    """Geometry of a depthwise conv call (mirrors ``msl_dwconv_geometry``)."""

    batch: int
    frames: int
    height: int
    width: int
    channels: int
    kernel: Tuple[int, int, int]
    in_frame0: int = 0
    in_frames: Optional[int] = None
    out_frame0: int = 0
    out_frames: Optional[int] = None
    zero_outside: bool = False  # input frames outside the window read as zero (sharded adjoint)

    def geometry(self, dtype: torch.dtype) -> DwconvGeometry:
        kt, kh, kw = self.kernel
        return DwconvGeometry(self.batch, self.frames, self.height, self.width, self.channels, kt, kh, kw,
                              self.in_frame0, self.in_frames if self.in_frames is not None else self.frames,
                              self.out_frame0, self.out_frames if self.out_frames is not None else self.frames,
                              dtype_code(dtype), 1 if self.zero_outside else 0)

    @property
    def out_rows(self) -> int:
        return self.batch * (self.out_frames if self.out_frames is not None else self.frames) * self.height * self.width


def conv_weight_kc(w: torch.Tensor) -> torch.Tensor:
    """nn.Conv3d depthwise weight [C, 1, kt, kh, kw] -> float32 tap-major [kt*kh*kw, C]."""
    C = w.shape[0]
    return w.detach().reshape(C, -1).t().contiguous().float()


def dwconv_fwd(shape: ConvShape, x: torch.Tensor, weight_kc: torch.Tensor, bias: Optional[torch.Tensor] = None,
               bias2: Optional[torch.Tensor] = None, epilogue: int = _lib.MSL_EPI_NONE,
               aux: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
               out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """y = epilogue(depthwise_conv(x) + bias [+ bias2]); x/y [rows, >=C] row views.  y (and aux)
    have ``out_dtype`` (default: x's dtype)."""
    _need_cuda(x, weight_kc, bias, bias2, aux)
    for t, nm in ((weight_kc, "weight"), (bias, "bias"), (bias2, "bias2")):
        if t is not None and (t.dtype != torch.float32 or not t.is_contiguous()):
            raise TypeError(f"{nm} must be a contiguous float32 tensor")
    if out is None:
        out = torch.empty(shape.out_rows, shape.channels, device=x.device, dtype=out_dtype or x.dtype)
    if aux is not None and aux.dtype != out.dtype:
        raise TypeError("aux must have the output's dtype")
    g = shape.geometry(x.dtype)
    with torch.cuda.device(x.device):
        rc = _call("msl_dwconv3d_fwd", x.device, lambda: _lib.load().msl_dwconv3d_fwd(
            ctypes.byref(g), _ptr(x), _rows(x, "x"), _ptr(weight_kc), _ptr(bias), _ptr(bias2), int(epilogue),
            _ptr(aux), _rows(aux, "aux") if aux is not None else 0, _ptr(out), _rows(out, "y"),
            dtype_code(out.dtype), _stream(x.device)))
    _lib.check("msl_dwconv3d_fwd", rc)
    return out


def dwconv_bwd_data(shape: ConvShape, dy: torch.Tensor, weight_kc: torch.Tensor,
                    out: Optional[torch.Tensor] = None, accumulate: bool = False) -> torch.Tensor:
    """dx = conv_transpose(dy); the geometry's input window is dy's frames, output is dx's.
    accumulate=True adds into ``out`` (float32) instead: dx += conv_transpose(dy)."""
    _need_cuda(dy, weight_kc)
    if accumulate:
        if out is None or out.dtype != torch.float32:
            raise TypeError("accumulate=True needs a float32 out")
    elif out is None:
        out = torch.empty(shape.out_rows, shape.channels, device=dy.device, dtype=dy.dtype)
    g = shape.geometry(dy.dtype)
    name = "msl_dwconv3d_bwd_data_acc" if accumulate else "msl_dwconv3d_bwd_data"
    with torch.cuda.device(dy.device):
        rc = _call(name, dy.device, lambda: getattr(_lib.load(), name)(
            ctypes.byref(g), _ptr(dy), _rows(dy, "dy"), _ptr(weight_kc), _ptr(out), _rows(out, "dx"),
            _stream(dy.device)))
    _lib.check(name, rc)
    return out


def dwconv_bwd_weight(shape: ConvShape, dy: torch.Tensor, x: torch.Tensor, dweight_kc: torch.Tensor,
                      dbias: Optional[torch.Tensor] = None) -> None:
    """dweight_kc [K, C] += sum dy * shifted x ; dbias [C] += sum dy (float32, accumulated)."""
    _need_cuda(dy, x, dweight_kc, dbias)
    g = shape.geometry(x.dtype)
    with torch.cuda.device(dy.device):
        rc = _call("msl_dwconv3d_bwd_weight", dy.device, lambda: _lib.load().msl_dwconv3d_bwd_weight(
            ctypes.byref(g), _ptr(dy), _rows(dy, "dy"), dtype_code(dy.dtype), _ptr(x), _rows(x, "x"),
            _ptr(dweight_kc), _ptr(dbias), _stream(dy.device)))
    _lib.check("msl_dwconv3d_bwd_weight", rc)


def offsets_absmax(offsets: torch.Tensor, heads: int, taps: int, offset_scale: float = 1.0,
                   out: Optional[torch.Tensor] = None, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Per-axis max |(offset + bias) * offset_scale| -> float32[3] on the device (channel 0, 1, 2)."""
    _need_cuda(offsets, bias)
    _check_offset_bias(bias, heads * taps * 3)
    if out is None:
        out = torch.zeros(3, device=offsets.device, dtype=torch.float32)
    with torch.cuda.device(offsets.device):
        rc = _lib.load().msl_offsets_absmax(_ptr(offsets), offsets.shape[0], _rows(offsets, "offsets"), _ptr(bias),
                                            heads, taps,
                                            float(offset_scale), _ptr(out), _stream(offsets.device))
    _lib.check("msl_offsets_absmax", rc)
    return out


def convert_f32(src: torch.Tensor, dst: torch.Tensor) -> torch.Tensor:
    _need_cuda(src, dst)
    with torch.cuda.device(src.device):
        rc = _lib.load().msl_convert_f32(_ptr(src), _rows(src, "src"), _ptr(dst), _rows(dst, "dst"),
                                         dtype_code(dst.dtype), src.shape[0], src.shape[1], _stream(src.device))
    _lib.check("msl_convert_f32", rc)
    return dst
