"""ctypes binding of libmegaslide_b200.so (the C ABI declared in include/megaslide_b200.h).

The library is loaded from ``megaslide_b200/lib/`` (built in-tree by ``megaslide_b200.build``).
There is no fallback: if the library is missing or fails to load, every entry point raises.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "lib" / "libmegaslide_b200.so"
_lock = threading.Lock()
_lib = None

MSL_OK = 0
MSL_ERR_INVALID = -1
MSL_ERR_UNSUPPORTED = -2
MSL_ERR_CUDA = -3
MSL_ERR_WORKSPACE = -4
MSL_DTYPE_F32 = 0
MSL_DTYPE_BF16 = 1
MSL_STATUS_HALO_MISS = 1
MSL_STATUS_TC_RANGE = 2
MSL_STATUS_TIMEOUT = 4
MSL_ALGO_AUTO = 0
MSL_ALGO_SIMT = 1
MSL_ALGO_TC = 2
MSL_EPI_NONE = 0
MSL_EPI_GELU = 1
MSL_EPI_GELU_GRAD = 2
MSL_EPI_ACCUM = 3
MSL_NOALLOC_SCRATCH_BYTES = 64 * 1024 * 1024

_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_f32 = ctypes.c_float
_u64 = ctypes.c_uint64
_vp = ctypes.c_void_p


class DsaGeometry(ctypes.Structure):
    """Mirror of ``msl_dsa_geometry``."""

    _fields_ = [
        ("batch", _i32), ("frames", _i32), ("height", _i32), ("width", _i32),
        ("heads", _i32), ("head_dim", _i32), ("kt", _i32), ("kh", _i32), ("kw", _i32),
        ("extra", _i32), ("q_frame0", _i32), ("q_frames", _i32), ("kv_frame0", _i32), ("kv_frames", _i32),
        ("dtype", _i32), ("softmax_scale", _f32), ("offset_scale", _f32), ("dropout_p", _f32),
        ("dropout_seed", _u64), ("algo", _i32),
    ]


class DsaFwdIO(ctypes.Structure):
    """Mirror of ``msl_dsa_fwd_io``."""

    _fields_ = [
        ("q", _vp), ("q_ld", _i64), ("k", _vp), ("k_ld", _i64), ("v", _vp), ("v_ld", _i64),
        ("offsets", _vp), ("off_ld", _i64), ("ek", _vp), ("ev", _vp), ("e_ld", _i64),
        ("out", _vp), ("out_ld", _i64), ("lse", _vp), ("status", _vp), ("probs", _vp), ("saved", _vp),
        ("offset_bias", _vp),
    ]


class DsaBwdIO(ctypes.Structure):
    """Mirror of ``msl_dsa_bwd_io``."""

    _fields_ = [
        ("q", _vp), ("q_ld", _i64), ("k", _vp), ("k_ld", _i64), ("v", _vp), ("v_ld", _i64),
        ("offsets", _vp), ("off_ld", _i64), ("ek", _vp), ("ev", _vp), ("e_ld", _i64),
        ("out", _vp), ("out_ld", _i64), ("lse", _vp), ("dout", _vp), ("dout_ld", _i64),
        ("dq", _vp), ("dq_ld", _i64), ("dk", _vp), ("dv", _vp), ("dkv_ld", _i64),
        ("dk_acc", _vp), ("dv_acc", _vp), ("acc_ld", _i64),
        ("doffsets", _vp), ("doff_ld", _i64), ("dek", _vp), ("dev", _vp), ("status", _vp), ("probs", _vp),
        ("saved", _vp), ("doff_dtype", ctypes.c_int32), ("offset_bias", _vp),
    ]


class DwconvGeometry(ctypes.Structure):
    """Mirror of ``msl_dwconv_geometry``."""

    _fields_ = [
        ("batch", _i32), ("frames", _i32), ("height", _i32), ("width", _i32), ("channels", _i32),
        ("kt", _i32), ("kh", _i32), ("kw", _i32), ("in_frame0", _i32), ("in_frames", _i32),
        ("out_frame0", _i32), ("out_frames", _i32), ("dtype", _i32), ("zero_outside", _i32),
    ]


# name -> (restype, argtypes); the full exported surface of include/megaslide_b200.h
SIGNATURES = {
    "msl_dsa_attn_fwd": (ctypes.c_int, [ctypes.POINTER(DsaGeometry), ctypes.POINTER(DsaFwdIO), _vp]),
    "msl_dsa_attn_bwd_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(DsaGeometry), _i32]),
    "msl_dsa_saved_bytes": (ctypes.c_size_t, [ctypes.POINTER(DsaGeometry)]),
    "msl_dsa_attn_bwd": (ctypes.c_int, [ctypes.POINTER(DsaGeometry), ctypes.POINTER(DsaBwdIO), _vp,
                                        ctypes.c_size_t, _vp]),
    "msl_dsa_attn_bwd_noalloc": (ctypes.c_int, [ctypes.POINTER(DsaGeometry), ctypes.POINTER(DsaBwdIO), _vp]),
    "msl_dwconv3d_fwd": (ctypes.c_int, [ctypes.POINTER(DwconvGeometry), _vp, _i64, _vp, _vp, _vp, _i32, _vp,
                                        _i64, _vp, _i64, _i32, _vp]),
    "msl_dwconv3d_bwd_data": (ctypes.c_int, [ctypes.POINTER(DwconvGeometry), _vp, _i64, _vp, _vp, _i64, _vp]),
    "msl_dwconv3d_bwd_data_acc": (ctypes.c_int, [ctypes.POINTER(DwconvGeometry), _vp, _i64, _vp, _vp, _i64, _vp]),
    "msl_dwconv3d_bwd_weight": (ctypes.c_int, [ctypes.POINTER(DwconvGeometry), _vp, _i64, _i32, _vp, _i64, _vp,
                                               _vp, _vp]),
    "msl_offsets_absmax": (ctypes.c_int, [_vp, _i64, _i64, _vp, _i32, _i32, _f32, _vp, _vp]),
    "msl_convert_f32": (ctypes.c_int, [_vp, _i64, _vp, _i64, _i32, _i64, _i64, _vp]),
    "msl_host_accumulate": (ctypes.c_int, [_vp, _vp, _i32, _i64, _i32, ctypes.POINTER(ctypes.c_double)]),
    "msl_host_adamw": (ctypes.c_int, [_vp, _vp, _vp, _vp, _i64, _f32, _f32, _f32, _f32, _f32, _i64, _f32, _vp, _i32]),
    "msl_abi_version": (_i32, []),
    "msl_launch_count": (_u64, []),
    "msl_last_error": (ctypes.c_char_p, []),
}


class MslError(RuntimeError):
    """A libmegaslide_b200 entry point returned an error code."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed ({code}): {msg}")
        self.code = code


def library_path() -> Path:
    return _LIB_PATH


def load() -> ctypes.CDLL:
    """Loads the CUDA library once; raises if it is missing (there is no CPU fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            from . import build as _build

            if not _build.is_current():
                # missing, or built from other sources: rebuild from the present ones (nvcc, sm_100a) so a
                # stale binary never runs
                try:
                    _build.build()
                except Exception as e:
                    raise RuntimeError(
                        f"megaslide_b200 CUDA library at {_LIB_PATH} is missing or out of date and could not be "
                        f"built ({e}); build it with `python -m megaslide_b200.build` (nvcc, sm_100a). "
                        "There is no CPU fallback.") from e
            lib = ctypes.CDLL(str(_LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            if lib.msl_abi_version() != 4:
                raise RuntimeError("libmegaslide_b200 ABI version mismatch")
            _lib = lib
    return _lib


def check(fn: str, rc: int) -> None:
    if rc != MSL_OK:
        msg = load().msl_last_error().decode("utf-8", "replace")
        raise MslError(fn, rc, msg)


def launch_count() -> int:
    return int(load().msl_launch_count())
