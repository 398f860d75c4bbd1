"""The C ABI library: it loads, exports exactly what include/megaslide_b200.h declares, its struct
layouts match the ctypes mirrors, and argument validation fails cleanly before any CUDA call."""

import ctypes
import re
import shutil
import subprocess
from pathlib import Path

import pytest

from megaslide_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "megaslide_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(msl_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_reports_version():
    lib = _lib.load()
    assert lib.msl_abi_version() == 4
    assert _lib.launch_count() >= 0


def test_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 10
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(_lib.SIGNATURES), set(names) ^ set(_lib.SIGNATURES)
    nm = shutil.which("nm")
    if nm:
        out = subprocess.run([nm, "-D", "--defined-only", str(_lib.library_path())], capture_output=True,
                             text=True, check=True).stdout
        exported = set(re.findall(r"\bT (msl_\w+)", out))
        assert set(names) <= exported


STRUCTS = {
    "msl_dsa_geometry": _lib.DsaGeometry,
    "msl_dsa_fwd_io": _lib.DsaFwdIO,
    "msl_dsa_bwd_io": _lib.DsaBwdIO,
    "msl_dwconv_geometry": _lib.DwconvGeometry,
}


def test_struct_layouts_match_header(tmp_path):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void) {"]
    for cname, py in STRUCTS.items():
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run([cc, str(src), "-o", str(exe)], check=True)
    got = {}
    for line in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.splitlines():
        s, f, v = line.split()
        got[(s, f)] = int(v)
    for cname, py in STRUCTS.items():
        assert got[(cname, "size")] == ctypes.sizeof(py), cname
        for fname, _ in py._fields_:
            assert got[(cname, fname)] == getattr(py, fname).offset, (cname, fname)


def _geom(**kw):
    base = dict(batch=1, frames=4, height=5, width=6, heads=2, head_dim=8, kt=3, kh=3, kw=3, extra=0, q_frame0=0,
                q_frames=4, kv_frame0=0, kv_frames=4, dtype=0, softmax_scale=0.35, offset_scale=1.0, dropout_p=0.0,
                dropout_seed=0)
    base.update(kw)
    return _lib.DsaGeometry(**base)


def _err():
    return _lib.load().msl_last_error().decode()


def test_validation_rejects_bad_geometry_without_touching_cuda():
    lib = _lib.load()
    assert lib.msl_dsa_attn_fwd(None, None, None) == _lib.MSL_ERR_INVALID
    assert "geometry" in _err()
    g = _geom(kh=4)
    assert lib.msl_dsa_attn_fwd(ctypes.byref(g), None, None) == _lib.MSL_ERR_INVALID
    assert "odd" in _err()
    g = _geom(q_frame0=2, q_frames=3)
    assert lib.msl_dsa_attn_fwd(ctypes.byref(g), None, None) == _lib.MSL_ERR_INVALID
    g = _geom(dropout_p=1.0)
    assert lib.msl_dsa_attn_fwd(ctypes.byref(g), None, None) == _lib.MSL_ERR_INVALID
    g = _geom(dtype=7)
    assert lib.msl_dsa_attn_fwd(ctypes.byref(g), None, None) == _lib.MSL_ERR_INVALID
    g = _geom()
    io = _lib.DsaFwdIO()
    assert lib.msl_dsa_attn_fwd(ctypes.byref(g), ctypes.byref(io), None) == _lib.MSL_ERR_INVALID
    assert "required" in _err()
    # head_dim beyond the register budget
    g = _geom(head_dim=136, heads=1)
    io = _lib.DsaFwdIO(q=16, q_ld=136, k=16, k_ld=136, v=16, v_ld=136, offsets=16, off_ld=81, out=16, out_ld=136,
                       lse=16)
    assert lib.msl_dsa_attn_fwd(ctypes.byref(g), ctypes.byref(io), None) == _lib.MSL_ERR_UNSUPPORTED


def test_workspace_size_formula():
    lib = _lib.load()
    g = _geom()
    C = 16
    rows = 1 * 4 * 5 * 6
    plane = -(-(4 * rows * C) // 256) * 256
    assert lib.msl_dsa_attn_bwd_workspace_bytes(ctypes.byref(g), 0) == 2 * plane
    assert lib.msl_dsa_attn_bwd_workspace_bytes(ctypes.byref(g), 1) == 0
    g = _geom(extra=3)
    xs = -(-(4 * 1 * 2 * rows * 3) // 256) * 256
    assert lib.msl_dsa_attn_bwd_workspace_bytes(ctypes.byref(g), 1) == 2 * xs
    assert lib.msl_dsa_attn_bwd_workspace_bytes(None, 0) == 0


def test_bwd_requires_workspace():
    lib = _lib.load()
    g = _geom()
    io = _lib.DsaBwdIO(q=16, q_ld=16, k=16, k_ld=16, v=16, v_ld=16, offsets=16, off_ld=162, out=16, out_ld=16,
                       lse=16, dout=16, dout_ld=16, dq=16, dq_ld=16, dk=16, dv=16, dkv_ld=16, doffsets=16,
                       doff_ld=162)
    assert lib.msl_dsa_attn_bwd(ctypes.byref(g), ctypes.byref(io), None, 0, None) == _lib.MSL_ERR_WORKSPACE


def test_dwconv_halo_coverage_is_checked():
    lib = _lib.load()
    g = _lib.DwconvGeometry(1, 8, 4, 4, 16, 3, 3, 3, 2, 3, 2, 3, 0)  # input frames [2,5) for outputs [2,5)
    rc = lib.msl_dwconv3d_fwd(ctypes.byref(g), 16, 16, 16, None, None, 0, None, 0, 16, 16, 0, None)
    assert rc == _lib.MSL_ERR_INVALID and "cover" in _err()
    g = _lib.DwconvGeometry(1, 4, 4, 4, 16, 3, 3, 3, 0, 4, 0, 4, 0)
    rc = lib.msl_dwconv3d_fwd(ctypes.byref(g), 16, 16, 16, None, None, 9, None, 0, 16, 16, 0, None)
    assert rc == _lib.MSL_ERR_INVALID and "epilogue" in _err()


def test_noalloc_capacity_matches_header():
    """The ctypes mirror of MSL_NOALLOC_SCRATCH_BYTES equals the header's #define."""
    m = re.search(r"#define\s+MSL_NOALLOC_SCRATCH_BYTES\s+\(([^)]*)\)", HEADER.read_text())
    assert m, "MSL_NOALLOC_SCRATCH_BYTES not found in the header"
    value = eval(m.group(1).replace("u", ""), {"__builtins__": {}})  # e.g. 64u * 1024u * 1024u
    assert value == _lib.MSL_NOALLOC_SCRATCH_BYTES
