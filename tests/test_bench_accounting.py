"""bench.py's roofline accounting on CPU: the algorithmic bytes per token (the op's boundary traffic)
and the bytes each entry point of this build moves, at the config-2 and config-4 widths, equal the
figures the profiles and the design notes quote."""

import importlib.util
import json
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_op_bytes_per_token(bench):
    # c2: C = 1152, 16 heads, bf16 -> fwd 5 C es + 4 nh, bwd 6 C es + 4 nh, op 22 C + 8 nh
    b = bench._op_bytes_per_token(1152, 16, 2)
    assert b["msl_dsa_attn_fwd"] == 11584
    assert b["msl_dsa_attn_bwd"] == 13888
    assert b["op"] == 22 * 1152 + 8 * 16
    b4 = bench._op_bytes_per_token(1536, 24, 2)
    assert b4["msl_dsa_attn_bwd"] == 18528


@pytest.mark.parametrize("C,nh,fwd,bwd", [(1152, 16, 65728, 60832), (1536, 24, 97056, 88176)])
def test_kernel_io_bytes_per_token(bench, C, nh, fwd, bwd):
    K = 3 * 7 * 7
    assert bench._kernel_io_bytes_per_token("msl_dsa_attn_fwd", C, nh, K, 2, probs=True) == fwd
    assert bench._kernel_io_bytes_per_token("msl_dsa_attn_bwd", C, nh, K, 2, probs=True) == bwd
    # without the tensor-core records the forward drops probs + records, the backward reads the offsets
    assert bench._kernel_io_bytes_per_token("msl_dsa_attn_fwd", C, nh, K, 2) == fwd - 12 * nh * K


def test_traffic_table_names_its_capture(bench):
    t = json.loads((ROOT / "profiles" / "traffic.json").read_text())
    for entry in ("msl_dsa_attn_fwd", "msl_dsa_attn_bwd"):
        for cfg, rec in t[entry].items():
            assert cfg in bench.CONFIGS, cfg
            assert rec["measured_on"] in bench.CONFIGS
            assert rec["bytes_per_token"] > 0
        # c2 is taken from the capture that keeps its sample spread (same T and W)
        src = bench.CONFIGS[t[entry]["c2"]["measured_on"]]
        assert (src["T"], src["W"]) == (bench.CONFIGS["c2"]["T"], bench.CONFIGS["c2"]["W"])
