"""bench.py's accounting, on the CPU: the algorithmic bytes per decode token
that roofline fractions divide by, and the launch count it reports.

The per-token bytes at position 0 must equal the figures derived from the
synthetic layouts (0.392 / 4.377 / 8.577 GB for the 0.5B / 7B / 14B shapes):
every weight matrix once, one embedding row, norms and biases.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402
from myllm_b200 import synth_gguf as sg  # noqa: E402


@pytest.mark.parametrize("name,gb", [("qwen2.5-0.5b", 0.392), ("qwen2.5-7b", 4.377), ("qwen2.5-14b", 8.577)])
def test_decode_bytes_per_token_at_position_zero(name, gb):
    spec = sg.CONFIGS[name]
    # the figures are quoted to three decimals of a GB
    assert abs(bench.decode_bytes_per_token(spec, 0) / 1e9 - gb) <= 5e-4


def test_decode_bytes_grow_by_the_kv_rows_read():
    spec = sg.CONFIGS["qwen2.5-7b"]
    kvd = spec.kv_heads * (spec.hidden // spec.heads)
    d = bench.decode_bytes_per_token(spec, 100) - bench.decode_bytes_per_token(spec, 99)
    assert d == spec.layers * 2 * kvd * 4  # one more K row and V row per layer, FP32


def test_gemv_launch_count_groups_formats_and_fused_pairs():
    # a run of one format, or of a fused pair (Q4_K + Q6_K, Q5_0 + Q8_0), is one launch
    assert bench.gemv_launches([sg.Q4_K, sg.Q4_K, sg.Q6_K]) == 1
    assert bench.gemv_launches([sg.Q5_0, sg.Q5_0, sg.Q8_0]) == 1
    assert bench.gemv_launches([sg.Q4_K, sg.Q8_0]) == 2
    assert bench.gemv_launches([sg.Q4_K, sg.Q6_K, sg.Q8_0]) == 2
    # the 7B attention projections: one launch per layer
    spec = sg.CONFIGS["qwen2.5-7b"]
    for layer in range(spec.layers):
        assert bench.gemv_launches([spec.types(layer, t) for t in ("attn_q", "attn_k", "attn_v")]) == 1


def test_sweep_shapes_are_the_config1_shapes():
    assert (18944, 3584) in bench.SWEEP_SHAPES and (3584, 18944) in bench.SWEEP_SHAPES
    # K-quants skip K = 896 (not a multiple of their 256-element blocks)
    assert 896 % sg.BLOCK[sg.Q4_K][0] != 0
