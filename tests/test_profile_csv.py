"""The profile CSV that CudaLLM / CudaMoeLLM write after enable_profiling,
against the reference Profiler's file for the same calls (CPU only).

Both writers get the same three calls (one prefill, two decode steps) with the
same logical metrics; the reference's Profiler is compiled from its own
sources (profiler.cpp) with a driver that opens one ForwardScope and one Scope
per call, as its GPU backends do.  Every column must agree except the wall
time and the rates derived from it; those are checked against their
definitions instead.
"""
import csv
import os
import shutil
import subprocess

import pytest

import oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HOST = os.path.join(ROOT, "myllm_b200", "csrc", "host")
TIMED = {"time_ms", "gflops", "logical_gbps", "estimated_gbps"}

pytestmark = pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")


def compile_and_run(sources, include, out_csv, tmp_path, name):
    exe = str(tmp_path / name)
    r = subprocess.run(["g++", "-std=c++17", "-O1", "-g", "-fsanitize=address,undefined", "-fno-sanitize-recover=all",
                        "-I", include] + sources + ["-o", exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    r = subprocess.run([exe, out_csv], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr[-2000:]
    with open(out_csv, newline="") as f:
        return list(csv.reader(f))


@pytest.fixture(scope="module")
def ours(tmp_path_factory):
    t = tmp_path_factory.mktemp("profile")
    return compile_and_run([os.path.join(ROOT, "tests", "native", "profile_check.cpp"),
                            os.path.join(HOST, "profile.cpp")], HOST, str(t / "ours.csv"), t, "ours")


def test_rows_and_derived_columns(ours):
    header, rows = ours[0], [dict(zip(ours[0], r)) for r in ours[1:]]
    assert len(header) == 19 and header[0] == "record_type" and header[-1] == "arithmetic_intensity_with_temporaries"
    kinds = [(r["record_type"], r["forward_index"], r["stage"]) for r in rows]
    assert kinds == [("forward_total", "0", "forward.total"), ("forward_stage", "0", "prefill.gpu_resident"),
                     ("forward_total", "1", "forward.total"), ("forward_stage", "1", "decode.gpu_resident"),
                     ("forward_total", "2", "forward.total"), ("forward_stage", "2", "decode.gpu_resident"),
                     ("global", "", "decode.gpu_resident"), ("global", "", "forward.total"),
                     ("global", "", "prefill.gpu_resident")]
    g = {r["stage"]: r for r in rows if r["record_type"] == "global"}
    assert g["decode.gpu_resident"]["calls"] == "2" and g["forward.total"]["calls"] == "3"
    assert g["decode.gpu_resident"]["time_ms"] == "2.500" and g["forward.total"]["time_ms"] == "5.000"
    assert int(g["decode.gpu_resident"]["flops"]) == 1_100_000_000
    for r in rows:
        read, write, tmp = int(r["read_bytes"]), int(r["write_bytes"]), int(r["temporary_bytes"])
        s = float(r["time_ms"]) / 1e3
        assert int(r["logical_bytes"]) == read + write and int(r["estimated_bytes_with_temporaries"]) == read + write + tmp
        assert float(r["gflops"]) == pytest.approx(int(r["flops"]) / s / 1e9, abs=1e-3)
        assert float(r["logical_gbps"]) == pytest.approx((read + write) / s / 1e9, abs=1e-3)
        assert float(r["arithmetic_intensity"]) == pytest.approx(int(r["flops"]) / (read + write), abs=1e-3)


@pytest.mark.skipif(not oracle.REFERENCE_SOURCES or not os.path.exists(os.path.join(oracle.REFERENCE_SOURCES, "profiler.cpp")),
                    reason="reference sources not present")
def test_matches_the_reference_profiler(ours, tmp_path):
    ref_dir = oracle.REFERENCE_SOURCES
    ref = compile_and_run([os.path.join(ROOT, "tests", "native", "ref_profile_check.cpp"),
                           os.path.join(ref_dir, "profiler.cpp")], ref_dir, str(tmp_path / "ref.csv"), tmp_path, "ref")
    assert ref[0] == ours[0]  # the header
    assert len(ref) == len(ours)
    for a, b in zip(ref[1:], ours[1:]):
        ra, rb = dict(zip(ref[0], a)), dict(zip(ours[0], b))
        for col in ref[0]:
            if col in TIMED or col.startswith("arithmetic_intensity"):
                continue
            assert ra[col] == rb[col], (col, ra, rb)
        for col in ("arithmetic_intensity", "arithmetic_intensity_with_temporaries"):
            assert ra[col] == rb[col], (col, ra, rb)
