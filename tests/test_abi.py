"""CPU tests of the C-ABI library: it loads, exports every declared symbol,
and its pure host queries agree with the GGUF block sizes."""
import os
import re

import pytest

from myllm_b200 import _native
from myllm_b200 import synth_gguf as sg

INCLUDE = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include")


def declared_symbols():
    names = []
    for fn in sorted(os.listdir(INCLUDE)):
        if not fn.endswith(".h"):
            continue
        text = open(os.path.join(INCLUDE, fn)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"^\s*#.*$", "", text, flags=re.M)
        for m in re.finditer(r"(?:CL_API|CUDALLM_API)\s+[^;(]*?\b(\w+)\s*\(", text):
            names.append(m.group(1))
    return names


def test_headers_declare_entry_points():
    names = declared_symbols()
    assert "cl_gemv_multi" in names and "cudallm_prefill" in names
    assert len(names) >= 40


def test_library_exports_every_declared_symbol():
    lib = _native.lib()
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_signatures_cover_exports():
    assert set(declared_symbols()) <= set(_native.SIGNATURES)


@pytest.mark.parametrize("gtype", [sg.Q4_K, sg.Q5_K, sg.Q6_K, sg.Q5_0, sg.Q8_0, sg.F32])
@pytest.mark.parametrize("k", [256, 896, 3584, 4864, 18944])
def test_row_sizes(gtype, k):
    lib = _native.lib()
    block = sg.BLOCK[gtype][0]
    if k % block:
        assert lib.cl_native_row_bytes(gtype, k) == -1
        assert lib.cl_row_stride(gtype, k) == -1
        return
    rb = sg.row_bytes(gtype, k)
    assert lib.cl_native_row_bytes(gtype, k) == rb
    assert lib.cl_row_stride(gtype, k) == (rb + 15) // 16 * 16


def test_xq_bytes():
    lib = _native.lib()
    assert lib.cl_xq_bytes(30) == 0
    k = 3584
    assert lib.cl_xq_bytes(k) >= 3 * k + k // 16 * 8 + k // 32 * 4


def test_invalid_arguments_are_rejected_without_a_gpu():
    lib = _native.lib()
    assert lib.cl_gemv(99, None, 0, 1, 256, None, None, None, None, None) == 1
    assert lib.cl_argmax(None, 10, None, None, 0, None) == 1
    assert lib.cl_status_string(4) == b"workspace missing or too small"


def test_peer_exchange_layout_and_argument_checks():
    """The tensor-parallel exchange buffer: a 256-byte header and two
    parities of 8 rank slots, each rounded up to 64 floats; bad arguments are
    rejected before anything touches a GPU."""
    import ctypes
    lib = _native.lib()
    assert lib.cl_peer_exchange_bytes(0) == 0
    assert lib.cl_peer_exchange_bytes(5120) == 256 + 2 * 8 * 5120 * 4
    assert lib.cl_peer_exchange_bytes(100) == 256 + 2 * 8 * 128 * 4
    assert lib.cl_peer_exchange_init(None, 5120, None) == 1
    assert lib.cl_peer_exchange_init(4096 + 16, 5120, None) == 1  # not 256-byte aligned
    assert lib.cl_peer_exchange_status(None) is None
    assert lib.cl_peer_exchange_status(4096) == 4096 + 96  # after epoch[8] and flag[2][8]
    bufs = (ctypes.c_void_p * 8)(*[4096 * (i + 1) for i in range(8)])
    a, b = 1 << 20, 2 << 20
    ok = dict(inp=a, out=b, n=5120, max_n=5120, rank=0, world=2)

    def call(**kw):
        p = {**ok, **kw}
        return lib.cl_peer_allreduce(p["inp"], p["out"], p["n"], p["max_n"], p["rank"], p["world"], bufs, None)
    assert call(n=5122) == 1                     # n % 4
    assert call(n=6000) == 1                     # n > max_n
    assert call(world=9) == 1 and call(world=0) == 1
    assert call(rank=2) == 1
    assert call(out=a + 64) == 1                 # overlapping in / out
    assert call(inp=a + 4) == 1                  # unaligned
    assert lib.cl_peer_allreduce(a, b, 5120, 5120, 0, 2, None, None) == 1
