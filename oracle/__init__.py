"""ORACLE — test infrastructure only.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg use this package, and only as the checker.  The product (``myllm_b200``)
never imports it.

Two checkers live here:

* ``port``: ``quant_oracle.c`` (this project's C restatement of the
  reference's block decoders and FP32 dequantize-then-matmul), built into
  ``oracle/lib/liboracle.so``.
* ``ReferenceCPU``: the reference's own ``CPULLM`` path compiled from its
  sources into ``oracle/_ref/libref_cpu.so`` by ``oracle/Makefile``, driven
  through ``ref_harness.cpp`` so the logits are visible.  Present only when
  the reference sources were available at build time.
* ``metal_ref``: the reference's Metal compute kernels for qwen35moe
  (``metal_llm.metal``) compiled as C++ into ``oracle/_ref/libref_metal.so``
  by the same target and run on the host in the reference's dispatch order,
  the check of the qwen35moe FP64 restatement (``moe_fp64.py``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional, Tuple

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_LIB = os.path.join(HERE, "lib", "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libref_cpu.so")
# The reference checkout (tianjin95/MyLLM sources) to compile the reference
# checker from: MYLLM_REFERENCE_DIR.  Unset, only an already built
# _ref/libref_cpu.so is used.
REFERENCE_SOURCES = os.environ.get("MYLLM_REFERENCE_DIR", "")

_port = None
_ref = None


def build(reference: Optional[str] = None) -> None:
    """Build the port and, when the reference sources exist, the reference."""
    subprocess.run(["make", "-C", HERE, "port"], check=True, capture_output=True)
    ref = reference or REFERENCE_SOURCES
    if ref and os.path.isdir(ref):
        subprocess.run(["make", "-C", HERE, "ref", f"REF={ref}"], check=True,
                       capture_output=True)


def port():
    global _port
    if _port is None:
        if not os.path.exists(PORT_LIB):
            subprocess.run(["make", "-C", HERE, "port"], check=True, capture_output=True)
        l = ctypes.CDLL(PORT_LIB)
        l.oracle_row_bytes.argtypes = [ctypes.c_int, ctypes.c_longlong]
        l.oracle_row_bytes.restype = ctypes.c_longlong
        l.oracle_dequant.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_longlong,
                                     ctypes.c_longlong, ctypes.c_void_p]
        l.oracle_dequant.restype = ctypes.c_int
        l.oracle_gemm.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_longlong,
                                  ctypes.c_longlong, ctypes.c_void_p, ctypes.c_longlong,
                                  ctypes.c_void_p, ctypes.c_void_p]
        l.oracle_gemm.restype = ctypes.c_int
        _port = l
    return _port


def dequant(gtype: int, data: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """Reference-exact FP32 values of `rows` native GGML rows."""
    data = np.ascontiguousarray(data, dtype=np.uint8)
    out = np.empty((rows, cols), dtype=np.float32)
    if port().oracle_dequant(gtype, data.ctypes.data, rows, cols, out.ctypes.data) != 0:
        raise ValueError("oracle_dequant failed")
    return out


def gemm(gtype: int, w: np.ndarray, n: int, k: int, x: np.ndarray,
         bias: Optional[np.ndarray] = None) -> np.ndarray:
    """Y = X W^T (+ b) with W dequantized per row and FP32 sequential sums."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
    m = x.shape[0]
    y = np.empty((m, n), dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    rc = port().oracle_gemm(gtype, w.ctypes.data, n, k, x.ctypes.data, m,
                            None if b is None else b.ctypes.data, y.ctypes.data)
    if rc != 0:
        raise ValueError("oracle_gemm failed")
    return y


def ref_available() -> bool:
    return os.path.exists(REF_LIB)


def _reflib():
    global _ref
    if _ref is None:
        l = ctypes.CDLL(REF_LIB)
        vp = ctypes.c_void_p
        l.ref_last_error.restype = ctypes.c_char_p
        l.ref_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(vp)]
        l.ref_close.argtypes = [vp]
        l.ref_config.argtypes = [vp, ctypes.POINTER(ctypes.c_longlong), ctypes.c_int]
        l.ref_reset.argtypes = [vp]
        l.ref_prefill.argtypes = [vp, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                                  ctypes.POINTER(ctypes.c_int32)]
        l.ref_decode.argtypes = [vp, ctypes.c_int32, ctypes.c_void_p,
                                 ctypes.POINTER(ctypes.c_int32)]
        l.ref_tensor.argtypes = [vp, ctypes.c_int, ctypes.c_char_p, ctypes.c_void_p,
                                 ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t),
                                 ctypes.POINTER(ctypes.c_size_t)]
        l.ref_cpullm_open.argtypes = [ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(vp)]
        l.ref_cpullm_close.argtypes = [vp]
        l.ref_cpullm_reset.argtypes = [vp]
        l.ref_cpullm_prefill.argtypes = [vp, ctypes.c_void_p, ctypes.c_size_t,
                                         ctypes.POINTER(ctypes.c_int32)]
        l.ref_cpullm_decode.argtypes = [vp, ctypes.c_int32, ctypes.POINTER(ctypes.c_int32)]
        _ref = l
    return _ref


def _check(rc: int) -> None:
    if rc != 0:
        msg = _reflib().ref_last_error().decode()
        raise {1: ValueError, 2: IndexError, 3: OverflowError}.get(rc, RuntimeError)(msg)


class ReferenceCPU:
    """The reference CPU forward (CPULLM's sequence) with logits exposed."""

    def __init__(self, path: str):
        self._h = ctypes.c_void_p()
        _check(_reflib().ref_open(path.encode(), ctypes.byref(self._h)))
        cfg = (ctypes.c_longlong * 8)()
        _check(_reflib().ref_config(self._h, cfg, 8))
        (self.layers, self.hidden, self.ffn, self.heads, self.kv_heads,
         self.head_dim, self.vocab, self.context) = list(cfg)

    def close(self) -> None:
        if self._h:
            _reflib().ref_close(self._h)
            self._h = ctypes.c_void_p()

    __del__ = close

    def reset(self) -> None:
        _reflib().ref_reset(self._h)

    def prefill(self, ids) -> Tuple[int, np.ndarray]:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        logits = np.empty(self.vocab, dtype=np.float32)
        tok = ctypes.c_int32()
        _check(_reflib().ref_prefill(self._h, ids.ctypes.data, ids.size, logits.ctypes.data,
                                     ctypes.byref(tok)))
        return tok.value, logits

    def decode(self, token: int) -> Tuple[int, np.ndarray]:
        logits = np.empty(self.vocab, dtype=np.float32)
        tok = ctypes.c_int32()
        _check(_reflib().ref_decode(self._h, int(token), logits.ctypes.data, ctypes.byref(tok)))
        return tok.value, logits

    def tensor(self, layer: int, which: str) -> np.ndarray:
        rows, cols = ctypes.c_size_t(), ctypes.c_size_t()
        _check(_reflib().ref_tensor(self._h, layer, which.encode(), None, 0,
                                    ctypes.byref(rows), ctypes.byref(cols)))
        out = np.empty((rows.value, cols.value), dtype=np.float32)
        _check(_reflib().ref_tensor(self._h, layer, which.encode(), out.ctypes.data, out.size,
                                    ctypes.byref(rows), ctypes.byref(cols)))
        return out


class ReferenceCPULLM:
    """The reference's CPULLM class itself (tokens only); the timed baseline."""

    def __init__(self, path: str, max_sequence: int = 0):
        self._h = ctypes.c_void_p()
        _check(_reflib().ref_cpullm_open(path.encode(), max_sequence, ctypes.byref(self._h)))

    def close(self) -> None:
        if self._h:
            _reflib().ref_cpullm_close(self._h)
            self._h = ctypes.c_void_p()

    __del__ = close

    def reset(self) -> None:
        _check(_reflib().ref_cpullm_reset(self._h))

    def prefill(self, ids) -> int:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        tok = ctypes.c_int32()
        _check(_reflib().ref_cpullm_prefill(self._h, ids.ctypes.data, ids.size,
                                            ctypes.byref(tok)))
        return tok.value

    def decode(self, token: int) -> int:
        tok = ctypes.c_int32()
        _check(_reflib().ref_cpullm_decode(self._h, int(token), ctypes.byref(tok)))
        return tok.value
