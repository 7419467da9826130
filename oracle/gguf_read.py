"""Minimal GGUF v3 reader for the oracle (test infrastructure only).

Reads the metadata and tensor table of a GGUF file (the layout the reference
readers parse, metal_model.cpp:450-562 / model.cpp:376-448) and returns a
tensor's raw block bytes as numpy rows, which ``oracle.dequant`` turns into
the reference-exact FP32 values.
"""
from __future__ import annotations

import mmap
import struct
from typing import Dict, Tuple

import numpy as np

_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}
_BLOCK = {0: (1, 4), 1: (1, 2), 6: (32, 22), 8: (32, 34), 12: (256, 144), 13: (256, 176), 14: (256, 210)}


class GgufReader:
    def __init__(self, path: str):
        self.path = path
        # mapped read-only: a full-size model is tens of GB, and a test or a
        # CPU sample touches only the rows it uses
        with open(path, "rb") as f:
            self._buf = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        b = self._buf
        magic, version, n_tensors, n_kv = struct.unpack_from("<IIQQ", b, 0)
        if magic != 0x46554747 or version != 3:
            raise ValueError(f"{path}: not a GGUF v3 file")
        pos = 24
        self.metadata: Dict[str, object] = {}
        for _ in range(n_kv):
            key, pos = self._str(pos)
            (vtype,) = struct.unpack_from("<I", b, pos)
            pos += 4
            value, pos = self._value(vtype, pos)
            self.metadata[key] = value
        self.tensors: Dict[str, Tuple[int, Tuple[int, ...], int]] = {}
        for _ in range(n_tensors):
            name, pos = self._str(pos)
            (nd,) = struct.unpack_from("<I", b, pos)
            pos += 4
            dims = struct.unpack_from(f"<{nd}Q", b, pos)
            pos += 8 * nd
            gtype, offset = struct.unpack_from("<IQ", b, pos)
            pos += 12
            self.tensors[name] = (gtype, tuple(dims), offset)
        align = int(self.metadata.get("general.alignment", 32))
        self.data_start = (pos + align - 1) // align * align

    def _str(self, pos):
        (n,) = struct.unpack_from("<Q", self._buf, pos)
        return self._buf[pos + 8:pos + 8 + n].decode(), pos + 8 + n

    def _value(self, vtype, pos):
        if vtype == 8:
            return self._str(pos)
        if vtype == 9:
            etype, count = struct.unpack_from("<IQ", self._buf, pos)
            pos += 12
            out = []
            for _ in range(count):
                v, pos = self._value(etype, pos)
                out.append(v)
            return out, pos
        fmt = _SCALAR[vtype]
        (v,) = struct.unpack_from(fmt, self._buf, pos)
        return v, pos + struct.calcsize(fmt)

    def rows(self, name: str) -> Tuple[int, int, int, np.ndarray]:
        """(ggml type, rows, cols, uint8 [rows, row_bytes]) of a tensor; any
        dimensions past the first are folded into rows."""
        gtype, dims, offset = self.tensors[name]
        cols = dims[0]
        nrows = 1
        for d in dims[1:]:
            nrows *= d
        be, bb = _BLOCK[gtype]
        rb = cols // be * bb
        start = self.data_start + offset
        data = np.frombuffer(self._buf, dtype=np.uint8, count=nrows * rb, offset=start)
        return gtype, nrows, cols, data.reshape(nrows, rb)
