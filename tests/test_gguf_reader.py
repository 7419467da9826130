"""The streaming GGUF reader (csrc/host/gguf.cpp) on damaged files, on the CPU.

The reference's readers throw std::runtime_error for a file they cannot
parse (model.cpp:376-448, metal_model.cpp:450-562); CudaLLM's reader must do
the same for every truncation and for corrupted header fields, and must never
crash or over-allocate.  The files are the seeded synthetic models, cut or
edited; `cudallm_gguf_inspect` runs the product's reader without a GPU, and a
build of the same reader under AddressSanitizer and UndefinedBehaviorSanitizer
runs over the whole corpus.
"""
import ctypes
import os
import random
import shutil
import struct
import subprocess
import sys

import numpy as np
import pytest

from myllm_b200 import _native
from myllm_b200 import synth_gguf as sg

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ERUNTIME = 4


def inspect(path):
    """(status, architecture, tensor count, error message)."""
    lib = _native.lib()
    arch = ctypes.create_string_buffer(64)
    count = ctypes.c_uint64(0)
    rc = lib.cudallm_gguf_inspect(path.encode(), arch, 64, ctypes.byref(count))
    return rc, arch.value.decode(), count.value, lib.cudallm_last_error().decode() if rc else ""


def header_length(data):
    """Bytes before the tensor data (the reader's data_start)."""
    n_tensors, n_kv = struct.unpack_from("<QQ", data, 8)
    pos = 24

    def skip(t, pos):
        sizes = {0: 1, 1: 1, 7: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 10: 8, 11: 8, 12: 8}
        if t in sizes:
            return pos + sizes[t]
        if t == 8:
            (n,) = struct.unpack_from("<Q", data, pos)
            return pos + 8 + n
        et, n = struct.unpack_from("<IQ", data, pos)
        pos += 12
        for _ in range(n):
            pos = skip(et, pos)
        return pos
    for _ in range(n_kv):
        (n,) = struct.unpack_from("<Q", data, pos)
        pos += 8 + n
        (t,) = struct.unpack_from("<I", data, pos)
        pos = skip(t, pos + 4)
    for _ in range(n_tensors):
        (n,) = struct.unpack_from("<Q", data, pos)
        pos += 8 + n
        (nd,) = struct.unpack_from("<I", data, pos)
        pos += 4 + 8 * nd + 4 + 8
    return (pos + 31) // 32 * 32


@pytest.fixture(scope="module")
def models(tmp_path_factory):
    d = tmp_path_factory.mktemp("gguf")
    q = str(d / "tiny_qwen2.gguf")
    sg.write_qwen2(sg.tiny_spec(seed=7), q)
    m = sg.cached_moe(sg.tiny_moe_spec(seed=5, layers=4), str(d))
    return {"qwen2": (q, len(sg.qwen2_tensors(sg.tiny_spec(seed=7)))),
            "qwen35moe": (m, len(sg.moe_tensors(sg.tiny_moe_spec(seed=5, layers=4))))}


def test_valid_models_are_read(models):
    for arch, (path, n) in models.items():
        assert inspect(path)[:3] == (0, arch, n)


def cut_points(data):
    head = header_length(data)
    return sorted(set(list(range(0, head + 1, 7)) + [head - 1, head + 1, len(data) // 2, len(data) - 1]))


def test_every_truncation_is_a_runtime_error(models, tmp_path):
    for arch, (path, _) in models.items():
        data = open(path, "rb").read()
        for cut in cut_points(data):
            p = str(tmp_path / f"cut_{arch}_{cut}.gguf")
            with open(p, "wb") as f:
                f.write(data[:cut])
            rc, _, _, msg = inspect(p)
            assert rc == ERUNTIME and msg, (arch, cut)


def raw_gguf(kvs=(), tensors=(), n_kv=None, n_tensors=None, version=3, magic=0x46554747, tail=b"\0" * 64):
    body = b"".join(kvs) + b"".join(tensors)
    head = struct.pack("<IIQQ", magic, version, len(tensors) if n_tensors is None else n_tensors,
                       len(kvs) if n_kv is None else n_kv)
    return head + body + tail


def tensor_info(name, dims, gtype, offset=0):
    return sg._gguf_str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims) + \
        struct.pack("<IQ", gtype, offset)


ARCH = sg._kv("general.architecture", "qwen2")
CORRUPT = {
    "magic": (raw_gguf([ARCH], magic=0x12345678), "not a GGUF file"),
    "version": (raw_gguf([ARCH], version=7), "unsupported GGUF version"),
    "tensor count": (raw_gguf([ARCH], n_tensors=1 << 62), "invalid GGUF header counts"),
    "metadata count": (raw_gguf([ARCH], n_kv=1 << 40), "invalid GGUF header counts"),
    "string length": (raw_gguf([sg._gguf_str("k") + struct.pack("<IQ", 8, 1 << 62)]), "invalid GGUF string length"),
    "metadata type": (raw_gguf([sg._gguf_str("k") + struct.pack("<I", 99)]), "unsupported GGUF metadata type"),
    "nested arrays": (raw_gguf([sg._gguf_str("k") + struct.pack("<I", 9) + struct.pack("<IQ", 9, 1) * 100 +
                                struct.pack("<IQ", 0, 0)]), "nested too deeply"),
    "array of huge strings": (raw_gguf([sg._gguf_str("k") + struct.pack("<IIQ", 9, 8, 3) + struct.pack("<Q", 1 << 60)]),
                              "invalid GGUF string length"),
    "string array count": (raw_gguf([sg._gguf_str("k") + struct.pack("<IIQ", 9, 8, 1 << 40)]), "truncated GGUF file"),
    "tensor rank": (raw_gguf([ARCH], [tensor_info("t", [], sg.F32)]), "invalid tensor rank"),
    "tensor type": (raw_gguf([ARCH], [tensor_info("t", [32], 99)]), "unsupported GGUF tensor type"),
    "block alignment": (raw_gguf([ARCH], [tensor_info("t", [100], sg.Q4_K)]), "not block aligned"),
    "size overflow": (raw_gguf([ARCH], [tensor_info("t", [1 << 40, 1 << 40], sg.F32)]), "overflows"),
    "outside file": (raw_gguf([ARCH], [tensor_info("t", [64], sg.F32, offset=1 << 20)]), "outside file"),
    "duplicate": (raw_gguf([ARCH], [tensor_info("t", [4], sg.F32), tensor_info("t", [4], sg.F32, 32)],
                           tail=b"\0" * 128), "duplicate GGUF tensor"),
    "alignment key": (raw_gguf([ARCH, sg._kv("general.alignment", 24)]), "invalid GGUF alignment"),
}


@pytest.mark.parametrize("case", sorted(CORRUPT))
def test_corrupted_fields_are_runtime_errors(tmp_path, case):
    data, message = CORRUPT[case]
    p = str(tmp_path / "bad.gguf")
    with open(p, "wb") as f:
        f.write(data)
    rc, _, _, msg = inspect(p)
    assert rc == ERUNTIME and message in msg, (case, rc, msg)


def test_missing_and_empty_files(tmp_path):
    assert inspect(str(tmp_path / "absent.gguf"))[0] == ERUNTIME
    p = tmp_path / "empty.gguf"
    p.write_bytes(b"")
    assert inspect(str(p))[0] == ERUNTIME


def damaged_copies(path, out_dir, n, seed):
    """n copies of `path` with 1-4 random header bytes overwritten."""
    data = open(path, "rb").read()
    head = header_length(data)
    rng = random.Random(seed)
    paths = []
    for i in range(n):
        b = bytearray(data[:head + 256])
        for _ in range(rng.randint(1, 4)):
            b[rng.randrange(head)] = rng.randrange(256)
        p = os.path.join(out_dir, f"damaged_{seed}_{i}.gguf")
        with open(p, "wb") as f:
            f.write(bytes(b))
        paths.append(p)
    return paths


def test_random_header_damage_never_crashes(models, tmp_path):
    paths = damaged_copies(models["qwen2"][0], str(tmp_path), 300, 1)
    # in a child process, so that a crash fails this test instead of ending the run
    code = ("import sys, ctypes; from myllm_b200 import _native; lib = _native.lib(); b = ctypes.create_string_buffer(64)\n"
            "codes = [lib.cudallm_gguf_inspect(p.encode(), b, 64, None) for p in sys.argv[1:]]\n"
            "assert set(codes) <= {0, 4}, set(codes); print(codes.count(0), codes.count(4))")
    r = subprocess.run([sys.executable, "-c", code] + paths, cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    ok, bad = map(int, r.stdout.split())
    assert ok + bad == len(paths) and bad > 0


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_reader_under_address_and_undefined_behavior_sanitizers(models, tmp_path):
    exe = str(tmp_path / "gguf_check")
    build = subprocess.run(["g++", "-std=c++17", "-O1", "-g", "-fsanitize=address,undefined",
                            "-fno-sanitize-recover=all", "-I", os.path.join(ROOT, "myllm_b200", "csrc", "host"),
                            os.path.join(ROOT, "tests", "native", "gguf_check.cpp"),
                            os.path.join(ROOT, "myllm_b200", "csrc", "host", "gguf.cpp"), "-o", exe],
                           capture_output=True, text=True, timeout=300)
    assert build.returncode == 0, build.stderr[-2000:]
    corpus = [p for p, _ in models.values()]
    for arch, (path, _) in models.items():
        data = open(path, "rb").read()
        for cut in cut_points(data)[::3]:
            p = str(tmp_path / f"cut_{arch}_{cut}.gguf")
            with open(p, "wb") as f:
                f.write(data[:cut])
            corpus.append(p)
    for i, (data, _) in enumerate(CORRUPT.values()):
        p = str(tmp_path / f"corrupt_{i}.gguf")
        with open(p, "wb") as f:
            f.write(data)
        corpus.append(p)
    corpus += damaged_copies(models["qwen2"][0], str(tmp_path), 200, 2)
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1:abort_on_error=0", UBSAN_OPTIONS="print_stacktrace=1")
    r = subprocess.run([exe] + corpus, capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0 and "runtime error" not in r.stderr and "AddressSanitizer" not in r.stderr, \
        r.stderr[-3000:]
    accepted, rejected = map(int, r.stdout.split())
    assert accepted >= 2 and accepted + rejected == len(corpus)


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_tokenizer_tables_are_read(tmp_path):
    """tokenizer.ggml.tokens / .merges / .pre, which a caller building its
    tokenizer from the backend's config needs (model.h:30-32), read back
    entry for entry through the product's reader (under ASan / UBSan), and
    cuts inside the tables are errors, not crashes."""
    tokens = [f"tok{i}" for i in range(997)] + ["<|im_end|>", "Ġthe", "中文"]
    merges = [f"a{i} b{i}" for i in range(499)] + ["Ġ t"]
    meta = {"general.architecture": "qwen2", "tokenizer.ggml.pre": "qwen2",
            "tokenizer.ggml.tokens": tokens, "tokenizer.ggml.merges": merges}
    t = sg.TensorSpec("t", sg.F32, (4,), lambda: np.zeros(4, dtype=np.float32).view(np.uint8))
    path = str(tmp_path / "vocab.gguf")
    sg.write_gguf(path, meta, [t])
    exe = str(tmp_path / "strings")
    build = subprocess.run(["g++", "-std=c++17", "-O1", "-g", "-fsanitize=address,undefined",
                            "-fno-sanitize-recover=all", "-I", os.path.join(ROOT, "myllm_b200", "csrc", "host"),
                            os.path.join(ROOT, "tests", "native", "gguf_strings_check.cpp"),
                            os.path.join(ROOT, "myllm_b200", "csrc", "host", "gguf.cpp"), "-o", exe],
                           capture_output=True, text=True, timeout=300)
    assert build.returncode == 0, build.stderr[-2000:]
    r = subprocess.run([exe, path], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.splitlines() == ["1000", "500", "tok0", "中文", "a0 b0", "Ġ t", "qwen2"]
    data = open(path, "rb").read()
    for cut in range(24, header_length(data), 97):
        p = str(tmp_path / f"cut{cut}.gguf")
        with open(p, "wb") as f:
            f.write(data[:cut])
        r = subprocess.run([exe, p], capture_output=True, text=True, timeout=60)
        assert r.returncode == 0 and r.stdout.startswith("error: "), (cut, r.stdout, r.stderr[-500:])
