"""CPU tests of the C-ABI library: it loads, exports every declared symbol,
and its pure host queries agree with the GGUF block sizes."""
import os
import re
import shutil

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


def test_peer_wait_limit_bounds():
    """The peer exchange's wait limit is settable within 1 ms .. 2 min."""
    from myllm_b200 import _native
    lib = _native.lib()
    assert lib.cl_peer_set_wait_limit_ns(10) == 1            # below 1 ms
    assert lib.cl_peer_set_wait_limit_ns(10 ** 12) == 1      # above 2 min
    assert lib.cl_peer_set_wait_limit_ns(20 * 10 ** 9) == 0  # the default


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


# pointers the header documents as optional: a NULL there is a valid call
OPTIONAL_POINTERS = {("cl_argmax_ex", 4),   # value
                     ("cl_rmsnorm", 5), ("cl_rmsnorm", 6),  # y or xq may be omitted
                     ("cl_rope_kv", 9)}     # device position (host pos0 used instead)


def _is_ptr(a):
    import ctypes
    return a in (ctypes.c_void_p, ctypes.c_char_p) or (isinstance(a, type) and issubclass(a, ctypes._Pointer))


# Entry points whose pointer arguments are host structs describing device
# memory (checked by test_fused_decode_description_checks instead).
HOST_STRUCT_ENTRIES = ("cl_qwen2_decode_supported", "cl_qwen2_decode_step")


def _fused_desc(n_layers=2, hidden=3584, ffn=18944, heads=28, kv=4, d=128, vocab=152064, types=None):
    """A cl_qwen2_decode / cl_qwen2_layer pair of the 7B shape with made-up,
    aligned device addresses (the checks never dereference them)."""
    import ctypes
    addr = iter(range(1 << 24, 1 << 40, 1 << 20))
    layers = (_native.Qwen2Layer * n_layers)()
    for l in range(n_layers):
        L = layers[l]
        for f in ("q", "k", "v", "o", "gate", "up", "down", "q_bias", "k_bias", "v_bias", "attn_norm", "ffn_norm",
                  "k_cache", "v_cache"):
            setattr(L, f, next(addr))
        t = types or {}
        L.q_type = t.get("q", sg.Q4_K)
        L.k_type = t.get("k", sg.Q4_K)
        L.v_type = t.get("v", sg.Q6_K)
        L.o_type = t.get("o", sg.Q4_K)
        L.gate_type = t.get("gate", sg.Q4_K)
        L.down_type = t.get("down", sg.Q6_K if l % 2 == 0 else sg.Q4_K)
    m = _native.Qwen2Decode()
    m.layers = next(addr)
    m.n_layers, m.hidden, m.ffn, m.vocab = n_layers, hidden, ffn, vocab
    m.q_heads, m.kv_heads, m.head_dim, m.capacity = heads, kv, d, 4096
    m.eps, m.scale = 1e-6, d ** -0.5
    for f in ("embd", "out_w", "out_norm", "rope", "ints", "h", "q", "k", "v", "att", "act", "logits"):
        setattr(m, f, next(addr))
    m.embd_stride, m.embd_type, m.out_type = 2016, sg.Q4_K, sg.Q6_K
    return m, layers, ctypes.byref(m), layers


def test_fused_decode_description_checks():
    """cl_qwen2_decode_supported / _step on host descriptions, without a GPU:
    the 7B and 14B shapes qualify; other head widths, 32-column formats, more
    than 8 query heads per KV head, missing or misaligned pointers do not;
    the step checks its workspace before launching."""
    import ctypes
    lib = _native.lib()
    m, layers, pm, pl = _fused_desc()
    assert lib.cl_qwen2_decode_supported(pm, pl) == 0
    m14, l14, pm14, pl14 = _fused_desc(hidden=5120, ffn=13824, heads=40, kv=8)
    assert lib.cl_qwen2_decode_supported(pm14, pl14) == 0
    assert lib.cl_qwen2_decode_supported(None, pl) == 1
    assert lib.cl_qwen2_decode_supported(pm, None) == 1
    for kw in (dict(d=64, hidden=1792), dict(heads=36, kv=4, hidden=36 * 128), dict(ffn=4864 + 128),
               dict(types={"q": sg.Q5_0}), dict(types={"down": sg.Q8_0}), dict(vocab=152064 + 8)):
        _, _, p2, l2 = _fused_desc(**kw)
        assert lib.cl_qwen2_decode_supported(p2, l2) == 2, kw
    for splits, rc in ((32, 0), (33, 2), (-1, 2), (0, 0)):  # attention key splits: 0 (automatic) .. 32
        m.attn_splits = splits
        assert lib.cl_qwen2_decode_supported(pm, pl) == rc, splits
    layers[1].up = None  # the tiled gate pack holds the up rows: `up` is not read
    assert lib.cl_qwen2_decode_supported(pm, pl) == 0
    layers[1].gate = None
    assert lib.cl_qwen2_decode_supported(pm, pl) == 1
    layers[1].gate = (1 << 30) + 8  # misaligned
    assert lib.cl_qwen2_decode_supported(pm, pl) == 1
    layers[1].gate = 1 << 30
    assert lib.cl_qwen2_decode_step(pm, pl, None, 1 << 20, None) == 1  # no workspace
    assert lib.cl_qwen2_decode_step(pm, pl, (1 << 30) + 16, 1 << 20, None) == 1  # misaligned workspace
    assert lib.cl_qwen2_decode_status(None) is None
    assert lib.cl_qwen2_decode_status(1 << 30) == (1 << 30) + 8  # after the barrier and done counters
    assert lib.cl_qwen2_decode_init(None, 256, None) == 1


def test_decode_pack_sizes():
    """The tiled decode layout: Q4_K units of 16 x 144 bytes, Q6_K half
    super-block units of 16 x 112 bytes; shapes off the 16-row (8 for a
    gate/up pair) or 256-column grid are refused."""
    lib = _native.lib()
    assert lib.cl_decode_pack_bytes(sg.Q4_K, 18944, 3584, 0) == 18944 // 16 * 14 * 16 * 144
    assert lib.cl_decode_pack_bytes(sg.Q4_K, 18944, 3584, 1) == 18944 // 8 * 14 * 16 * 144
    assert lib.cl_decode_pack_bytes(sg.Q6_K, 152064, 3584, 0) == 152064 // 16 * 28 * 16 * 112
    assert lib.cl_decode_pack_bytes(sg.Q5_0, 896, 896, 0) == 0
    assert lib.cl_decode_pack_bytes(sg.Q4_K, 100, 3584, 0) == 0
    assert lib.cl_decode_pack_bytes(sg.Q4_K, 3584, 1000, 0) == 0
    assert lib.cl_decode_pack_bytes(sg.Q4_K, 16, 768, 0) == 16 * 4 * 144  # an odd count padded to two units
    assert lib.cl_decode_pack_bytes(sg.Q6_K, 16, 768, 0) == 16 * 3 * 210 + 16 * 3 * 14
    assert lib.cl_decode_pack(sg.Q4_K, None, 2016, 16, 3584, None, 1 << 20, None) == 1


def test_grouped_expert_sizes_and_checks():
    """The grouped prefill expert GEMV: XQ planes of 128 bytes per 32 input
    columns per input row; at most 4095 local experts; the planes scratch
    must hold every input row (ceil(routes / x_group) of them); the checks
    come before any launch."""
    lib = _native.lib()
    assert lib.cl_moe_xq_planes_bytes(64, 2048) == 64 * 64 * 128
    assert lib.cl_moe_xq_planes_bytes(512, 512) == 512 * 16 * 128
    assert lib.cl_moe_xq_planes_bytes(0, 2048) == 0 and lib.cl_moe_xq_planes_bytes(4, 100) == 0
    F = 1 << 20
    assert lib.cl_moe_group_routes(F, 8, 4096, 0, 1, F, F, None) == 1   # too many local experts
    assert lib.cl_moe_group_routes(F, 8, 256, 2, 2, F, F, None) == 1    # rank outside the world
    assert lib.cl_moe_group_routes(F, 0, 256, 0, 1, F, F, None) == 1    # no routes
    assert lib.cl_moe_group_routes(F, 8, 256, 0, 1, F, F, None) == 3    # reaches the launch (no GPU here)
    st = lib.cl_row_stride(sg.Q4_K, 256)

    def grouped(routes=8, x_group=4, n_local=4, planes_bytes=2 * 8 * 128, gtype=sg.Q4_K, x_stride=256):
        return lib.cl_moe_expert_gemv_grouped(gtype, F, None, st, 16, 256, F, x_stride, x_group, F, routes, 0, 1, F,
                                              F, n_local, F, planes_bytes, F, None)

    assert grouped() == 3
    assert grouped(planes_bytes=2 * 8 * 128 - 16) == 1                  # planes too small for 2 input rows
    assert grouped(routes=9, planes_bytes=2 * 8 * 128) == 1            # 9 routes over groups of 4: 3 rows
    assert grouped(routes=9, planes_bytes=3 * 8 * 128) == 3
    assert grouped(x_group=0) == 1 and grouped(n_local=0) == 1 and grouped(x_stride=6) == 1
    assert grouped(gtype=sg.F32) != 3


def test_gemv_pack_sizes_and_checks():
    """The fragment-packed GEMV layout: units of 16 rows x one super-block
    (Q4_K 2304 bytes, Q6_K 3360), ragged row counts padded to a whole tile
    (8 rows per tile for a gate/up pair); other formats and k % 256 != 0
    are refused; cl_gemv_packed checks its segments and alignments before
    it looks at the device."""
    import ctypes
    lib = _native.lib()
    assert lib.cl_gemv_pack_bytes(sg.Q4_K, 18944, 3584, 0) == 1184 * 14 * 2304
    assert lib.cl_gemv_pack_bytes(sg.Q4_K, 18944, 3584, 1) == 2368 * 14 * 2304
    assert lib.cl_gemv_pack_bytes(sg.Q6_K, 152064, 3584, 0) == 9504 * 14 * 3360
    assert lib.cl_gemv_pack_bytes(sg.Q4_K, 17, 256, 0) == 2 * 2304
    assert lib.cl_gemv_pack_bytes(sg.Q6_K, 17, 256, 1) == 3 * 3360
    assert lib.cl_gemv_pack_bytes(sg.Q5_0, 896, 896, 0) == 0
    assert lib.cl_gemv_pack_bytes(sg.Q4_K, 3584, 1000, 0) == 0
    F, M = 1 << 20, (1 << 20) + 4
    st = lib.cl_row_stride(sg.Q4_K, 256)
    assert lib.cl_gemv_pack(sg.Q4_K, F, st, 16, 256, None, M, None) == 1  # misaligned output
    assert lib.cl_gemv_pack(sg.Q4_K, F, st - 16, 16, 256, None, F, None) == 1  # stride too short

    def seg(w=F, gtype=sg.Q4_K, n=16, bias=None):
        return _native.GemvPackedSegment(gtype, w, n, bias, None, F)

    one = (_native.GemvPackedSegment * 1)(seg())
    two = (_native.GemvPackedSegment * 2)(seg(), seg())
    assert lib.cl_gemv_packed(one, 1, 256, M, None, 1e-6, 0, F, 1 << 20, None) == 1  # misaligned x
    assert lib.cl_gemv_packed(one, 1, 256, F, None, 1e-6, 0, M, 1 << 20, None) == 1  # misaligned workspace
    assert lib.cl_gemv_packed((_native.GemvPackedSegment * 1)(seg(w=M)), 1, 256, F, None, 1e-6, 0, F, 1 << 20,
                              None) == 1  # misaligned weights
    assert lib.cl_gemv_packed((_native.GemvPackedSegment * 1)(seg(gtype=sg.Q8_0)), 1, 256, F, None, 1e-6, 0, F,
                              1 << 20, None) == 1  # not a K-quant
    assert lib.cl_gemv_packed(two, 2, 256, F, None, 1e-6, 1, F, 1 << 20, None) == 1  # SwiGLU takes one pair
    assert lib.cl_gemv_packed((_native.GemvPackedSegment * 1)(seg(bias=F)), 1, 256, F, None, 1e-6, 1, F, 1 << 20,
                              None) == 1  # no bias on the SwiGLU form
    assert lib.cl_gemv_packed(one, 1, 300, F, None, 1e-6, 0, F, 1 << 20, None) == 1  # k % 256
    assert lib.cl_gemv_packed(one, 1, 256 * 85, F, None, 1e-6, 0, F, 1 << 20, None) == 2  # k beyond 21504
    assert lib.cl_gemv_packed(ctypes.cast(None, ctypes.POINTER(_native.GemvPackedSegment)), 1, 256, F, None, 1e-6,
                              0, F, 1 << 20, None) == 1
    # valid arguments reach the device query (CL_ERR_CUDA without a GPU)
    if not _gpu_present():
        assert lib.cl_gemv_packed(one, 1, 256, F, None, 1e-6, 0, F, 1 << 20, None) == 3


def _gpu_present():
    import torch
    return torch.cuda.is_available()


def test_null_pointers_are_rejected_before_any_launch():
    """Every kernel entry point returns an error status for a NULL required
    pointer instead of launching: on a GPU such a launch would read or write
    address 0.  Without a GPU, a call that got as far as a launch returns
    CL_ERR_CUDA (3); a checked argument returns CL_ERR_INVALID (1) or the
    workspace error (4).  The no-allocation attention variant resolves its
    scratch array before delegating to cl_attn_decode's checks, so without a
    device it stops earlier and is left out here."""
    import ctypes
    lib = _native.lib()
    fake = 1 << 20
    unchecked = []
    for name, (rt, args) in sorted(_native.SIGNATURES.items()):
        if not name.startswith("cl_") or rt is not ctypes.c_int or name in HOST_STRUCT_ENTRIES + (
                "cl_device_error", "cl_attn_decode_noalloc"):
            continue
        base = [(ctypes.cast(fake, a) if isinstance(a, type) and issubclass(a, ctypes._Pointer) else fake)
                if _is_ptr(a) else (1.0 if a is ctypes.c_float else 64) for a in args]
        for i, a in enumerate(args[:-1]):  # the last argument is the stream: NULL is the default stream
            if not _is_ptr(a) or (name, i) in OPTIONAL_POINTERS:
                continue
            v = list(base)
            v[i] = None
            rc = getattr(lib, name)(*v)
            if rc not in (1, 4):
                unchecked.append((name, i, rc))
    assert not unchecked, unchecked


def test_misaligned_pointers_are_rejected_where_kernels_use_wide_loads():
    """Pointers that a kernel reads with 16-byte vector loads, bulk copies or
    cp.async must be 16-byte aligned (F32 weight rows read as floats: 4), or
    the call returns CL_ERR_INVALID instead of faulting on the GPU; the same
    call with aligned pointers gets past the checks (CL_ERR_CUDA: no GPU)."""
    import ctypes
    lib = _native.lib()
    F, M = 1 << 20, (1 << 20) + 4
    q4 = sg.Q4_K
    st = lib.cl_row_stride(q4, 256)
    ws = lib.cl_attn_decode_workspace_bytes(4, 64, 128)
    cases = {
        "cl_gemv": (lambda w=F, x=F: lib.cl_gemv(q4, w, st, 16, 256, x, None, None, F, None), ("w", "x")),
        "cl_gemv_swiglu": (lambda w=F, x=F: lib.cl_gemv_swiglu(q4, w, F, st, 16, 256, x, None, 1e-6, F, None),
                           ("w", "x")),
        "cl_gemm_tc": (lambda w=F, x=F: lib.cl_gemm_tc(q4, w, st, 128, 256, x, 128, None, None, F, 0, None),
                       ("w", "x")),
        "cl_attn_decode": (lambda q=F, kc=F, vc=F, xq=None: lib.cl_attn_decode(q, kc, vc, F, 128, 4, 2, 64, 0.1, F,
                                                                               xq, F, ws, None),
                           ("q", "kc", "vc", "xq")),
        "cl_attn_decode_rope": (lambda q=F, kc=F, vc=F: lib.cl_attn_decode_rope(q, F, F, F, F, 64, kc, vc, 128, 4, 2,
                                                                                64, 0.1, F, None, F, ws, None),
                                ("q", "kc", "vc")),
        "cl_moe_expert_gemv": (lambda w=F, x=F: lib.cl_moe_expert_gemv(q4, w, F, st, 16, 256, x, 0, F, 2, 0, 1, F,
                                                                       None), ("w", "x")),
        "cl_moe_expert_gemv_grouped": (lambda w=F, x=F, planes=2 * F: lib.cl_moe_expert_gemv_grouped(
            q4, w, None, st, 16, 256, x, 256, 1, F, 2, 0, 1, F, F, 4, planes, 4096, F, None),
                                       ("w", "x", "planes")),
        "cl_gemv_f32": (lambda w=F, x=F: lib.cl_gemv_f32(w, 16, 256, x, F, None), ("w", "x")),
        "cl_peer_allreduce": (lambda inp=F, out=2 * F: lib.cl_peer_allreduce(
            inp, out, 256, 256, 0, 1, (ctypes.c_void_p * 1)(4 * F), None), ("inp", "out")),
    }
    for name, (call, ptrs) in cases.items():
        assert call() == 3, name  # aligned: reaches the launch
        for p in ptrs:
            assert call(**{p: M}) == 1, (name, p)
    # F32 rows are read as floats: 4-byte alignment; quantized rows byte by byte
    f32 = sg.F32
    st32 = lib.cl_row_stride(f32, 256)
    assert lib.cl_embed(f32, F + 2, st32, 8, 256, F, 1, F, F, None) == 1
    assert lib.cl_embed(q4, F + 2, st, 8, 256, F, 1, F, F, None) == 3
    assert lib.cl_gemm_simt(f32, F + 2, st32, 16, 256, F, 4, None, None, F, None) == 1


def test_backend_queries_without_a_model():
    import ctypes
    lib = _native.lib()
    assert lib.cudallm_available(None) == 0
    out = (ctypes.c_uint64 * 3)()
    assert lib.cudallm_expert_cache(None, out) == 1  # CUDALLM_EINVAL


@pytest.mark.skipif(shutil.which("gcc") is None or shutil.which("g++") is None, reason="needs gcc and g++")
@pytest.mark.parametrize("header,lang", [("cudallm.h", "c"), ("cudallm_kernels.h", "c"),
                                         ("cuda_llm.h", "c++"), ("cuda_moe_llm.h", "c++")])
def test_headers_stand_alone(tmp_path, header, lang):
    """The C-ABI headers compile as plain C11 (cgo, ctypes-generated stubs and
    other C hosts include them); the C++ API headers as C++17, each on its own."""
    import subprocess
    src = tmp_path / ("h.c" if lang == "c" else "h.cpp")
    src.write_text(f'#include "{header}"\nint main(void) {{ return 0; }}\n')
    cmd = (["gcc", "-std=c11"] if lang == "c" else ["g++", "-std=c++17"]) + [
        "-Wall", "-Wextra", "-Werror", "-fsyntax-only", "-I", INCLUDE, "-I", "/usr/local/cuda/include", str(src)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_a_c_host_links_and_calls_the_backend_abi(tmp_path):
    """C linkage of the backend ABI: a C program built against include/ and
    linked to libcudallm.so reads a model's header and the shard plans."""
    import subprocess
    root = os.path.dirname(INCLUDE)
    exe = str(tmp_path / "c_abi_check")
    libdir = os.path.dirname(_native.LIB_PATH)
    r = subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-I", INCLUDE,
                        os.path.join(root, "tests", "native", "c_abi_check.c"), "-L", libdir, "-lcudallm",
                        "-Wl,-rpath," + libdir, "-o", exe], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    model = str(tmp_path / "tiny.gguf")
    sg.write_qwen2(sg.tiny_spec(seed=7), model)
    r = subprocess.run([exe, model], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    arch, tensors, q0, vrows, gather, er13, sr3 = r.stdout.split()
    assert arch == "qwen2" and int(tensors) == len(sg.qwen2_tensors(sg.tiny_spec(seed=7)))
    # 14B at 8 ranks, rank 7: heads 35..39, the last 19008 vocabulary rows, gathered attention
    assert (int(q0), int(vrows), int(gather)) == (35, 19008, 1)
    assert (int(er13), int(sr3)) == (13 % 4, 3 % 4)


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_a_cxx_host_links_the_cxx_api(tmp_path):
    """The C++ API (cuda_llm.h, cuda_moe_llm.h) is exported from the shared
    library: a C++17 program links it, plans shards, reads a model's
    architecture, and gets std::runtime_error (not a crash) when it builds a
    model on a host without a GPU."""
    import subprocess
    import torch
    root = os.path.dirname(INCLUDE)
    exe = str(tmp_path / "cxx_api_check")
    libdir = os.path.dirname(_native.LIB_PATH)
    r = subprocess.run(["g++", "-std=c++17", "-Wall", "-Werror", "-I", INCLUDE,
                        os.path.join(root, "tests", "native", "cxx_api_check.cpp"), "-L", libdir, "-lcudallm",
                        "-Wl,-rpath," + libdir, "-o", exe], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    model = str(tmp_path / "tiny.gguf")
    sg.write_qwen2(sg.tiny_spec(seed=7), model)
    r = subprocess.run([exe, model], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    arch, q0, gather, outcome = r.stdout.split()
    assert (arch, q0, gather) == ("qwen2", "35", "1")
    assert outcome == ("constructed" if torch.cuda.is_available() else "runtime_error")


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_generic_backend_host_compiles():
    """A generic host of the reference's backend contract (generate<Backend>
    style: capacity checks, stop token, tokenizer tables, stats in the
    caller's own struct) compiles for both CUDA backends."""
    import subprocess
    root = os.path.dirname(INCLUDE)
    r = subprocess.run(["g++", "-std=c++17", "-Wall", "-Wextra", "-Werror", "-fsyntax-only", "-I", INCLUDE,
                        os.path.join(root, "tests", "native", "generic_backend_check.cpp")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
