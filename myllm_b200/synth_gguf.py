"""Seeded synthetic GGUF models for parity tests and benchmarks.

Writes GGUF v3 files that the reference readers accept
(model.cpp:376-448 for the CPU path, metal_model.cpp:450-562 for the
streaming reader) and that ``CudaLLM`` / ``CudaMoeLLM`` load:

* ``qwen2``: the keys model.cpp:725-776 reads, an explicit ``output.weight``
  (both reference readers require it; a "tied" model stores a byte-identical
  copy of ``token_embd.weight``), every tensor consumed, block-aligned rows.
* ``qwen35moe``: the keys metal_model.cpp:573-688 reads and the tensor schema
  of moe_model.cpp:84-247 (no MTP/NextN block).

Values come from ``csrc/synth/synth.c``: a counter-based normal generator
keyed by (config seed, tensor name), so the same seed always produces the
same bytes.
"""
from __future__ import annotations

import ctypes
import dataclasses
import hashlib
import os
import struct
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import numpy as np

F32, F16, Q5_0, Q8_0, Q4_K, Q5_K, Q6_K = 0, 1, 6, 8, 12, 13, 14
TYPE_NAMES = {F32: "F32", F16: "F16", Q5_0: "Q5_0", Q8_0: "Q8_0",
              Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K"}
BLOCK = {F32: (1, 4), F16: (1, 2), Q5_0: (32, 22), Q8_0: (32, 34),
         Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210)}

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "lib", "libsynth.so")
_lib = None


def row_bytes(gtype: int, cols: int) -> int:
    block, size = BLOCK[gtype]
    if cols % block:
        raise ValueError(f"{TYPE_NAMES[gtype]} row of {cols} columns is not block aligned")
    return cols // block * size


def lib():
    """Load (building on first use) the C helper library."""
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            from . import build as _build
            _build.build_synth()
        l = ctypes.CDLL(_LIB_PATH)
        l.synth_fill.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong,
                                 ctypes.c_longlong, ctypes.c_ulonglong, ctypes.c_double,
                                 ctypes.c_double, ctypes.c_int]
        l.synth_fill.restype = ctypes.c_int
        l.synth_quantize.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                     ctypes.c_longlong, ctypes.c_longlong]
        l.synth_quantize.restype = ctypes.c_int
        l.synth_normal_f32.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_ulonglong,
                                       ctypes.c_double, ctypes.c_double]
        l.synth_negexp_f32.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_ulonglong,
                                       ctypes.c_double, ctypes.c_double]
        l.synth_uniform_ids.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_ulonglong,
                                        ctypes.c_longlong]
        l.synth_mix64.argtypes = [ctypes.c_ulonglong]
        l.synth_mix64.restype = ctypes.c_ulonglong
        l.synth_set_threads.argtypes = [ctypes.c_int]
        # every core the process may run on, whatever OMP_NUM_THREADS says
        l.synth_set_threads(len(os.sched_getaffinity(0)))
        _lib = l
    return _lib


def stream_key(seed: int, name: str) -> int:
    """64-bit stream key for one tensor of one seeded model."""
    h = 0xCBF29CE484222325
    for b in name.encode():
        h = ((h ^ b) * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return lib().synth_mix64((seed * 0x9E3779B97F4A7C15 ^ h) & 0xFFFFFFFFFFFFFFFF)


def normal(n: int, key: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().synth_normal_f32(out.ctypes.data, n, key, mean, std)
    return out


def uniform_ids(n: int, key: int, bound: int) -> np.ndarray:
    out = np.empty(n, dtype=np.int32)
    lib().synth_uniform_ids(out.ctypes.data, n, key, bound)
    return out


def quantize(x: np.ndarray, gtype: int) -> np.ndarray:
    """Pack a 2-D FP32 array into native GGML rows (uint8 [rows, row_bytes])."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    out = np.empty((rows, row_bytes(gtype, cols)), dtype=np.uint8)
    if lib().synth_quantize(x.ctypes.data, out.ctypes.data, gtype, rows, cols) != 0:
        raise ValueError("quantize failed")
    return out


def fill(gtype: int, rows: int, cols: int, key: int, mean: float, std: float) -> np.ndarray:
    out = np.empty((rows, row_bytes(gtype, cols)), dtype=np.uint8)
    if lib().synth_fill(out.ctypes.data, gtype, rows, cols, key, mean, std, len(os.sched_getaffinity(0))) != 0:
        raise ValueError("synth_fill failed")
    return out


# ---------------------------------------------------------------------------
# GGUF v3 writer
# ---------------------------------------------------------------------------
_GGUF_U32, _GGUF_I32, _GGUF_F32, _GGUF_BOOL, _GGUF_STR, _GGUF_ARR, _GGUF_U64 = 4, 5, 6, 7, 8, 9, 10


def _gguf_str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _kv(key: str, value) -> bytes:
    if isinstance(value, bool):
        return _gguf_str(key) + struct.pack("<IB", _GGUF_BOOL, int(value))
    if isinstance(value, int):
        return _gguf_str(key) + struct.pack("<II", _GGUF_U32, value)
    if isinstance(value, float):
        return _gguf_str(key) + struct.pack("<If", _GGUF_F32, value)
    if isinstance(value, str):
        return _gguf_str(key) + struct.pack("<I", _GGUF_STR) + _gguf_str(value)
    if isinstance(value, (list, tuple)):
        if all(isinstance(v, str) for v in value):
            body = b"".join(_gguf_str(v) for v in value)
            return _gguf_str(key) + struct.pack("<IIQ", _GGUF_ARR, _GGUF_STR, len(value)) + body
        if all(isinstance(v, bool) for v in value):
            body = bytes(int(v) for v in value)
            return _gguf_str(key) + struct.pack("<IIQ", _GGUF_ARR, _GGUF_BOOL, len(value)) + body
        body = b"".join(struct.pack("<i", int(v)) for v in value)
        return _gguf_str(key) + struct.pack("<IIQ", _GGUF_ARR, _GGUF_I32, len(value)) + body
    raise TypeError(f"unsupported metadata value for {key}: {value!r}")


@dataclasses.dataclass
class TensorSpec:
    name: str
    gtype: int
    dims: Tuple[int, ...]          # GGUF order: dims[0] = columns
    producer: Callable[[], np.ndarray]

    @property
    def cols(self) -> int:
        return self.dims[0]

    @property
    def rows(self) -> int:
        r = 1
        for d in self.dims[1:]:
            r *= d
        return r

    @property
    def nbytes(self) -> int:
        return self.rows * row_bytes(self.gtype, self.cols)


def write_gguf(path: str, metadata: Dict[str, object], tensors: Sequence[TensorSpec],
               alignment: int = 32) -> str:
    """Write a GGUF v3 file; returns the SHA-256 of its bytes."""
    head = bytearray()
    head += struct.pack("<IIQQ", 0x46554747, 3, len(tensors), len(metadata))
    for k, v in metadata.items():
        head += _kv(k, v)
    offset = 0
    offsets = []
    for t in tensors:
        offsets.append(offset)
        head += _gguf_str(t.name) + struct.pack("<I", len(t.dims))
        head += b"".join(struct.pack("<Q", d) for d in t.dims)
        head += struct.pack("<IQ", t.gtype, offset)
        offset += t.nbytes
        offset = (offset + alignment - 1) // alignment * alignment
    pad = (-len(head)) % alignment
    head += b"\0" * pad
    sha = hashlib.sha256()
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(head)
        sha.update(head)
        pos = 0
        for t, off in zip(tensors, offsets):
            if off > pos:
                f.write(b"\0" * (off - pos))
                sha.update(b"\0" * (off - pos))
                pos = off
            data = t.producer()
            if data.nbytes != t.nbytes:
                raise ValueError(f"{t.name}: produced {data.nbytes} bytes, expected {t.nbytes}")
            mv = memoryview(np.ascontiguousarray(data).reshape(-1))
            f.write(mv)
            sha.update(mv)
            pos += t.nbytes
    os.replace(tmp, path)
    return sha.hexdigest()


# ---------------------------------------------------------------------------
# qwen2 models
# ---------------------------------------------------------------------------
@dataclasses.dataclass
class Qwen2Spec:
    name: str
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    ffn: int
    vocab: int
    context: int = 4096
    rope_theta: float = 1000000.0
    eps: float = 1e-6
    seed: int = 1
    # per-layer tensor types: callable(layer, tensor_name) -> ggml type
    types: Optional[Callable[[int, str], int]] = None
    embed_type: int = Q8_0
    output_type: Optional[int] = None   # None = tied copy of the embedding
    weight_std: float = 0.02


def qwen2_q4km_types(layer: int, tensor: str) -> int:
    """Q4_K_M-style recipe for 7B/14B shapes: Q4_K everywhere except attn_v and
    even-layer ffn_down, which are Q6_K."""
    if tensor == "attn_v":
        return Q6_K
    if tensor == "ffn_down":
        return Q6_K if layer % 2 == 0 else Q4_K
    return Q4_K


def qwen2_05b_types(layer: int, tensor: str) -> int:
    """Q4_K_M layout at hidden 896 (not a multiple of 256): 896-column tensors
    are Q5_0 (attn_v Q8_0); ffn_down (K = 4864) alternates Q6_K / Q4_K."""
    if tensor == "attn_v":
        return Q8_0
    if tensor == "ffn_down":
        return Q6_K if layer % 2 == 0 else Q4_K
    return Q5_0


CONFIGS: Dict[str, Qwen2Spec] = {
    # Qwen2.5-0.5B architecture.
    "qwen2.5-0.5b": Qwen2Spec("qwen2.5-0.5b", hidden=896, layers=24, heads=14, kv_heads=2,
                              ffn=4864, vocab=151936, seed=0x05B, types=qwen2_05b_types,
                              embed_type=Q8_0, output_type=None),
    # Qwen2.5-7B architecture.
    "qwen2.5-7b": Qwen2Spec("qwen2.5-7b", hidden=3584, layers=28, heads=28, kv_heads=4,
                            ffn=18944, vocab=152064, seed=0x7B, types=qwen2_q4km_types,
                            embed_type=Q4_K, output_type=Q6_K),
    # The 7B's widths and formats with 4 layers (1.4 GB): a profiling case that
    # fits a full ncu capture while its weights still exceed the L2.
    "qwen2.5-7b-4l": Qwen2Spec("qwen2.5-7b-4l", hidden=3584, layers=4, heads=28, kv_heads=4,
                               ffn=18944, vocab=152064, seed=0x7B4, types=qwen2_q4km_types,
                               embed_type=Q4_K, output_type=Q6_K),
    # Qwen2.5-14B architecture.
    "qwen2.5-14b": Qwen2Spec("qwen2.5-14b", hidden=5120, layers=48, heads=40, kv_heads=8,
                             ffn=13824, vocab=152064, seed=0x14B, types=qwen2_q4km_types,
                             embed_type=Q4_K, output_type=Q6_K),
}


def q4km_small_spec(seed: int = 0x128, layers: int = 3) -> Qwen2Spec:
    """A small model with the 7B's structure: Q4_K_M layout, head_dim 128,
    7 query heads per KV head (hidden 1792 = 14 x 128, 2 KV heads), ffn 4864."""
    return Qwen2Spec(f"q4km-d128-s{seed}", hidden=1792, layers=layers, heads=14, kv_heads=2,
                     ffn=4864, vocab=8192, context=2048, seed=seed, types=qwen2_q4km_types,
                     embed_type=Q4_K, output_type=Q6_K)


def tiny_mixed_types(layer: int, tensor: str) -> int:
    """Every format on some tensor: even layers K-quants, odd layers 32-blocks."""
    if layer % 2 == 0:
        return {"attn_v": Q6_K, "ffn_down": Q6_K}.get(tensor, Q4_K)
    return {"attn_v": Q8_0, "ffn_down": Q4_K}.get(tensor, Q5_0)


def tiny_spec(seed: int = 7, layers: int = 2, hidden: int = 256, heads: int = 4,
              kv_heads: int = 2, ffn: int = 512, vocab: int = 1024) -> Qwen2Spec:
    return Qwen2Spec(f"tiny-s{seed}", hidden=hidden, layers=layers, heads=heads,
                     kv_heads=kv_heads, ffn=ffn, vocab=vocab, context=256, seed=seed,
                     types=tiny_mixed_types, embed_type=Q8_0, output_type=Q6_K)


def qwen2_tensors(spec: Qwen2Spec) -> List[TensorSpec]:
    H, F, V = spec.hidden, spec.ffn, spec.vocab
    hd = H // spec.heads
    KV = spec.kv_heads * hd
    std = spec.weight_std
    out: List[TensorSpec] = []

    def mat(name, gtype, rows, cols, key_name=None):
        key = stream_key(spec.seed, key_name or name)
        out.append(TensorSpec(name, gtype, (cols, rows),
                              lambda g=gtype, r=rows, c=cols, k=key: fill(g, r, c, k, 0.0, std)))

    def vec(name, n, mean):
        key = stream_key(spec.seed, name)
        out.append(TensorSpec(name, F32, (n,),
                              lambda n=n, k=key, m=mean: normal(n, k, m, std).view(np.uint8)))

    mat("token_embd.weight", spec.embed_type, V, H)
    vec("output_norm.weight", H, 1.0)
    if spec.output_type is None:
        mat("output.weight", spec.embed_type, V, H, key_name="token_embd.weight")
    else:
        mat("output.weight", spec.output_type, V, H)
    types = spec.types or qwen2_q4km_types
    for l in range(spec.layers):
        p = f"blk.{l}."
        vec(p + "attn_norm.weight", H, 1.0)
        mat(p + "attn_q.weight", types(l, "attn_q"), H, H)
        vec(p + "attn_q.bias", H, 0.0)
        mat(p + "attn_k.weight", types(l, "attn_k"), KV, H)
        vec(p + "attn_k.bias", KV, 0.0)
        mat(p + "attn_v.weight", types(l, "attn_v"), KV, H)
        vec(p + "attn_v.bias", KV, 0.0)
        mat(p + "attn_output.weight", types(l, "attn_output"), H, H)
        vec(p + "ffn_norm.weight", H, 1.0)
        mat(p + "ffn_gate.weight", types(l, "ffn_gate"), F, H)
        mat(p + "ffn_up.weight", types(l, "ffn_up"), F, H)
        mat(p + "ffn_down.weight", types(l, "ffn_down"), H, F)
    return out


def qwen2_metadata(spec: Qwen2Spec) -> Dict[str, object]:
    return {
        "general.architecture": "qwen2",
        "general.name": spec.name,
        "qwen2.block_count": spec.layers,
        "qwen2.context_length": spec.context,
        "qwen2.embedding_length": spec.hidden,
        "qwen2.feed_forward_length": spec.ffn,
        "qwen2.attention.head_count": spec.heads,
        "qwen2.attention.head_count_kv": spec.kv_heads,
        "qwen2.rope.freq_base": float(spec.rope_theta),
        "qwen2.attention.layer_norm_rms_epsilon": float(spec.eps),
        "tokenizer.ggml.pre": "qwen2",
        "tokenizer.ggml.tokens_count": spec.vocab,
        "tokenizer.ggml.eos_token_id": min(spec.vocab - 1, 151645),
    }


def write_qwen2(spec: Qwen2Spec, path: str) -> str:
    return write_gguf(path, qwen2_metadata(spec), qwen2_tensors(spec))


def prompt_ids(spec_seed: int, n: int, vocab: int) -> np.ndarray:
    """The seeded uniform random prompt of a config."""
    return uniform_ids(n, stream_key(spec_seed, "prompt"), vocab)


def cached_qwen2(spec: Qwen2Spec, directory: str) -> str:
    """Path of the model file for `spec` under `directory`, writing it once."""
    os.makedirs(directory, exist_ok=True)
    path = os.path.join(directory, f"{spec.name}.gguf")
    if not os.path.exists(path):
        write_qwen2(spec, path)
    return path


# ---------------------------------------------------------------------------
# qwen35moe models (moe_model.cpp:84-247, metal_model.cpp:573-688)
# ---------------------------------------------------------------------------
@dataclasses.dataclass
class MoeSpec:
    name: str
    hidden: int
    layers: int
    experts: int
    experts_used: int
    expert_ffn: int
    shared_ffn: int
    heads: int
    kv_heads: int
    head_dim: int
    rot_dim: int
    ssm_state: int        # DeltaNet head size
    ssm_groups: int       # DeltaNet key heads
    ssm_rank: int         # DeltaNet value heads
    vocab: int
    conv_kernel: int = 4
    attn_interval: int = 4
    context: int = 4096
    rope_theta: float = 10000000.0
    eps: float = 1e-6
    seed: int = 1
    weight_std: float = 0.02

    @property
    def ssm_inner(self) -> int:
        return self.ssm_rank * self.ssm_state

    @property
    def qkv_width(self) -> int:
        return 2 * self.ssm_groups * self.ssm_state + self.ssm_inner

    def is_attention(self, layer: int) -> bool:
        return (layer + 1) % self.attn_interval == 0


def moe_a3b_types(layer: int, tensor: str) -> int:
    """The real Qwen3.6-35B-A3B Q4_K_M recipe (per-tensor types listed in the
    reference's compatibility notes), alternating where the real file mixes
    two types over the layers."""
    odd = layer % 2 == 1
    return {
        "attn_qkv": Q6_K, "attn_gate": Q4_K, "ssm_out": Q8_0 if odd else Q4_K,
        "attn_q": Q6_K if odd else Q4_K, "attn_k": Q8_0, "attn_v": Q8_0, "attn_output": Q5_K,
        "ffn_gate_exps": Q4_K, "ffn_up_exps": Q4_K, "ffn_down_exps": Q6_K if odd else Q4_K,
        "ffn_gate_shexp": Q8_0 if odd else Q6_K, "ffn_up_shexp": Q8_0 if odd else Q6_K,
        "ffn_down_shexp": Q8_0 if odd else Q6_K,
    }[tensor]


MOE_CONFIGS: Dict[str, MoeSpec] = {
    # Qwen3.6-35B-A3B architecture.
    "qwen3.6-35b-a3b": MoeSpec("qwen3.6-35b-a3b", hidden=2048, layers=40, experts=256, experts_used=8,
                               expert_ffn=512, shared_ffn=512, heads=16, kv_heads=2, head_dim=256,
                               rot_dim=64, ssm_state=128, ssm_groups=16, ssm_rank=32, vocab=248320,
                               seed=0x35A3B),
}


def a3b_width_spec(layers: int = 4, vocab: int = 4096, seed: int = 0xA3B4) -> MoeSpec:
    """BASELINE config 4's layer widths (hidden 2048, 256 experts top-8 of
    FFN 512 plus a shared expert, 16 / 2 attention heads of 256 with RoPE on
    64, DeltaNet 16 key / 32 value heads of 128) in fewer layers and a
    smaller vocabulary, so that an FP64 restatement runs it on a CPU: every
    full-width operator of the model, at a fraction of its bytes."""
    return dataclasses.replace(MOE_CONFIGS["qwen3.6-35b-a3b"], name=f"a3b-width-{layers}l", layers=layers,
                               vocab=vocab, context=1024, seed=seed)


def tiny_moe_spec(seed: int = 5, layers: int = 8, experts: int = 16, used: int = 4) -> MoeSpec:
    """Every qwen35moe operator at small sizes (K-quant rows stay 256-aligned)."""
    return MoeSpec(f"tiny-moe-s{seed}", hidden=256, layers=layers, experts=experts, experts_used=used,
                   expert_ffn=256, shared_ffn=256, heads=4, kv_heads=2, head_dim=64, rot_dim=32,
                   ssm_state=64, ssm_groups=2, ssm_rank=4, vocab=1024, context=512, seed=seed)


def moe_tensors(spec: MoeSpec) -> List[TensorSpec]:
    H, V, E = spec.hidden, spec.vocab, spec.experts
    std = spec.weight_std
    out: List[TensorSpec] = []

    def mat(name, gtype, rows, cols, s=std, depth=None):
        key = stream_key(spec.seed, name)
        dims = (cols, rows) if depth is None else (cols, rows, depth)
        total_rows = rows * (depth or 1)
        out.append(TensorSpec(name, gtype, dims,
                              lambda g=gtype, r=total_rows, c=cols, k=key, s=s: fill(g, r, c, k, 0.0, s)))

    def f32mat(name, rows, cols, s):
        key = stream_key(spec.seed, name)
        out.append(TensorSpec(name, F32, (cols, rows),
                              lambda n=rows * cols, k=key, s=s: normal(n, k, 0.0, s).view(np.uint8)))

    def vec(name, n, mean, s=std, transform=None):
        key = stream_key(spec.seed, name)

        def make(n=n, k=key, m=mean, s=s, tr=transform):
            v = normal(n, k, m, s)
            return (tr(v) if tr else v).astype(np.float32).view(np.uint8)
        out.append(TensorSpec(name, F32, (n,), make))

    router_std = 1.0 / float(np.sqrt(H))  # router logits ~ N(0, 1) after the norm
    mat("token_embd.weight", Q4_K, V, H)
    vec("output_norm.weight", H, 1.0)
    mat("output.weight", Q6_K, V, H)
    for l in range(spec.layers):
        p = f"blk.{l}."
        t = lambda name, l=l: moe_a3b_types(l, name)
        vec(p + "attn_norm.weight", H, 1.0)
        vec(p + "post_attention_norm.weight", H, 1.0)
        if spec.is_attention(l):
            qw = spec.heads * spec.head_dim
            kvw = spec.kv_heads * spec.head_dim
            mat(p + "attn_q.weight", t("attn_q"), 2 * qw, H)
            mat(p + "attn_k.weight", t("attn_k"), kvw, H)
            mat(p + "attn_v.weight", t("attn_v"), kvw, H)
            vec(p + "attn_q_norm.weight", spec.head_dim, 1.0)
            vec(p + "attn_k_norm.weight", spec.head_dim, 1.0)
            mat(p + "attn_output.weight", t("attn_output"), H, qw)
        else:
            mat(p + "attn_qkv.weight", t("attn_qkv"), spec.qkv_width, H)
            mat(p + "attn_gate.weight", t("attn_gate"), spec.ssm_inner, H)
            f32mat(p + "ssm_alpha.weight", spec.ssm_rank, H, std)
            f32mat(p + "ssm_beta.weight", spec.ssm_rank, H, std)
            f32mat(p + "ssm_conv1d.weight", spec.qkv_width, spec.conv_kernel, 0.5)
            vec(p + "ssm_dt.bias", spec.ssm_rank, 0.0, 0.1)
            # real files store A = -exp(A_log): negative, so the decay stays below 1
            vec(p + "ssm_a", spec.ssm_rank, 0.0, 0.5, transform=lambda v: -np.exp(v))
            vec(p + "ssm_norm.weight", spec.ssm_state, 1.0)
            mat(p + "ssm_out.weight", t("ssm_out"), H, spec.ssm_inner)
        f32mat(p + "ffn_gate_inp.weight", E, H, router_std)
        mat(p + "ffn_gate_exps.weight", t("ffn_gate_exps"), spec.expert_ffn, H, depth=E)
        mat(p + "ffn_up_exps.weight", t("ffn_up_exps"), spec.expert_ffn, H, depth=E)
        mat(p + "ffn_down_exps.weight", t("ffn_down_exps"), H, spec.expert_ffn, depth=E)
        vec(p + "ffn_gate_inp_shexp.weight", H, 0.0, router_std)
        mat(p + "ffn_gate_shexp.weight", t("ffn_gate_shexp"), spec.shared_ffn, H)
        mat(p + "ffn_up_shexp.weight", t("ffn_up_shexp"), spec.shared_ffn, H)
        mat(p + "ffn_down_shexp.weight", t("ffn_down_shexp"), H, spec.shared_ffn)
    return out


def moe_metadata(spec: MoeSpec) -> Dict[str, object]:
    a = "qwen35moe."
    return {
        "general.architecture": "qwen35moe",
        "general.name": spec.name,
        a + "block_count": spec.layers,
        a + "context_length": spec.context,
        a + "embedding_length": spec.hidden,
        a + "attention.head_count": spec.heads,
        a + "attention.head_count_kv": spec.kv_heads,
        a + "attention.key_length": spec.head_dim,
        a + "attention.value_length": spec.head_dim,
        a + "rope.dimension_count": spec.rot_dim,
        a + "rope.freq_base": float(spec.rope_theta),
        a + "attention.layer_norm_rms_epsilon": float(spec.eps),
        a + "expert_count": spec.experts,
        a + "expert_used_count": spec.experts_used,
        a + "expert_feed_forward_length": spec.expert_ffn,
        a + "expert_shared_feed_forward_length": spec.shared_ffn,
        a + "full_attention_interval": spec.attn_interval,
        a + "ssm.conv_kernel": spec.conv_kernel,
        a + "ssm.state_size": spec.ssm_state,
        a + "ssm.group_count": spec.ssm_groups,
        a + "ssm.time_step_rank": spec.ssm_rank,
        a + "ssm.inner_size": spec.ssm_inner,
        "tokenizer.ggml.pre": "qwen35",
        "tokenizer.ggml.tokens_count": spec.vocab,
        "tokenizer.ggml.eos_token_id": spec.vocab - 1,
    }


def write_moe(spec: MoeSpec, path: str) -> str:
    return write_gguf(path, moe_metadata(spec), moe_tensors(spec))


def cached_moe(spec: MoeSpec, directory: str) -> str:
    os.makedirs(directory, exist_ok=True)
    path = os.path.join(directory, f"{spec.name}.gguf")
    if not os.path.exists(path):
        write_moe(spec, path)
    return path
