"""Python mirror of the backend contract (cpu_llm.h:167-194, metal_llm.h:20-51).

``CudaLLM(path, max_sequence=0)`` behaves like the reference's ``CPULLM``:
``reset()``, ``prefill(ids) -> token``, ``decode(id) -> token``,
``position``, ``max_sequence``, ``memory_stats()``, ``uses_gpu()`` and
profiling switches, with the reference's error conventions mapped to Python
exceptions:

==========================  ==========================
reference C++ exception     raised here
==========================  ==========================
std::invalid_argument       :class:`InvalidArgument` (ValueError)
std::out_of_range           :class:`OutOfRange` (IndexError)
std::length_error           :class:`LengthError` (ValueError)
std::runtime_error          :class:`BackendError` (RuntimeError)
==========================  ==========================

All work happens in ``libcudallm.so``; nothing here computes.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

from . import _native


class InvalidArgument(ValueError):
    pass


class OutOfRange(IndexError):
    pass


class LengthError(ValueError):
    pass


class BackendError(RuntimeError):
    pass


_ERRORS = {1: InvalidArgument, 2: OutOfRange, 3: LengthError, 4: BackendError}


def _check(rc: int) -> None:
    if rc != 0:
        msg = _native.lib().cudallm_last_error().decode()
        raise _ERRORS.get(rc, BackendError)(msg)


@dataclass
class MemoryStats:
    weight_bytes: int
    kv_cache_bytes: int
    recurrent_state_bytes: int
    intermediate_bytes: int
    intermediate_is_estimate: bool = False

    def total_bytes(self) -> int:
        return self.weight_bytes + self.kv_cache_bytes + self.recurrent_state_bytes + self.intermediate_bytes


@dataclass
class ExpertCacheStats:
    """ExpertCacheStats of the reference's MoeLLM (moe_llm.h:9-17)."""
    hits: int
    misses: int

    def requests(self) -> int:
        return self.hits + self.misses


@dataclass
class ModelConfig:
    layer_count: int
    embedding_size: int
    feed_forward_size: int
    attention_head_count: int
    kv_head_count: int
    head_size: int
    vocabulary_size: int
    context_length: int


def nccl_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    _check(_native.lib().cudallm_nccl_unique_id(buf))
    return buf.raw


@dataclass
class TensorParallelShard:
    """One rank's share of a tensor-parallel qwen2 model (``cudallm_tp_plan``):
    half-open ranges of query / KV heads, FFN rows (= ffn_down input columns),
    o_proj input columns (of the all-gathered attention output when
    ``gather_attn``) and LM-head rows."""
    q_heads: range
    kv_heads: range
    ffn_rows: range
    o_cols: range
    vocab_rows: range
    gather_attn: bool


def tp_plan(feed_forward: int, vocabulary: int, heads: int, kv_heads: int, head_size: int, o_block: int,
            world: int, rank: int) -> TensorParallelShard:
    """The shard ``CudaLLM(..., rank=rank, world=world)`` loads (no GPU needed).
    ``o_block`` is the widest column block of the layers' attn_output types."""
    s = _native.TpShard()
    _check(_native.lib().cudallm_tp_plan(feed_forward, vocabulary, heads, kv_heads, head_size, o_block, world, rank,
                                         ctypes.byref(s)))
    r = lambda a, n: range(a, a + n)  # noqa: E731
    return TensorParallelShard(r(s.q_head0, s.q_heads), r(s.kv_head0, s.kv_heads), r(s.ffn0, s.ffn_rows),
                               r(s.o_col0, s.o_cols), r(s.vocab0, s.vocab_rows), bool(s.gather_attn))


def ep_plan(experts: int, layers: int, world: int):
    """Expert-parallel placement (``cudallm_ep_plan``): arrays (rank of each
    routed expert, its index in that rank's stacked expert tensors, rank of
    each layer's shared expert)."""
    er = np.empty(experts, dtype=np.int32)
    el = np.empty(experts, dtype=np.int32)
    sr = np.empty(layers, dtype=np.int32)
    _check(_native.lib().cudallm_ep_plan(experts, layers, world, er.ctypes.data, el.ctypes.data, sr.ctypes.data))
    return er, el, sr


class CudaLLM:
    """qwen2 GGUF model on one GPU, or tensor-parallel over ``world`` GPUs."""

    def __init__(self, gguf_path: str, max_sequence: int = 0, device: int = -1, rank: int = 0,
                 world: int = 1, nccl_id: Optional[bytes] = None):
        L = _native.lib()
        self._h = ctypes.c_void_p()
        idbuf = None
        if world > 1:
            if nccl_id is None or len(nccl_id) != 128:
                raise InvalidArgument("world > 1 needs the 128-byte NCCL unique id")
            idbuf = ctypes.create_string_buffer(nccl_id, 128)
        _check(L.cudallm_create(gguf_path.encode(), max_sequence, device, rank, world, idbuf,
                                ctypes.byref(self._h)))
        cfg = (ctypes.c_longlong * 8)()
        _check(L.cudallm_config(self._h, cfg, 8))
        self._config = ModelConfig(*[int(v) for v in cfg])

    def close(self) -> None:
        if getattr(self, "_h", None):
            _native.lib().cudallm_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # ---- contract -----------------------------------------------------------
    def reset(self) -> None:
        _check(_native.lib().cudallm_reset(self._h))

    def prefill(self, token_ids: Sequence[int]) -> int:
        ids = np.ascontiguousarray(np.asarray(token_ids, dtype=np.int64))
        if ids.size and (ids.min() < -2**31 or ids.max() >= 2**31):
            raise OutOfRange("token id does not fit in int32")
        ids = ids.astype(np.int32)
        tok = ctypes.c_int32()
        _check(_native.lib().cudallm_prefill(self._h, ids.ctypes.data if ids.size else None, ids.size,
                                             ctypes.byref(tok)))
        return tok.value

    def decode(self, token_id: int) -> int:
        if not -2**31 <= int(token_id) < 2**31:
            raise OutOfRange("token id does not fit in int32")
        tok = ctypes.c_int32()
        _check(_native.lib().cudallm_decode(self._h, int(token_id), ctypes.byref(tok)))
        return tok.value

    def enable_profiling(self, csv_path: str) -> None:
        _check(_native.lib().cudallm_enable_profiling(self._h, csv_path.encode()))

    def disable_profiling(self) -> None:
        _check(_native.lib().cudallm_disable_profiling(self._h))

    # ---- queries ------------------------------------------------------------
    def config(self) -> ModelConfig:
        return self._config

    @property
    def position(self) -> int:
        return int(_native.lib().cudallm_position(self._h))

    @property
    def max_sequence(self) -> int:
        return int(_native.lib().cudallm_max_sequence(self._h))

    def uses_gpu(self) -> bool:
        return True

    def available(self) -> bool:
        return bool(_native.lib().cudallm_available(self._h))

    def _expert_cache(self):
        out = (ctypes.c_uint64 * 3)()
        _check(_native.lib().cudallm_expert_cache(self._h, out))
        return [int(v) for v in out]

    def expert_cache_count(self) -> int:
        """qwen35moe: experts resident per layer on this rank (all of them); 0 for qwen2."""
        return self._expert_cache()[0]

    def expert_cache_stats(self) -> ExpertCacheStats:
        _, hits, misses = self._expert_cache()
        return ExpertCacheStats(hits, misses)

    def memory_stats(self) -> MemoryStats:
        out = (ctypes.c_uint64 * 4)()
        _check(_native.lib().cudallm_memory_stats(self._h, out))
        return MemoryStats(*[int(v) for v in out])

    def device_name(self) -> str:
        buf = ctypes.create_string_buffer(256)
        _check(_native.lib().cudallm_device_name(self._h, buf, 256))
        return buf.value.decode()

    def last_logits(self) -> np.ndarray:
        out = np.empty(self._config.vocabulary_size, dtype=np.float32)
        _check(_native.lib().cudallm_last_logits(self._h, out.ctypes.data, out.size))
        return out

    def last_call_ms(self) -> float:
        return float(_native.lib().cudallm_last_call_ms(self._h))

    def last_kernel_ms(self) -> float:
        """Device time of the last decode's one-launch step kernel alone (0
        when the decode ran as the per-operator graph)."""
        return float(_native.lib().cudallm_last_kernel_ms(self._h))
