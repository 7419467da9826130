"""ctypes bindings of libcudallm.so (include/cudallm_kernels.h, include/cudallm.h).

The library is built in-tree by ``myllm_b200.build``.  There is no fallback:
if it is missing or cannot be loaded, importing the backend raises.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libcudallm.so")

_lib = None

c_int, c_ll, c_size, c_float, c_vp, c_char_p = (ctypes.c_int, ctypes.c_longlong, ctypes.c_size_t,
                                                ctypes.c_float, ctypes.c_void_p, ctypes.c_char_p)


class TpShard(ctypes.Structure):
    """cudallm_tp_shard (include/cudallm.h)."""
    _fields_ = [(n, ctypes.c_uint64) for n in ("q_head0", "q_heads", "kv_head0", "kv_heads", "ffn0", "ffn_rows",
                                               "o_col0", "o_cols", "vocab0", "vocab_rows")] + [
        ("gather_attn", ctypes.c_int32)]


class GemvSegment(ctypes.Structure):
    _fields_ = [("type", c_int), ("w", c_vp), ("stride", c_ll), ("n", c_int), ("bias", c_vp),
                ("residual", c_vp), ("y", c_vp)]


class GemvPackedSegment(ctypes.Structure):
    """cl_gemv_packed_segment (include/cudallm_kernels.h)."""
    _fields_ = [("type", c_int), ("w", c_vp), ("n", c_int), ("bias", c_vp), ("residual", c_vp), ("y", c_vp)]


# name -> (restype, argtypes)
SIGNATURES = {
    "cl_status_string": (c_char_p, [c_int]),
    "cl_set_pdl": (None, [c_int]),
    "cl_native_row_bytes": (c_ll, [c_int, c_int]),
    "cl_row_stride": (c_ll, [c_int, c_int]),
    "cl_repack_rows": (c_int, [c_int, c_vp, c_vp, c_int, c_int, c_vp]),
    "cl_xq_bytes": (c_size, [c_int]),
    "cl_quantize_xq": (c_int, [c_vp, c_int, c_vp, c_vp]),
    "cl_gemv": (c_int, [c_int, c_vp, c_ll, c_int, c_int, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "cl_gemv_multi": (c_int, [ctypes.POINTER(GemvSegment), c_int, c_int, c_vp, c_vp, c_float, c_vp]),
    "cl_gemv_swiglu": (c_int, [c_int, c_vp, c_vp, c_ll, c_int, c_int, c_vp, c_vp, c_float, c_vp, c_vp]),
    "cl_gemv_pack_bytes": (c_size, [c_int, c_int, c_int, c_int]),
    "cl_gemv_pack": (c_int, [c_int, c_vp, c_ll, c_int, c_int, c_vp, c_vp, c_vp]),
    "cl_gemv_packed_workspace_bytes": (c_size, [c_int]),
    "cl_gemv_packed": (c_int, [ctypes.POINTER(GemvPackedSegment), c_int, c_int, c_vp, c_vp, c_float, c_int, c_vp,
                               c_size, c_vp]),
    "cl_device_error": (c_int, [ctypes.POINTER(c_int), c_int]),
    "cl_gemm": (c_int, [c_int, c_vp, c_ll, c_int, c_int, c_vp, c_int, c_vp, c_vp, c_vp, c_vp]),
    "cl_gemm_simt": (c_int, [c_int, c_vp, c_ll, c_int, c_int, c_vp, c_int, c_vp, c_vp, c_vp, c_vp]),
    "cl_gemm_tc": (c_int, [c_int, c_vp, c_ll, c_int, c_int, c_vp, c_int, c_vp, c_vp, c_vp, c_int, c_vp]),
    "cl_rmsnorm": (c_int, [c_vp, c_vp, c_int, c_int, c_float, c_vp, c_vp, c_vp]),
    "cl_embed": (c_int, [c_int, c_vp, c_ll, c_int, c_int, c_vp, c_int, c_vp, c_vp, c_vp]),
    "cl_rope_kv": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_vp, c_vp, c_int,
                           c_vp, c_vp, c_vp]),
    "cl_swiglu": (c_int, [c_vp, c_vp, c_vp, c_ll, c_vp]),
    "cl_add": (c_int, [c_vp, c_vp, c_vp, c_ll, c_vp]),
    "cl_attn_decode_workspace_bytes": (c_size, [c_int, c_int, c_int]),
    "cl_attn_decode": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_float, c_vp, c_vp,
                               c_vp, c_size, c_vp]),
    "cl_attn_decode_rope": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_vp, c_vp, c_int, c_int, c_int, c_int,
                                    c_float, c_vp, c_vp, c_vp, c_size, c_vp]),
    "cl_attn_decode_noalloc_limit_bytes": (c_size, []),
    "cl_attn_decode_noalloc": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_float, c_vp, c_vp]),
    "cl_attn_prefill": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_vp, c_vp]),
    "cl_attn_prefill_tc": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_vp, c_vp]),
    "cl_attn_prefill_tc3": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_vp, c_vp]),
    "cl_argmax_workspace_bytes": (c_size, [c_int]),
    "cl_argmax": (c_int, [c_vp, c_int, c_vp, c_vp, c_size, c_vp]),
    "cl_argmax_ex": (c_int, [c_vp, c_int, c_int, c_vp, c_vp, c_vp, c_size, c_vp]),
    "cl_argmax_merge": (c_int, [c_vp, c_int, c_vp, c_vp]),
    "cl_counter_add": (c_int, [c_vp, c_int, c_int, c_vp]),
    "cl_gemv_f32": (c_int, [c_vp, c_int, c_int, c_vp, c_vp, c_vp]),
    "cl_moe_route": (c_int, [c_vp, c_int, c_int, c_vp, c_vp, c_vp]),
    "cl_moe_expert_gemv": (c_int, [c_int, c_vp, c_vp, c_ll, c_int, c_int, c_vp, c_int, c_vp, c_int, c_int, c_int,
                                   c_vp, c_vp]),
    "cl_moe_combine": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "cl_gdn_prep": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_float, c_vp,
                            c_vp, c_vp, c_vp]),
    "cl_gdn_step": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_float, c_vp, c_vp]),
    "cl_attn_gate_prep": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_vp, c_vp, c_float,
                                  c_vp, c_vp, c_vp, c_vp, c_vp]),
    "cl_mul_sigmoid": (c_int, [c_vp, c_vp, c_vp, c_int, c_vp]),
    "cl_select_token": (c_int, [c_vp, c_vp, c_vp, c_vp]),
    "cl_peer_exchange_bytes": (c_size, [c_int]),
    "cl_peer_exchange_init": (c_int, [c_vp, c_int, c_vp]),
    "cl_peer_exchange_status": (c_vp, [c_vp]),
    "cl_peer_allreduce": (c_int, [c_vp, c_vp, c_int, c_int, c_int, c_int, c_vp, c_vp]),
    "cl_peer_set_wait_limit_ns": (c_int, [ctypes.c_ulonglong]),
    "cl_dequant16": (c_int, [c_int, c_vp, c_ll, c_int, c_int, c_vp, c_int, c_vp]),
    "cl_convert16": (c_int, [c_vp, c_ll, c_vp, c_int, c_vp]),
    "cl_split16": (c_int, [c_vp, c_int, c_int, c_vp, c_vp, c_vp]),
    "cl_moe_route_rows": (c_int, [c_vp, c_int, c_int, c_int, c_vp, c_vp, c_vp]),
    "cl_moe_expert_gemv_rows": (c_int, [c_int, c_vp, c_vp, c_ll, c_int, c_int, c_vp, c_int, c_int, c_vp, c_int,
                                        c_int, c_int, c_vp, c_vp]),
    "cl_moe_xq_planes_bytes": (c_size, [c_int, c_int]),
    "cl_moe_group_routes": (c_int, [c_vp, c_int, c_int, c_int, c_int, c_vp, c_vp, c_vp]),
    "cl_moe_expert_gemv_grouped": (c_int, [c_int, c_vp, c_vp, c_ll, c_int, c_int, c_vp, c_int, c_int, c_vp, c_int,
                                           c_int, c_int, c_vp, c_vp, c_int, c_vp, c_size, c_vp, c_vp]),
    "cl_moe_combine_rows": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_vp, c_vp, c_vp, c_vp, c_int,
                                    c_vp]),
    "cl_gdn_prep_rows": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_float,
                                 c_int, c_vp, c_vp, c_vp, c_vp]),
    "cl_gdn_step_rows": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_float, c_int, c_vp,
                                 c_vp]),
    "cl_attn_gate_prep_rows": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_vp, c_int,
                                       c_int, c_float, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "cl_amax": (c_int, [c_vp, c_ll, c_vp, c_vp]),
    "cl_amax_dequant": (c_int, [c_int, c_vp, c_ll, c_int, c_int, c_vp, c_vp]),
    "cl_dequant16_split": (c_int, [c_int, c_vp, c_ll, c_int, c_int, c_vp, c_vp, c_vp]),
    "cl_gemm16_workspace_bytes": (c_size, [c_int, c_int, c_int]),
    "cl_gemm16_run": (c_int, [c_vp, c_int, c_int, c_vp, c_int, c_vp, c_int, c_int, c_vp, c_size, c_vp]),
    "cl_decode_pack_bytes": (c_size, [c_int, c_int, c_int, c_int]),
    "cl_decode_pack": (c_int, [c_int, c_vp, c_ll, c_int, c_int, c_vp, c_vp, c_vp]),
    "cl_qwen2_decode_supported": (c_int, [c_vp, c_vp]),
    "cl_qwen2_decode_workspace_bytes": (c_size, [c_vp]),
    "cl_qwen2_decode_init": (c_int, [c_vp, c_size, c_vp]),
    "cl_qwen2_decode_step": (c_int, [c_vp, c_vp, c_vp, c_size, c_vp]),
    "cl_qwen2_decode_status": (c_vp, [c_vp]),
    # backend
    "cudallm_last_error": (c_char_p, []),
    "cudallm_nccl_unique_id": (c_int, [c_vp]),
    "cudallm_create": (c_int, [c_char_p, c_size, c_int, c_int, c_int, c_vp, ctypes.POINTER(c_vp)]),
    "cudallm_destroy": (None, [c_vp]),
    "cudallm_reset": (c_int, [c_vp]),
    "cudallm_prefill": (c_int, [c_vp, c_vp, c_size, ctypes.POINTER(ctypes.c_int32)]),
    "cudallm_decode": (c_int, [c_vp, ctypes.c_int32, ctypes.POINTER(ctypes.c_int32)]),
    "cudallm_last_logits": (c_int, [c_vp, c_vp, c_size]),
    "cudallm_last_call_ms": (c_float, [c_vp]),
    "cudallm_last_kernel_ms": (c_float, [c_vp]),
    "cudallm_position": (c_size, [c_vp]),
    "cudallm_max_sequence": (c_size, [c_vp]),
    "cudallm_config": (c_int, [c_vp, ctypes.POINTER(c_ll), c_int]),
    "cudallm_memory_stats": (c_int, [c_vp, ctypes.POINTER(ctypes.c_uint64)]),
    "cudallm_enable_profiling": (c_int, [c_vp, c_char_p]),
    "cudallm_disable_profiling": (c_int, [c_vp]),
    "cudallm_device_name": (c_int, [c_vp, c_vp, c_size]),
    "cudallm_available": (c_int, [c_vp]),
    "cudallm_expert_cache": (c_int, [c_vp, ctypes.POINTER(ctypes.c_uint64)]),
    "cudallm_gguf_inspect": (c_int, [c_char_p, c_vp, c_size, c_vp]),
    "cudallm_tp_plan": (c_int, [ctypes.c_uint64] * 6 + [c_int, c_int, c_vp]),
    "cudallm_ep_plan": (c_int, [ctypes.c_uint64, ctypes.c_uint64, c_int, c_vp, c_vp, c_vp]),
}


class GemmOut(ctypes.Structure):
    """cl_gemm_out of cudallm_kernels.h: one column range of a cl_gemm16_run product."""
    _fields_ = [("y", c_vp), ("bias", c_vp), ("residual", c_vp), ("xmax", c_vp), ("wmax", c_vp), ("col0", c_int),
                ("cols", c_int), ("ld", c_int)]


class Qwen2Layer(ctypes.Structure):
    """cl_qwen2_layer of cudallm_kernels.h: one layer of the one-launch decode step."""
    _fields_ = ([(n, c_vp) for n in ("q", "k", "v", "o", "gate", "up", "down", "q_bias", "k_bias", "v_bias",
                                    "attn_norm", "ffn_norm", "k_cache", "v_cache")] +
                [(n, c_int) for n in ("q_type", "k_type", "v_type", "o_type", "gate_type", "down_type")] +
                [("reserved", c_int * 2)])


class Qwen2Decode(ctypes.Structure):
    """cl_qwen2_decode of cudallm_kernels.h: the model of the one-launch decode step."""
    _fields_ = ([("layers", c_vp)] +
                [(n, c_int) for n in ("n_layers", "hidden", "ffn", "vocab", "q_heads", "kv_heads", "head_dim",
                                      "capacity")] +
                [("eps", c_float), ("scale", c_float), ("embd", c_vp), ("embd_stride", c_ll), ("embd_type", c_int),
                 ("out_type", c_int), ("out_w", c_vp), ("out_norm", c_vp), ("rope", c_vp), ("ints", c_vp)] +
                [(n, c_vp) for n in ("h", "q", "k", "v", "att", "act", "logits", "trace")] +
                [("attn_splits", c_int)])


def lib():
    """The loaded library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m myllm_b200.build`")
        l = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(l, name)
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


class KernelError(RuntimeError):
    pass


def check(status: int, what: str = "") -> None:
    if status != 0:
        msg = lib().cl_status_string(status).decode()
        raise KernelError(f"{what}: {msg} (status {status})")
