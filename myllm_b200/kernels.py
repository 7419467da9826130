"""Torch-tensor front end of the kernel C-ABI (include/cudallm_kernels.h).

PyTorch only supplies device memory and the current stream; every call lands
in an sm_100a kernel of libcudallm.so.  Used by the GPU parity tests and the
kernel benchmarks.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence

import numpy as np
import torch

from . import _native
from ._native import check

F32, F16, Q5_0, Q8_0, Q4_K, Q5_K, Q6_K = 0, 1, 6, 8, 12, 13, 14


def _p(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def row_stride(gtype: int, k: int) -> int:
    s = _native.lib().cl_row_stride(gtype, k)
    if s < 0:
        raise ValueError(f"type {gtype} cannot hold rows of {k} columns")
    return int(s)


def native_row_bytes(gtype: int, k: int) -> int:
    return int(_native.lib().cl_native_row_bytes(gtype, k))


def repack(gtype: int, native: np.ndarray, k: int, device="cuda") -> torch.Tensor:
    """Native GGML rows (uint8 [rows, row_bytes]) -> device layout [rows, stride]."""
    native = np.ascontiguousarray(native, dtype=np.uint8)
    rows = native.shape[0]
    src = torch.from_numpy(native).to(device)
    dst = torch.empty((rows, row_stride(gtype, k)), dtype=torch.uint8, device=device)
    check(_native.lib().cl_repack_rows(gtype, _p(src), _p(dst), rows, k, _stream()), "cl_repack_rows")
    return dst


def xq_bytes(k: int) -> int:
    return int(_native.lib().cl_xq_bytes(k))


def quantize_xq(x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    k = x.numel()
    if out is None:
        out = torch.empty(xq_bytes(k), dtype=torch.uint8, device=x.device)
    check(_native.lib().cl_quantize_xq(_p(x), k, _p(out), _stream()), "cl_quantize_xq")
    return out


def gemv(gtype: int, w: torch.Tensor, n: int, k: int, x: torch.Tensor, bias=None, residual=None,
         out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = W x (+ bias) (+ residual) with the TMA-staged decode GEMV."""
    if out is None:
        out = torch.empty(n, dtype=torch.float32, device=w.device)
    check(_native.lib().cl_gemv(gtype, _p(w), w.stride(0), n, k, _p(x), _p(bias), _p(residual), _p(out),
                                _stream()), "cl_gemv")
    return out


def gemv_multi(segments: Sequence[tuple], k: int, x: torch.Tensor, gamma=None, eps: float = 1e-6) -> None:
    """segments: (gtype, w, n, bias, residual, out) tuples sharing x (RMS-normalised by gamma if given)."""
    arr = (_native.GemvSegment * len(segments))()
    for i, (gtype, w, n, bias, res, out) in enumerate(segments):
        arr[i] = _native.GemvSegment(gtype, w.data_ptr(), w.stride(0), n,
                                     0 if bias is None else bias.data_ptr(),
                                     0 if res is None else res.data_ptr(), out.data_ptr())
    check(_native.lib().cl_gemv_multi(arr, len(segments), k, _p(x), _p(gamma), eps, _stream()), "cl_gemv_multi")


def gemv_swiglu(gtype: int, w_gate: torch.Tensor, w_up: torch.Tensor, n: int, k: int, x: torch.Tensor,
                gamma=None, eps: float = 1e-6):
    out = torch.empty(n, dtype=torch.float32, device=w_gate.device)
    check(_native.lib().cl_gemv_swiglu(gtype, _p(w_gate), _p(w_up), w_gate.stride(0), n, k, _p(x), _p(gamma), eps,
                                       _p(out), _stream()), "cl_gemv_swiglu")
    return out


def gemv_pack(gtype: int, w: torch.Tensor, n: int, k: int, w_up: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Device-layout rows (repack) -> the fragment-packed layout of cl_gemv_packed
    (with w_up: gate/up pair units for the SwiGLU form)."""
    nbytes = _native.lib().cl_gemv_pack_bytes(gtype, n, k, 0 if w_up is None else 1)
    if nbytes == 0:
        raise ValueError("cl_gemv_pack: unsupported type or shape")
    out = torch.empty(nbytes, dtype=torch.uint8, device=w.device)
    check(_native.lib().cl_gemv_pack(gtype, _p(w), w.stride(0), n, k, _p(w_up), _p(out), _stream()), "cl_gemv_pack")
    return out


def gemv_packed_workspace(max_tiles: int, device="cuda") -> torch.Tensor:
    """A zeroed workspace for cl_gemv_packed launches of up to max_tiles tiles."""
    return torch.zeros(_native.lib().cl_gemv_packed_workspace_bytes(max_tiles), dtype=torch.uint8, device=device)


def gemv_packed(segments: Sequence[tuple], k: int, x: torch.Tensor, gamma=None, eps: float = 1e-6,
                swiglu: bool = False, ws: Optional[torch.Tensor] = None) -> None:
    """segments: (gtype, packed w, n, bias, residual, out) tuples sharing x (RMS-normalised by
    gamma if given); swiglu: one pair-packed (gate, up) matrix, out = SiLU(gate.x) * (up.x)."""
    arr = (_native.GemvPackedSegment * len(segments))()
    tiles = 0
    for i, (gtype, w, n, bias, res, out) in enumerate(segments):
        arr[i] = _native.GemvPackedSegment(gtype, w.data_ptr(), n, 0 if bias is None else bias.data_ptr(),
                                           0 if res is None else res.data_ptr(), out.data_ptr())
        tiles += (n + 7) // 8 if swiglu else (n + 15) // 16
    if ws is None:
        ws = gemv_packed_workspace(tiles, x.device)
    check(_native.lib().cl_gemv_packed(arr, len(segments), k, _p(x), _p(gamma), eps, 1 if swiglu else 0, _p(ws),
                                       ws.numel(), _stream()), "cl_gemv_packed")


def device_error(clear: bool = True) -> int:
    code = ctypes.c_int(0)
    check(_native.lib().cl_device_error(ctypes.byref(code), 1 if clear else 0), "cl_device_error")
    return code.value


GEMM_TF32X3, GEMM_F16, GEMM_BF16, GEMM_F16X3 = 0, 1, 2, 3


def dequant16(gtype: int, w: torch.Tensor, n: int, k: int, fmt: int = GEMM_F16):
    """Device-layout rows -> row-major [n, k] FP16 / BF16 (cl_dequant16); the
    split form (GEMM_F16X3) -> ([n, 2k] FP16 rows [hi | lo] of the scaled
    values, the device maximum that set the scale) (cl_amax_dequant,
    cl_dequant16_split)."""
    lib = _native.lib()
    if fmt == GEMM_F16X3:
        amax = torch.empty(1, dtype=torch.float32, device=w.device)
        check(lib.cl_amax_dequant(gtype, _p(w), w.stride(0), n, k, _p(amax), _stream()), "cl_amax_dequant")
        out = torch.empty((n, 2 * k), dtype=torch.float16, device=w.device)
        check(lib.cl_dequant16_split(gtype, _p(w), w.stride(0), n, k, _p(amax), _p(out), _stream()),
              "cl_dequant16_split")
        return out, amax
    out = torch.empty((n, k), dtype=torch.bfloat16 if fmt == GEMM_BF16 else torch.float16, device=w.device)
    check(lib.cl_dequant16(gtype, _p(w), w.stride(0), n, k, _p(out), fmt, _stream()), "cl_dequant16")
    return out


def convert16(x: torch.Tensor, fmt: int = GEMM_F16):
    """FP32 [m, k] -> FP16 / BF16 (cl_convert16), or, split, ([m, 2k] rows
    [hi | lo] of the scaled values, the device maximum) (cl_amax, cl_split16)."""
    if fmt == GEMM_F16X3:
        m, k = x.shape
        lib = _native.lib()
        amax = torch.empty(1, dtype=torch.float32, device=x.device)
        check(lib.cl_amax(_p(x), x.numel(), _p(amax), _stream()), "cl_amax")
        out = torch.empty((m, 2 * k), dtype=torch.float16, device=x.device)
        check(lib.cl_split16(_p(x), m, k, _p(amax), _p(out), _stream()), "cl_split16")
        return out, amax
    out = torch.empty(x.shape, dtype=torch.bfloat16 if fmt == GEMM_BF16 else torch.float16, device=x.device)
    check(_native.lib().cl_convert16(_p(x), x.numel(), _p(out), fmt, _stream()), "cl_convert16")
    return out


def gemm16_run(w16: torch.Tensor, x16: torch.Tensor, outs, fmt: int = GEMM_F16, split: bool = True) -> None:
    """cl_gemm16_run over column ranges: outs = [(y, bias, residual, col0, cols)]
    with y row-major [m, cols]; for GEMM_F16X3, w16 and x16 are the pairs
    dequant16 / convert16 return."""
    xmax = wmax = None
    if fmt == GEMM_F16X3:  # (rows [hi | lo], device maximum) pairs
        (w16, wm), (x16, xm) = w16, x16
        xmax, wmax = xm.data_ptr(), wm.data_ptr()
    n, k = w16.shape
    if fmt == GEMM_F16X3:
        k //= 2
    m = x16.shape[0]
    arr = (_native.GemmOut * len(outs))()
    for i, (y, bias, res, col0, cols) in enumerate(outs):
        arr[i] = _native.GemmOut(y.data_ptr(), bias.data_ptr() if bias is not None else None,
                                 res.data_ptr() if res is not None else None, xmax, wmax, col0, cols, y.stride(0))
    lib = _native.lib()
    wsb = int(lib.cl_gemm16_workspace_bytes(m, n, k)) if split else 0
    ws = torch.empty(wsb, dtype=torch.uint8, device=x16.device) if wsb else None
    check(lib.cl_gemm16_run(_p(w16), n, k, _p(x16), m, arr, len(outs), fmt, _p(ws), wsb, _stream()),
          "cl_gemm16_run")


def gemm16(gtype: int, w: torch.Tensor, n: int, k: int, x: torch.Tensor, bias=None, residual=None,
           fmt: int = GEMM_F16, split: bool = True) -> torch.Tensor:
    """Y = X W^T (+bias) (+residual) on the 16-bit tensor-core path."""
    m = x.shape[0]
    y = torch.empty((m, n), dtype=torch.float32, device=x.device)
    gemm16_run(dequant16(gtype, w, n, k, fmt), convert16(x, fmt), [(y, bias, residual, 0, n)], fmt, split)
    return y


def gemm(gtype: int, w: torch.Tensor, n: int, k: int, x: torch.Tensor, bias=None, residual=None, path="auto",
         out=None):
    """Y = X W^T (+bias) (+residual).  path: "auto" (cl_gemm), "simt", "tf32x3" or "f16"."""
    m = x.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=x.device)
    lib = _native.lib()
    args = (gtype, _p(w), w.stride(0), n, k, _p(x), m, _p(bias), _p(residual), _p(out))
    if path == "auto":
        check(lib.cl_gemm(*args, _stream()), "cl_gemm")
    elif path == "simt":
        check(lib.cl_gemm_simt(*args, _stream()), "cl_gemm_simt")
    else:
        prec = {"tf32x3": GEMM_TF32X3, "f16": GEMM_F16}[path]
        check(lib.cl_gemm_tc(*args, prec, _stream()), "cl_gemm_tc")
    return out


def rmsnorm(x: torch.Tensor, gamma: torch.Tensor, eps: float, want_xq: bool = False):
    rows, k = x.shape
    y = torch.empty_like(x)
    xq = torch.empty(rows * xq_bytes(k), dtype=torch.uint8, device=x.device) if want_xq else None
    check(_native.lib().cl_rmsnorm(_p(x), _p(gamma), rows, k, eps, _p(y), _p(xq), _stream()), "cl_rmsnorm")
    return (y, xq) if want_xq else y


def embed(gtype: int, table: torch.Tensor, vocab: int, k: int, ids: torch.Tensor):
    out = torch.empty((ids.numel(), k), dtype=torch.float32, device=ids.device)
    flag = torch.zeros(1, dtype=torch.int32, device=ids.device)
    check(_native.lib().cl_embed(gtype, _p(table), table.stride(0), vocab, k, _p(ids), ids.numel(), _p(out),
                                 _p(flag), _stream()), "cl_embed")
    return out, flag


def rope_kv(q, k, v, rows, hq, hkv, d, rot, table, pos: int, k_cache, v_cache, pos_dev=None):
    check(_native.lib().cl_rope_kv(_p(q), _p(k), _p(v), rows, hq, hkv, d, rot, _p(table), _p(pos_dev), pos,
                                   _p(k_cache), _p(v_cache), _stream()), "cl_rope_kv")


def attn_decode(q, k_cache, v_cache, length: int, max_len: int, hq, hkv, d, scale, want_xq=False):
    dev = q.device
    out = torch.empty(hq * d, dtype=torch.float32, device=dev)
    wsb = int(_native.lib().cl_attn_decode_workspace_bytes(hq, d, max_len))
    ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
    ln = torch.tensor([length], dtype=torch.int32, device=dev)
    xq = torch.empty(xq_bytes(hq * d), dtype=torch.uint8, device=dev) if want_xq else None
    check(_native.lib().cl_attn_decode(_p(q), _p(k_cache), _p(v_cache), _p(ln), max_len, hq, hkv, d, scale,
                                       _p(out), _p(xq), _p(ws), wsb, _stream()), "cl_attn_decode")
    return (out, xq) if want_xq else out


def attn_decode_rope(q, k_new, v_new, cos_sin, pos: int, rot: int, k_cache, v_cache, max_len: int, hq, hkv, d,
                     scale):
    """RoPE at `pos` + KV append + decode attention over keys 0..pos in one call."""
    dev = q.device
    out = torch.empty(hq * d, dtype=torch.float32, device=dev)
    wsb = int(_native.lib().cl_attn_decode_workspace_bytes(hq, d, max_len))
    ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
    pd = torch.tensor([pos], dtype=torch.int32, device=dev)
    check(_native.lib().cl_attn_decode_rope(_p(q), _p(k_new), _p(v_new), _p(cos_sin), _p(pd), rot, _p(k_cache),
                                            _p(v_cache), max_len, hq, hkv, d, scale, _p(out), None, _p(ws), wsb,
                                            _stream()), "cl_attn_decode_rope")
    return out


def attn_prefill(q, k_cache, v_cache, pos0: int, rows: int, hq, hkv, d, tensor_cores=False):
    """Causal prefill attention: FP32 CUDA cores, the FP16 tensor-core kernel
    (tensor_cores=True), or its split-FP16 FP32-grade form (tensor_cores="split")."""
    out = torch.empty((rows, hq * d), dtype=torch.float32, device=q.device)
    lib = _native.lib()
    fn = lib.cl_attn_prefill_tc3 if tensor_cores == "split" else lib.cl_attn_prefill_tc if tensor_cores \
        else lib.cl_attn_prefill
    check(fn(_p(q), _p(k_cache), _p(v_cache), pos0, rows, hq, hkv, d, _p(out), _stream()), "cl_attn_prefill")
    return out


def argmax_workspace(n: int, device="cuda") -> torch.Tensor:
    """Zeroed argmax workspace (the kernel re-arms it after every call)."""
    return torch.zeros(int(_native.lib().cl_argmax_workspace_bytes(n)), dtype=torch.uint8, device=device)


def argmax(x: torch.Tensor, ws: Optional[torch.Tensor] = None) -> torch.Tensor:
    n = x.numel()
    if ws is None:
        ws = argmax_workspace(n, x.device)
    tok = torch.empty(1, dtype=torch.int32, device=x.device)
    check(_native.lib().cl_argmax(_p(x), n, _p(tok), _p(ws), ws.numel(), _stream()), "cl_argmax")
    return tok


def swiglu(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    out = torch.empty_like(g)
    check(_native.lib().cl_swiglu(_p(g), _p(u), _p(out), g.numel(), _stream()), "cl_swiglu")
    return out


# ---- qwen35moe -----------------------------------------------------------------
def gemv_f32(w: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    n, k = w.shape
    y = torch.empty(n, dtype=torch.float32, device=x.device)
    check(_native.lib().cl_gemv_f32(_p(w), n, k, _p(x), _p(y), _stream()), "cl_gemv_f32")
    return y


def moe_route(logits: torch.Tensor, k: int):
    ids = torch.empty(k, dtype=torch.int32, device=logits.device)
    wts = torch.empty(k, dtype=torch.float32, device=logits.device)
    check(_native.lib().cl_moe_route(_p(logits), logits.numel(), k, _p(ids), _p(wts), _stream()), "cl_moe_route")
    return ids, wts


def moe_expert_gemv(gtype: int, w: torch.Tensor, n: int, k: int, x: torch.Tensor, ids: torch.Tensor,
                    x_stride: int = 0, w_up=None, rank: int = 0, world: int = 1, out=None):
    routes = ids.numel()
    y = out if out is not None else torch.zeros((routes, n), dtype=torch.float32, device=x.device)
    check(_native.lib().cl_moe_expert_gemv(gtype, _p(w), _p(w_up), w.stride(0), n, k, _p(x), x_stride, _p(ids),
                                           routes, rank, world, _p(y), _stream()), "cl_moe_expert_gemv")
    return y


def moe_expert_gemv_rows(gtype: int, w: torch.Tensor, n: int, k: int, x: torch.Tensor, ids: torch.Tensor,
                         x_stride: int, x_group: int, w_up=None, rank: int = 0, world: int = 1, out=None):
    """Prefill form: route r reads input row r // x_group (rows x_stride apart)."""
    routes = ids.numel()
    y = out if out is not None else torch.zeros((routes, n), dtype=torch.float32, device=x.device)
    check(_native.lib().cl_moe_expert_gemv_rows(gtype, _p(w), _p(w_up), w.stride(0), n, k, _p(x), x_stride, x_group,
                                                _p(ids), routes, rank, world, _p(y), _stream()),
          "cl_moe_expert_gemv_rows")
    return y


def moe_group_routes(ids: torch.Tensor, n_local: int, rank: int = 0, world: int = 1):
    """(offsets [n_local + 1], list [routes]) of this rank's routes by local expert."""
    routes = ids.numel()
    offsets = torch.empty(n_local + 1, dtype=torch.int32, device=ids.device)
    lst = torch.empty(routes, dtype=torch.int32, device=ids.device)
    check(_native.lib().cl_moe_group_routes(_p(ids), routes, n_local, rank, world, _p(offsets), _p(lst), _stream()),
          "cl_moe_group_routes")
    return offsets, lst


def moe_expert_gemv_grouped(gtype: int, w: torch.Tensor, n: int, k: int, x: torch.Tensor, ids: torch.Tensor,
                            x_stride: int, x_group: int, n_local: int, w_up=None, rank: int = 0, world: int = 1,
                            groups=None, planes=None, out=None):
    """The grouped prefill expert GEMV; `groups` = moe_group_routes(...) over
    the same ids (made here when None), `planes` its scratch (made when None)."""
    routes = ids.numel()
    if groups is None:
        groups = moe_group_routes(ids, n_local, rank, world)
    nbytes = int(_native.lib().cl_moe_xq_planes_bytes((routes + x_group - 1) // x_group, k))
    if planes is None:
        planes = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=x.device)
    y = out if out is not None else torch.zeros((routes, n), dtype=torch.float32, device=x.device)
    check(_native.lib().cl_moe_expert_gemv_grouped(gtype, _p(w), _p(w_up), w.stride(0), n, k, _p(x), x_stride,
                                                   x_group, _p(ids), routes, rank, world, _p(groups[0]),
                                                   _p(groups[1]), n_local, _p(planes), planes.numel(), _p(y),
                                                   _stream()), "cl_moe_expert_gemv_grouped")
    return y


def moe_combine(y: torch.Tensor, ids, wts, shared_y=None, shared_logit=None, residual=None, rank=0, world=1):
    routes, n = y.shape
    out = torch.empty(n, dtype=torch.float32, device=y.device)
    check(_native.lib().cl_moe_combine(_p(y), _p(ids), _p(wts), routes, n, rank, world, _p(shared_y),
                                       _p(shared_logit), _p(residual), _p(out), _stream()), "cl_moe_combine")
    return out


def gdn_prep(qkv, alpha, beta_raw, conv_w, hist, dt_bias, a, key_heads, value_heads, head_dim, eps):
    kc = conv_w.shape[1]
    act = torch.empty_like(qkv)
    decay = torch.empty(value_heads, dtype=torch.float32, device=qkv.device)
    beta = torch.empty_like(decay)
    check(_native.lib().cl_gdn_prep(_p(qkv), _p(alpha), _p(beta_raw), _p(conv_w), _p(hist), _p(dt_bias), _p(a),
                                    key_heads, value_heads, head_dim, kc, eps, _p(act), _p(decay), _p(beta),
                                    _stream()), "cl_gdn_prep")
    return act, decay, beta


def gdn_step(act, decay, beta, z, gamma, state, key_heads, value_heads, head_dim, eps):
    out = torch.empty(value_heads * head_dim, dtype=torch.float32, device=act.device)
    check(_native.lib().cl_gdn_step(_p(act), _p(decay), _p(beta), _p(z), _p(gamma), _p(state), key_heads,
                                    value_heads, head_dim, eps, _p(out), _stream()), "cl_gdn_step")
    return out


def attn_gate_prep(mixed, k_raw, v_raw, q_norm, k_norm, hq, hkv, d, rot, cos_sin, pos: int, eps, k_cache, v_cache):
    q = torch.empty(hq * d, dtype=torch.float32, device=mixed.device)
    gate = torch.empty_like(q)
    pos_dev = torch.tensor([pos], dtype=torch.int32, device=mixed.device)
    check(_native.lib().cl_attn_gate_prep(_p(mixed), _p(k_raw), _p(v_raw), _p(q_norm), _p(k_norm), hq, hkv, d, rot,
                                          _p(cos_sin), _p(pos_dev), eps, _p(q), _p(gate), _p(k_cache), _p(v_cache),
                                          _stream()), "cl_attn_gate_prep")
    return q, gate


def mul_sigmoid(a, g):
    out = torch.empty_like(a)
    check(_native.lib().cl_mul_sigmoid(_p(a), _p(g), _p(out), a.numel(), _stream()), "cl_mul_sigmoid")
    return out
