"""ORACLE (test infrastructure only): the reference's own qwen35moe kernels.

The reference runs qwen35moe on Metal only (moe_llm.mm + metal_llm.metal), so
its FP64 restatement (``moe_fp64.py``) cannot be checked against a reference
CPU path.  ``oracle/Makefile`` (target ``metal``, part of ``ref``) compiles
the reference's ``metal_llm.metal`` where it lies, as C++ through
``metal_shim.h``, into ``oracle/_ref/libref_metal.so``; this module calls
those kernels in the order and with the parameters the reference's MoE host
encodes them (moe_llm.mm), so the restatement's formulas can be pinned to the
reference kernels' own arithmetic (run in IEEE FP32 on the host).

Sequences restated here (each function cites its source):

* ``deltanet``: moe_llm.mm:2436-2640 after the projections;
* ``route``: moe_llm.mm:2642-2690 after the router product;
* ``experts``: moe_llm.mm:2692-2843 (routed experts only);
* ``attention``: moe_llm.mm:2238-2434 between the projections;
* ``MoeReference``: one whole token step (embedding, every layer's mixer,
  router, routed and shared experts, residuals, final norm, LM head) with
  every product, norm and activation a reference kernel, in the layer order
  of the reference's forward (moe_llm.mm:2845-3039).
"""
from __future__ import annotations

import ctypes
import os
from typing import Dict, Tuple

import numpy as np

from .gguf_read import GgufReader

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_ref", "libref_metal.so")

_lib = None
_u, _f, _p, _i = ctypes.c_uint, ctypes.c_float, ctypes.c_void_p, ctypes.c_int

_SIGS = {
    "mref_rmsnorm": [_p, _p, _p, _u, _u, _f],
    "mref_softmax": [_p, _p, _u, _u],
    "mref_unary": [_i, _p, _p, _u],
    "mref_binary": [_i, _p, _p, _p, _u],
    "mref_channel": [_i, _p, _p, _p, _u, _u],
    "mref_conv1d": [_p, _p, _p, _p, _u, _u, _u],
    "mref_conv_commit": [_p, _p, _u, _u, _u],
    "mref_l2norm_heads": [_p, _p, _u, _u, _u, _u, _f],
    "mref_gdn": [_p, _p, _p, _p, _p, _p, _p, _u, _u, _u, _u, _u, _u, _u, _u],
    "mref_topk": [_p, _p, _p, _u, _u, _u],
    "mref_topk_renorm": [_p, _u, _u],
    "mref_expert": [_i, _p, _p, _p, _p, _u, _u, _u, _u, _u, _u, _u, _u],
    "mref_weighted_reduce": [_p, _p, _p, _u, _u, _u],
    "mref_split_q_gate": [_p, _p, _p, _u, _u, _u],
    "mref_rope_heads": [_p, _p, _u, _u, _u, _u, _u, _f],
    "mref_kv_write": [_p, _p, _p, _p, _u, _u, _u, _u],
    "mref_qk": [_p, _p, _p, _u, _u, _u, _u, _u, _u, _u, _u, _f],
    "mref_av": [_p, _p, _p, _u, _u, _u, _u, _u, _u, _u, _u],
    "mref_gevm": [_i, _p, _p, _p, _u, _u, _u],
    "mref_embedding": [_i, _p, _p, _p, _u, _u, _u, _u],
    "mref_row_scale": [_p, _p, _p, _u, _u, _u, _u],
    "mref_residual": [_p, _p, _p, _u],
}
_INT_RESULT = {"mref_expert", "mref_gevm", "mref_embedding"}


def available() -> bool:
    return os.path.exists(LIB)


def lib():
    global _lib
    if _lib is None:
        l = ctypes.CDLL(LIB)
        for name, args in _SIGS.items():
            fn = getattr(l, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int if name in _INT_RESULT else None
        _lib = l
    return _lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data)


def _new(*shape) -> np.ndarray:
    return np.zeros(shape, dtype=np.float32)


def _unary(op: int, x: np.ndarray) -> np.ndarray:
    x = _f32(x)
    out = np.empty_like(x)
    lib().mref_unary(op, _ptr(x), _ptr(out), x.size)
    return out


def _binary(op: int, a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a, b = _f32(a), _f32(b)
    out = np.empty_like(a)
    lib().mref_binary(op, _ptr(a), _ptr(b), _ptr(out), a.size)
    return out


def _channel(op: int, x: np.ndarray, ch: np.ndarray) -> np.ndarray:
    x, ch = _f32(x), _f32(ch)
    out = np.empty_like(x)
    lib().mref_channel(op, _ptr(x), _ptr(ch), _ptr(out), x.shape[0], x.shape[1])
    return out


def rmsnorm_rows(x: np.ndarray, gamma: np.ndarray, eps: float) -> np.ndarray:
    x, gamma = _f32(x), _f32(gamma)
    out = np.empty_like(x)
    lib().mref_rmsnorm(_ptr(x), _ptr(gamma), _ptr(out), x.shape[0], x.shape[1], eps)
    return out


def softmax_rows(x: np.ndarray) -> np.ndarray:
    x = _f32(x)
    out = np.empty_like(x)
    lib().mref_softmax(_ptr(x), _ptr(out), x.shape[0], x.shape[1])
    return out


def deltanet(qkv, z, beta_raw, alpha, dt_bias, a, conv_w, hist, state, norm, key_heads: int, head_dim: int,
             value_heads: int, eps: float):
    """One DeltaNet mixer over a chunk of T tokens after its projections
    (moe_llm.mm:2470-2635): beta = sigmoid(beta_raw); decay =
    exp(softplus(alpha + dt_bias) * a); causal conv over [history, qkv] and
    the history commit; SiLU; per-head L2 norm of q and k; the recurrence;
    per-head RMSNorm of its output; times silu(z).  qkv [T, 2 K d + V d],
    z [T, V d], beta_raw / alpha [T, V], conv_w [channels, kernel], hist
    [kernel - 1, channels], state [V, d, d] (row = key dim).  Returns
    (gated [T, V d], new history, new state)."""
    qkv, z = _f32(qkv), _f32(z)
    T, width = qkv.shape
    kw, vw = key_heads * head_dim, value_heads * head_dim
    kc = conv_w.shape[1]
    L = lib()
    beta = _unary(0, beta_raw)
    decay = _unary(3, _channel(1, _unary(2, _channel(0, alpha, dt_bias)), a))
    conv_w, hist, state = _f32(conv_w), _f32(hist).copy(), _f32(state).copy()
    conv = _new(T, width)
    L.mref_conv1d(_ptr(qkv), _ptr(hist), _ptr(conv_w), _ptr(conv), T, width, kc)
    L.mref_conv_commit(_ptr(qkv), _ptr(hist), T, width, kc)
    act = _unary(1, conv)
    qn, kn = _new(T, kw), _new(T, kw)
    L.mref_l2norm_heads(_ptr(act), _ptr(qn), T, key_heads, head_dim, width, eps)
    L.mref_l2norm_heads(_ptr(act[:, kw:]), _ptr(kn), T, key_heads, head_dim, width, eps)
    v = np.ascontiguousarray(act[:, 2 * kw:])
    out = _new(T, vw)
    L.mref_gdn(_ptr(qn), _ptr(kn), _ptr(v), _ptr(decay), _ptr(beta), _ptr(state), _ptr(out), T, key_heads,
               value_heads, head_dim, kw, kw, vw, vw)
    normed = rmsnorm_rows(out.reshape(T * value_heads, head_dim), norm, eps).reshape(T, vw)
    return _binary(0, normed, _unary(1, z)), hist, state


def route(logits: np.ndarray, k: int) -> Tuple[np.ndarray, np.ndarray]:
    """Router softmax, top-k (strict '>', lower id first on ties) and the
    renormalisation per token (moe_llm.mm:2642-2690).  logits [T, E] ->
    (ids [T, k], weights [T, k])."""
    probs = softmax_rows(np.atleast_2d(logits))
    T, E = probs.shape
    ids = np.zeros((T, k), dtype=np.uint32)
    wts = _new(T, k)
    L = lib()
    L.mref_topk(_ptr(probs), _ptr(ids), _ptr(wts), T, E, k)
    L.mref_topk_renorm(_ptr(wts), T, k)
    return ids, wts


def _expert_product(gtype: int, act: np.ndarray, w: np.ndarray, ids: np.ndarray, tokens: int, routes: int,
                    rows: int, cols: int, routed: bool) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8)
    row_bytes = w.shape[1]
    out = _new(tokens * routes, rows)
    act = _f32(act)
    if lib().mref_expert(gtype, _ptr(act), _ptr(w), _ptr(ids), _ptr(out), tokens, routes, rows, cols, act.shape[1],
                         row_bytes, rows * row_bytes, 1 if routed else 0) != 0:
        raise ValueError("the reference's expert product takes Q4_K and Q6_K only")
    return out


def experts(x: np.ndarray, ids: np.ndarray, weights: np.ndarray, gate_type: int, gate: np.ndarray, up: np.ndarray,
            down_type: int, down: np.ndarray, ffn: int) -> np.ndarray:
    """Routed experts of T tokens (moe_llm.mm:2692-2843): gate and up
    products of each route's expert, SwiGLU, the down product of the routed
    rows, then the weighted reduce over each token's routes.  x [T, H],
    ids / weights [T, k], gate / up [E * ffn, row bytes] and down
    [E * H, row bytes] native GGML rows -> [T, H]."""
    x = _f32(np.atleast_2d(x))
    T, H = x.shape
    k = ids.shape[1]
    ids = np.ascontiguousarray(ids, dtype=np.uint32)
    g = _expert_product(gate_type, x, gate, ids, T, k, ffn, H, False)
    u = _expert_product(gate_type, x, up, ids, T, k, ffn, H, False)
    act = _binary(1, g, u)
    d = _expert_product(down_type, act, down, ids, T, k, H, ffn, True)
    out = _new(T, H)
    w = _f32(weights)
    lib().mref_weighted_reduce(_ptr(d), _ptr(w), _ptr(out), T, k, H)
    return out


def attention(mixed, k, v, q_norm, k_norm, k_cache, v_cache, position: int, q_heads: int, kv_heads: int,
              head_dim: int, rot: int, theta: float, eps: float):
    """Gated attention of T tokens at `position` between the projections
    (moe_llm.mm:2256-2428): split the packed [query, gate] heads, RMSNorm q
    and k per head, NeoX RoPE on the first `rot` dims of each head, append
    k / v to the caches at `position`, causal scores times 1 / sqrt(d),
    softmax, the value mix, times sigmoid(gate).  mixed [T, 2 hq d],
    k / v [T, hkv d], caches [capacity, hkv d] (updated copies returned).
    Returns (gated [T, hq d], k_cache, v_cache)."""
    mixed, k, v = _f32(mixed), _f32(k), _f32(v)
    T = mixed.shape[0]
    qw, kvw = q_heads * head_dim, kv_heads * head_dim
    L = lib()
    q, gate = _new(T, qw), _new(T, qw)
    L.mref_split_q_gate(_ptr(mixed), _ptr(q), _ptr(gate), T, q_heads, head_dim)
    qn = rmsnorm_rows(q.reshape(T * q_heads, head_dim), q_norm, eps).reshape(T, qw)
    kn = rmsnorm_rows(k.reshape(T * kv_heads, head_dim), k_norm, eps).reshape(T, kvw)
    qr, kr = _new(T, qw), _new(T, kvw)
    L.mref_rope_heads(_ptr(qn), _ptr(qr), T, qw, head_dim, rot, position, theta)
    L.mref_rope_heads(_ptr(kn), _ptr(kr), T, kvw, head_dim, rot, position, theta)
    kc, vc = _f32(k_cache).copy(), _f32(v_cache).copy()
    L.mref_kv_write(_ptr(kr), _ptr(v), _ptr(kc), _ptr(vc), T, kvw, kvw, position)
    klen = position + T
    scores = _new(T * q_heads, klen)
    scale = np.float32(1.0) / np.sqrt(np.float32(head_dim))
    L.mref_qk(_ptr(qr), _ptr(kc), _ptr(scores), T, klen, q_heads, kv_heads, kvw, qw, head_dim, position,
              float(scale))
    probs = softmax_rows(scores)
    out = _new(T, qw)
    L.mref_av(_ptr(probs), _ptr(vc), _ptr(out), T, klen, q_heads, kv_heads, kvw, klen, head_dim, qw)
    return _binary(0, out, _unary(0, gate)), kc, vc


def _residual(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a, b = _f32(a), _f32(b)
    out = np.empty_like(a)
    lib().mref_residual(_ptr(a), _ptr(b), _ptr(out), a.size)
    return out


class MoeReference:
    """A qwen35moe GGUF run token by token through the reference's kernels.

    The layer order restates the reference's forward (moe_llm.mm:2845-3039):
    h = embed(token); per layer h += mixer(rmsnorm(h)) with the mixer the
    gated attention or the DeltaNet of its layer kind (moe_model.cpp:164-166),
    then h += routed experts + sigmoid(shared router) * shared expert of
    rmsnorm(h); logits = LM head(rmsnorm(h)).  Every product is the
    reference's one-row product kernel for the tensor's type (rows == 1, as
    in the reference's decode), every other step the kernel the reference
    encodes for it.  State (DeltaNet state and history, KV caches) is FP32
    as in the reference."""

    def __init__(self, path: str, max_sequence: int = 64):
        r = GgufReader(path)
        m = r.metadata
        a = "qwen35moe."
        self.H = int(m[a + "embedding_length"])
        self.L = int(m[a + "block_count"]) - int(m.get(a + "nextn_predict_layers", 0))
        self.E = int(m[a + "expert_count"])
        self.K = int(m[a + "expert_used_count"])
        self.hq = int(m[a + "attention.head_count"])
        self.hkv = int(m[a + "attention.head_count_kv"])
        self.hd = int(m[a + "attention.key_length"])
        self.rot = int(m[a + "rope.dimension_count"])
        self.theta = float(m[a + "rope.freq_base"])
        self.eps = float(m[a + "attention.layer_norm_rms_epsilon"])
        self.interval = int(m[a + "full_attention_interval"])
        self.ck = int(m[a + "ssm.conv_kernel"])
        self.sd = int(m[a + "ssm.state_size"])
        self.sg = int(m[a + "ssm.group_count"])
        self.sr = int(m[a + "ssm.time_step_rank"])
        self.si = int(m[a + "ssm.inner_size"])
        self.V = int(m["tokenizer.ggml.tokens_count"])
        self.max_sequence = max_sequence
        self._r = r
        self._t: Dict[str, tuple] = {}
        self.reset()

    def is_attention(self, l: int) -> bool:
        return (l + 1) % self.interval == 0

    def reset(self):
        self.pos = 0
        qkvw = 2 * self.sg * self.sd + self.si
        kvw = self.hkv * self.hd
        self.S = {l: _new(self.sr, self.sd, self.sd) for l in range(self.L) if not self.is_attention(l)}
        self.hist = {l: _new(self.ck - 1, qkvw) for l in range(self.L) if not self.is_attention(l)}
        self.kc = {l: _new(self.max_sequence, kvw) for l in range(self.L) if self.is_attention(l)}
        self.vc = {l: _new(self.max_sequence, kvw) for l in range(self.L) if self.is_attention(l)}

    def t(self, name: str):
        """(type, rows, cols, native rows [rows, row bytes]) of a tensor."""
        if name not in self._t:
            self._t[name] = self._r.rows(name)
        return self._t[name]

    def f32(self, name: str) -> np.ndarray:
        gtype, rows, cols, data = self.t(name)
        assert gtype == 0, name
        return np.ascontiguousarray(data).view(np.float32).reshape(rows, cols)

    def vec(self, name: str) -> np.ndarray:
        return self.f32(name).reshape(-1)

    def product(self, name: str, x: np.ndarray) -> np.ndarray:
        gtype, rows, cols, data = self.t(name)
        x = _f32(x).reshape(-1)
        assert x.size == cols, name
        out = _new(rows)
        w = np.ascontiguousarray(data)
        if lib().mref_gevm(gtype, _ptr(w), _ptr(x), _ptr(out), rows, cols, w.shape[1]) != 0:
            raise ValueError(f"no reference product kernel for type {gtype} ({name})")
        return out

    def _rms(self, x, name):
        return rmsnorm_rows(x[None, :], self.vec(name), self.eps)[0]

    def _attention(self, l, xn):
        p = f"blk.{l}."
        gated, self.kc[l], self.vc[l] = attention(
            self.product(p + "attn_q.weight", xn)[None, :], self.product(p + "attn_k.weight", xn)[None, :],
            self.product(p + "attn_v.weight", xn)[None, :], self.vec(p + "attn_q_norm.weight"),
            self.vec(p + "attn_k_norm.weight"), self.kc[l], self.vc[l], self.pos, self.hq, self.hkv, self.hd,
            self.rot, self.theta, self.eps)
        return self.product(p + "attn_output.weight", gated[0])

    def _deltanet(self, l, xn):
        p = f"blk.{l}."
        gated, self.hist[l], self.S[l] = deltanet(
            self.product(p + "attn_qkv.weight", xn)[None, :], self.product(p + "attn_gate.weight", xn)[None, :],
            self.product(p + "ssm_beta.weight", xn)[None, :], self.product(p + "ssm_alpha.weight", xn)[None, :],
            self.vec(p + "ssm_dt.bias"), self.vec(p + "ssm_a"), self.f32(p + "ssm_conv1d.weight"), self.hist[l],
            self.S[l], self.vec(p + "ssm_norm.weight"), self.sg, self.sd, self.sr, self.eps)
        return self.product(p + "ssm_out.weight", gated[0])

    def _moe(self, l, xn):
        p = f"blk.{l}."
        ids, wts = route(self.product(p + "ffn_gate_inp.weight", xn)[None, :], self.K)
        gt, _, _, gate = self.t(p + "ffn_gate_exps.weight")
        _, _, _, up = self.t(p + "ffn_up_exps.weight")
        dt, _, ffn, down = self.t(p + "ffn_down_exps.weight")
        routed = experts(xn[None, :], ids, wts, gt, gate, up, dt, down, ffn)[0]
        sgate = _unary(0, self.product(p + "ffn_gate_inp_shexp.weight", xn))
        act = _binary(1, self.product(p + "ffn_gate_shexp.weight", xn), self.product(p + "ffn_up_shexp.weight", xn))
        down_sh = self.product(p + "ffn_down_shexp.weight", act)
        scaled = np.empty_like(down_sh)
        lib().mref_row_scale(_ptr(down_sh), _ptr(sgate), _ptr(scaled), 1, down_sh.size, 1, 0)
        return _residual(routed, scaled)

    def step(self, token: int) -> np.ndarray:
        """Advance one token; returns the logits."""
        if self.pos >= self.max_sequence:
            raise IndexError("capacity")
        gtype, rows, cols, data = self.t("token_embd.weight")
        w = np.ascontiguousarray(data)
        ids = np.array([token], dtype=np.int32)
        x = _new(cols)
        if lib().mref_embedding(gtype, _ptr(ids), _ptr(w), _ptr(x), 1, cols, rows, w.shape[1]) != 0:
            raise ValueError(f"no reference embedding kernel for type {gtype}")
        for l in range(self.L):
            p = f"blk.{l}."
            xn = self._rms(x, p + "attn_norm.weight")
            mix = self._attention(l, xn) if self.is_attention(l) else self._deltanet(l, xn)
            x = _residual(x, mix)
            x = _residual(x, self._moe(l, self._rms(x, p + "post_attention_norm.weight")))
        self.pos += 1
        return self.product("output.weight", self._rms(x, "output_norm.weight"))
