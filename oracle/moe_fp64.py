"""ORACLE (test infrastructure only): FP64 restatement of the qwen35moe path.

The reference has no CPU implementation of qwen35moe (Metal only), so parity
for the MoE model rests on this host re-implementation of its formulas, run
in float64 over the reference-exact FP32 weight values (``oracle.dequant``).
The reference ships no test or golden vector for this path; instead the
per-step functions below (``deltanet_token``, ``route_probs``,
``routed_experts``, ``attention_token``) are checked against the reference's
own Metal kernels compiled as C++ and run on the host in the reference's
dispatch order (``oracle/metal_ref.py``, tests/test_oracle_moe_pinned.py).
Whole token steps are also checked against ``metal_ref.MoeReference``,
which chains the reference kernels in the layer order of the reference's
forward (moe_llm.mm:2845-3039, restated: that host code is Objective-C++ on
Metal).

Followed step by step (reference files):

* layer kind: full attention iff (layer + 1) % full_attention_interval == 0
  (moe_model.cpp:164-166); layer loop h += mixer(rmsnorm(h)); h += moe(rmsnorm(h))
  (moe_llm.mm:2845-2885).
* gated attention (moe_llm.mm:2238-2434): the q projection packs each head
  as [query(d), gate(d)] (metal_llm.metal:1164-1183); per-head RMSNorm of q
  and k (metal_llm.metal:785-823); NeoX RoPE on the first rot dims of each
  head (metal_llm.metal:928-967); GQA head h reads KV head h / (hq / hkv)
  (metal_llm.metal:995-1017); softmax over positions <= current; output
  times sigmoid(gate), then the output projection.
* Gated DeltaNet (moe_llm.mm:2436-2640; metal_llm.metal:1186-1420): qkv, z,
  beta = sigmoid(W_b x), decay = exp(softplus(W_a x + dt_bias) * a) with the
  +-20 softplus thresholds; causal depthwise conv over [history, qkv], then
  SiLU; q, k L2-normalised per key head with rsqrt(sum x^2 + eps); value
  head h uses key head h % key_heads; S <- decay S; pred = S^T k;
  S += k (beta (v - pred))^T; o = S^T q / sqrt(d); per-head RMSNorm of o,
  times silu(z), output projection.
* routing (moe_llm.mm:2642-2690; metal_llm.metal:1424-1474): softmax over the
  router logits, top-k by strict '>' (lower expert id first on ties), the
  selected probabilities renormalised to sum 1.
* experts (moe_llm.mm:2692-2843): sum_r w_r down_e(silu(gate_e x) up_e x)
  plus sigmoid(w_sh . x) down_sh(silu(gate_sh x) up_sh x).
* output: final RMSNorm, LM head, argmax with the lowest index on ties.
"""
from __future__ import annotations

from typing import Dict, Tuple

import numpy as np

from . import dequant
from .gguf_read import GgufReader


def _rmsnorm(x, g, eps):
    return x / np.sqrt(np.mean(x * x) + eps) * g


def _sigmoid(v):
    return np.where(v >= 0, 1.0 / (1.0 + np.exp(-np.abs(v))), np.exp(-np.abs(v)) / (1.0 + np.exp(-np.abs(v))))


def _silu(v):
    return v * _sigmoid(v)


def _softplus(v):
    return np.where(v > 20.0, v, np.where(v < -20.0, np.exp(np.minimum(v, 0.0)), np.log1p(np.exp(np.minimum(v, 20.0)))))


# ---- one mixer / router / expert step after its projections (float64) ----
# The class below calls these; tests/test_oracle_moe_pinned.py checks them
# against the reference's own kernels run in the reference's order
# (oracle/metal_ref.py).

def rope_neox(v, pos, rot, theta):
    """NeoX RoPE of one head's first `rot` dims at position `pos`
    (metal_llm.metal:928-967: pair i with i + rot/2, angle pos * theta^(-2i/rot))."""
    half = rot // 2
    p = np.arange(half, dtype=np.float64)
    ang = pos * theta ** (-2.0 * p / rot)
    c, s = np.cos(ang), np.sin(ang)
    a, b = v[:half].copy(), v[half:rot].copy()
    out = v.copy()
    out[:half] = a * c - b * s
    out[half:rot] = a * s + b * c
    return out


def attention_token(mixed, k, v, q_norm, k_norm, pos, k_hist, v_hist, hq, hkv, hd, rot, theta, eps):
    """Gated attention of one token between its projections
    (moe_llm.mm:2256-2428): split [query, gate] per head, RMSNorm and RoPE of
    q and k per head, append k / v to the history lists, softmax over the
    keys so far, the value mix, times sigmoid(gate)."""
    mixed = mixed.reshape(hq, 2, hd)
    q, gate = mixed[:, 0, :], mixed[:, 1, :].reshape(-1)
    k = k.reshape(hkv, hd)
    v = v.reshape(hkv, hd)
    q = np.stack([rope_neox(_rmsnorm(q[h], q_norm, eps), pos, rot, theta) for h in range(hq)])
    k = np.stack([rope_neox(_rmsnorm(k[h], k_norm, eps), pos, rot, theta) for h in range(hkv)])
    k_hist.append(k)
    v_hist.append(v)
    K = np.stack(k_hist)  # [T, hkv, hd]
    Vv = np.stack(v_hist)
    grp = hq // hkv
    out = np.empty((hq, hd))
    for h in range(hq):
        g = h // grp
        s = K[:, g, :] @ q[h] / np.sqrt(hd)
        e = np.exp(s - s.max())
        out[h] = (e / e.sum()) @ Vv[:, g, :]
    return out.reshape(-1) * _sigmoid(gate)


def deltanet_token(qkv, z, beta_raw, alpha, dt_bias, a, conv_w, hist, S, norm, sg, sd, sr, eps):
    """One token of the Gated DeltaNet mixer after its projections
    (moe_llm.mm:2470-2635).  conv_w [channels, kernel], hist [kernel - 1,
    channels], S [value heads, d, d] (row = key dim) updated in place.
    Returns (gated output [value heads * d], the new history)."""
    kw = sg * sd
    beta = _sigmoid(beta_raw)
    decay = np.exp(_softplus(alpha + dt_bias) * a)
    cat = np.concatenate([hist, qkv[None, :]], axis=0)  # [kernel, channels]
    conv = np.einsum("tc,ct->c", cat, conv_w)
    act = _silu(conv)
    q = act[:kw].reshape(sg, sd)
    k = act[kw:2 * kw].reshape(sg, sd)
    v = act[2 * kw:].reshape(sr, sd)
    q = q / np.sqrt((q * q).sum(axis=1, keepdims=True) + eps)
    k = k / np.sqrt((k * k).sum(axis=1, keepdims=True) + eps)
    o = np.empty((sr, sd))
    for h in range(sr):
        kh = h % sg
        S[h] *= decay[h]
        pred = S[h].T @ k[kh]
        delta = beta[h] * (v[h] - pred)
        S[h] += np.outer(k[kh], delta)
        o[h] = _rmsnorm(S[h].T @ q[kh] / np.sqrt(sd), norm, eps)
    return o.reshape(-1) * _silu(z), cat[1:].copy()


def route_probs(logits, k):
    """Softmax of the router logits, the top k by strict '>' with the lower
    expert id first on ties, renormalised (moe_llm.mm:2642-2690)."""
    e = np.exp(logits - logits.max())
    prob = e / e.sum()
    order = sorted(range(len(prob)), key=lambda i: (-prob[i], i))[:k]
    sel = prob[order]
    return np.array(order), sel / sel.sum()


def routed_experts(x, ids, wts, expert_rows):
    """sum_r w_r down_e(silu(gate_e x) * up_e x) (moe_llm.mm:2692-2843);
    expert_rows(kind, e) gives expert e's float64 rows, kind in gate / up / down."""
    acc = np.zeros(len(x))
    for e, wt in zip(ids, wts):
        g = expert_rows("gate", e) @ x
        u = expert_rows("up", e) @ x
        acc += wt * (expert_rows("down", e) @ (_silu(g) * u))
    return acc


class MoeFP64:
    """Token-serial FP64 forward of a qwen35moe GGUF with its own state."""

    def __init__(self, path: str, max_sequence: int = 1024):
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
        self._cache: Dict[str, np.ndarray] = {}
        self.reset()

    # weights (reference-exact FP32 values, promoted to float64 on use)
    def w(self, name: str) -> np.ndarray:
        if name not in self._cache:
            gtype, rows, cols, data = self._r.rows(name)
            if gtype == 0:
                v = data.view(np.float32).reshape(rows, cols).copy()
            else:
                v = dequant(gtype, data, rows, cols)
            self._cache[name] = v.astype(np.float64)
        return self._cache[name]

    def vec(self, name: str) -> np.ndarray:
        return self.w(name).reshape(-1)

    def expert(self, name: str, e: int) -> np.ndarray:
        """Expert e's rows of a stacked [experts * rows, cols] tensor, in
        float64.  Dequantized on use and not cached: a token touches K of the
        E experts, and a whole stack in float64 is gigabytes at full width.
        GGML blocks lie within a row, so these rows equal the same rows of
        the whole tensor's dequantization."""
        gtype, rows, cols, data = self._r.rows(name)
        per = rows // self.E
        part = data[e * per:(e + 1) * per]
        if gtype == 0:
            return part.view(np.float32).reshape(per, cols).astype(np.float64)
        return dequant(gtype, part, per, cols).astype(np.float64)

    def is_attention(self, l: int) -> bool:
        return (l + 1) % self.interval == 0

    def reset(self):
        self.pos = 0
        kw = self.sg * self.sd
        qkvw = 2 * kw + self.si
        self.S = {l: np.zeros((self.sr, self.sd, self.sd)) for l in range(self.L) if not self.is_attention(l)}
        self.hist = {l: np.zeros((self.ck - 1, qkvw)) for l in range(self.L) if not self.is_attention(l)}
        self.kc = {l: [] for l in range(self.L) if self.is_attention(l)}
        self.vc = {l: [] for l in range(self.L) if self.is_attention(l)}

    # ---- blocks ----
    def _rope(self, v, pos):
        return rope_neox(v, pos, self.rot, self.theta)

    def _attention(self, l, x):
        p = f"blk.{l}."
        gated = attention_token(self.w(p + "attn_q.weight") @ x, self.w(p + "attn_k.weight") @ x,
                                self.w(p + "attn_v.weight") @ x, self.vec(p + "attn_q_norm.weight"),
                                self.vec(p + "attn_k_norm.weight"), self.pos, self.kc[l], self.vc[l], self.hq,
                                self.hkv, self.hd, self.rot, self.theta, self.eps)
        return self.w(p + "attn_output.weight") @ gated

    def _deltanet(self, l, x):
        p = f"blk.{l}."
        gated, self.hist[l] = deltanet_token(
            self.w(p + "attn_qkv.weight") @ x, self.w(p + "attn_gate.weight") @ x,
            self.w(p + "ssm_beta.weight") @ x, self.w(p + "ssm_alpha.weight") @ x, self.vec(p + "ssm_dt.bias"),
            self.vec(p + "ssm_a"), self.w(p + "ssm_conv1d.weight"), self.hist[l], self.S[l],
            self.vec(p + "ssm_norm.weight"), self.sg, self.sd, self.sr, self.eps)
        return self.w(p + "ssm_out.weight") @ gated

    def route(self, l, x) -> Tuple[np.ndarray, np.ndarray]:
        """(expert ids, renormalised weights) for the normalised input x."""
        return route_probs(self.w(f"blk.{l}.ffn_gate_inp.weight") @ x, self.K)

    def _moe(self, l, x):
        p = f"blk.{l}."
        ids, wts = self.route(l, x)
        acc = routed_experts(x, ids, wts, lambda kind, e: self.expert(p + f"ffn_{kind}_exps.weight", e))
        sgate = _sigmoid(self.vec(p + "ffn_gate_inp_shexp.weight") @ x)
        sa = _silu(self.w(p + "ffn_gate_shexp.weight") @ x) * (self.w(p + "ffn_up_shexp.weight") @ x)
        return acc + (self.w(p + "ffn_down_shexp.weight") @ sa) * sgate

    def step(self, token: int) -> np.ndarray:
        """Advance one token; returns the logits."""
        if self.pos >= self.max_sequence:
            raise IndexError("capacity")
        x = self.w("token_embd.weight")[token].copy()
        for l in range(self.L):
            p = f"blk.{l}."
            xn = _rmsnorm(x, self.vec(p + "attn_norm.weight"), self.eps)
            x = x + (self._attention(l, xn) if self.is_attention(l) else self._deltanet(l, xn))
            xn = _rmsnorm(x, self.vec(p + "post_attention_norm.weight"), self.eps)
            x = x + self._moe(l, xn)
        self.pos += 1
        xn = _rmsnorm(x, self.vec("output_norm.weight"), self.eps)
        return self.w("output.weight") @ xn

    def prefill(self, ids) -> Tuple[int, np.ndarray]:
        logits = None
        for t in ids:
            logits = self.step(int(t))
        return int(np.argmax(logits)), logits

    def decode(self, token: int) -> Tuple[int, np.ndarray]:
        logits = self.step(int(token))
        return int(np.argmax(logits)), logits

    def margin(self, logits: np.ndarray) -> float:
        s = np.sort(logits)
        return float(s[-1] - s[-2])
