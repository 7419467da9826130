"""Golden outputs of the reference's own qwen35moe kernels.

Runs the reference's Metal compute kernels (metal_llm.metal, compiled as C++
into oracle/_ref/libref_metal.so by oracle/Makefile's `metal` target, see
oracle/metal_ref.py) in the reference's dispatch order on seeded inputs and
stores their outputs in tests/golden/moe_metal_ref.npz.  The inputs are not
stored: `cases()` rebuilds them from seeds with this project's deterministic
synthetic generator (myllm_b200.synth_gguf), here and in
tests/test_oracle_moe_pinned.py.

It also runs whole token steps of two seeded tiny qwen35moe models through
the reference kernels (oracle.metal_ref.MoeReference: a 6-token prompt, then
4 greedy steps) and stores the tokens fed and the logits of every step in
tests/golden/moe_metal_ref_model.npz; and the same for the 4-layer model with
every config-4 width (synth_gguf.a3b_width_spec, a 2 GB GGUF written to a
temporary directory) over the prompt of tests/golden/moe_a3b_width.npz, then
4 greedy steps, storing the model's SHA-256, the greedy tokens and the
logits of the last prompt step and the 4 decodes (the FP64 fixture's layout).

    python tests/golden/make_moe_metal_golden.py      # needs the built library
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from myllm_b200 import synth_gguf as sg  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "moe_metal_ref.npz")
OUT_MODEL = os.path.join(os.path.dirname(os.path.abspath(__file__)), "moe_metal_ref_model.npz")
MODEL_SEEDS = (5, 11)
PROMPT, DECODES = 6, 4
EPS = 1e-6


def _v(n, seed, name, std=1.0):
    return sg.normal(int(n), sg.stream_key(seed, name), 0.0, std).astype(np.float32)


def deltanet_case(name, key_heads, head_dim, value_heads, tokens, seed):
    """One DeltaNet mixer over `tokens` tokens after its projections, from a
    non-zero state and history (as after earlier tokens)."""
    kw, vw = key_heads * head_dim, value_heads * head_dim
    width, kc = 2 * kw + vw, 4
    return {
        "kind": "deltanet", "name": name, "key_heads": key_heads, "head_dim": head_dim,
        "value_heads": value_heads,
        "qkv": _v(tokens * width, seed, name + "qkv").reshape(tokens, width),
        "z": _v(tokens * vw, seed, name + "z").reshape(tokens, vw),
        "beta_raw": _v(tokens * value_heads, seed, name + "b").reshape(tokens, value_heads),
        "alpha": _v(tokens * value_heads, seed, name + "a").reshape(tokens, value_heads),
        "dt_bias": _v(value_heads, seed, name + "dt", 0.5),
        # real checkpoints store ssm_a = -exp(A_log): negative
        "a": -np.exp(_v(value_heads, seed, name + "A", 0.5)),
        "conv_w": _v(width * kc, seed, name + "cw", 0.5).reshape(width, kc),
        "hist": _v((kc - 1) * width, seed, name + "h").reshape(kc - 1, width),
        "state": _v(value_heads * head_dim * head_dim, seed, name + "S", 0.1).reshape(value_heads, head_dim,
                                                                                      head_dim),
        "norm": 1.0 + _v(head_dim, seed, name + "n", 0.05),
    }


def route_case(name, experts, k, tokens, seed):
    logits = _v(tokens * experts, seed, name + "l", 2.0).reshape(tokens, experts)
    logits[0, [5, 9, 40]] = logits[0].max() + 1.0  # an exact three-way tie at the top of token 0
    return {"kind": "route", "name": name, "k": k, "logits": logits}


def experts_case(name, n_experts, hidden, ffn, k, tokens, gate_type, down_type, seed):
    rng = np.random.default_rng(seed)
    ids = np.stack([rng.permutation(n_experts)[:k] for _ in range(tokens)]).astype(np.uint32)
    w = rng.random((tokens, k)).astype(np.float32)
    return {
        "kind": "experts", "name": name, "ffn": ffn, "gate_type": gate_type, "down_type": down_type,
        "x": _v(tokens * hidden, seed, name + "x").reshape(tokens, hidden),
        "ids": ids, "weights": (w / w.sum(axis=1, keepdims=True)).astype(np.float32),
        "gate": sg.fill(gate_type, n_experts * ffn, hidden, sg.stream_key(seed, name + "g"), 0.0, 0.02),
        "up": sg.fill(gate_type, n_experts * ffn, hidden, sg.stream_key(seed, name + "u"), 0.0, 0.02),
        "down": sg.fill(down_type, n_experts * hidden, ffn, sg.stream_key(seed, name + "d"), 0.0, 0.02),
    }


def attention_case(name, q_heads, kv_heads, head_dim, rot, position, tokens, seed):
    """`tokens` tokens at `position` after `position` earlier cache rows."""
    qw, kvw = q_heads * head_dim, kv_heads * head_dim
    cap = position + tokens
    kc = np.zeros((cap, kvw), np.float32)
    vc = np.zeros((cap, kvw), np.float32)
    kc[:position] = _v(position * kvw, seed, name + "kc").reshape(position, kvw)
    vc[:position] = _v(position * kvw, seed, name + "vc").reshape(position, kvw)
    return {
        "kind": "attention", "name": name, "q_heads": q_heads, "kv_heads": kv_heads, "head_dim": head_dim,
        "rot": rot, "position": position, "theta": 1.0e7,
        "mixed": _v(tokens * 2 * qw, seed, name + "m").reshape(tokens, 2 * qw),
        "k": _v(tokens * kvw, seed, name + "k").reshape(tokens, kvw),
        "v": _v(tokens * kvw, seed, name + "v").reshape(tokens, kvw),
        "q_norm": 1.0 + _v(head_dim, seed, name + "qn", 0.05),
        "k_norm": 1.0 + _v(head_dim, seed, name + "kn", 0.05),
        "k_cache": kc, "v_cache": vc,
    }


def cases():
    return [
        deltanet_case("gdn_tiny", 2, 32, 4, 4, 1),
        deltanet_case("gdn_d128", 2, 128, 4, 3, 2),   # config 4's state size; value head h reads key head h % 2
        route_case("route_a3b", 256, 8, 4, 3),        # config 4's router: 256 experts, top 8
        experts_case("experts_q4q6", 4, 256, 256, 2, 3, sg.Q4_K, sg.Q6_K, 4),
        experts_case("experts_q4q4", 4, 512, 256, 3, 2, sg.Q4_K, sg.Q4_K, 5),
        attention_case("attn_a3b", 4, 2, 256, 64, 5, 3, 6),  # config 4's head size and rotary width
    ]


def run_reference(c):
    """The reference kernels' outputs for case c (a dict of arrays)."""
    from oracle import metal_ref as M
    if c["kind"] == "deltanet":
        g, h, s = M.deltanet(c["qkv"], c["z"], c["beta_raw"], c["alpha"], c["dt_bias"], c["a"], c["conv_w"],
                             c["hist"], c["state"], c["norm"], c["key_heads"], c["head_dim"], c["value_heads"], EPS)
        return {"gated": g, "hist": h, "state": s}
    if c["kind"] == "route":
        ids, w = M.route(c["logits"], c["k"])
        return {"ids": ids, "weights": w}
    if c["kind"] == "experts":
        return {"out": M.experts(c["x"], c["ids"], c["weights"], c["gate_type"], c["gate"], c["up"],
                                 c["down_type"], c["down"], c["ffn"])}
    out, kc, vc = M.attention(c["mixed"], c["k"], c["v"], c["q_norm"], c["k_norm"], c["k_cache"], c["v_cache"],
                              c["position"], c["q_heads"], c["kv_heads"], c["head_dim"], c["rot"], c["theta"], EPS)
    return {"out": out, "k_cache": kc, "v_cache": vc}


def tiny_model(seed, directory):
    """(spec, path) of the seeded tiny qwen35moe model (the one the other
    qwen35moe tests use), written under `directory` if it is not there."""
    spec = sg.tiny_moe_spec(seed=seed)
    return spec, sg.cached_moe(spec, directory)


def run_reference_model(path, prompt, steps, max_sequence=32):
    """Tokens fed and logits [steps, vocab] of the reference-kernel model:
    the prompt, then greedy steps on its own argmax (lowest index on ties)."""
    from oracle import metal_ref as M
    ref = M.MoeReference(path, max_sequence)
    fed, logits = [], []
    for i in range(steps):
        t = int(prompt[i]) if i < len(prompt) else int(np.argmax(logits[-1]))
        fed.append(t)
        logits.append(ref.step(t))
    return np.array(fed, dtype=np.int32), np.stack(logits)


def main():
    import tempfile
    from oracle import metal_ref as M
    if not M.available():
        raise SystemExit("build oracle/_ref/libref_metal.so first (make -C oracle metal REF=<reference checkout>)")
    arrays = {}
    for c in cases():
        for key, val in run_reference(c).items():
            arrays[f"{c['name']}.{key}"] = val
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT}: {len(arrays)} arrays")
    model = {}
    with tempfile.TemporaryDirectory() as d:
        for seed in MODEL_SEEDS:
            spec, path = tiny_model(seed, d)
            fed, logits = run_reference_model(path, sg.prompt_ids(spec.seed, PROMPT, spec.vocab), PROMPT + DECODES)
            model[f"s{seed}.tokens"] = fed
            model[f"s{seed}.logits"] = logits
    fp64 = np.load(os.path.join(os.path.dirname(OUT), "moe_a3b_width.npz"))
    with tempfile.TemporaryDirectory(dir=os.environ.get("MYLLM_GOLDEN_TMP")) as d:
        path = os.path.join(d, "a3b_width.gguf")
        sha = sg.write_moe(sg.a3b_width_spec(), path)
        prompt = fp64["prompt"]
        fed, logits = run_reference_model(path, prompt, len(prompt) + 4, max_sequence=64)
    tail = logits[len(prompt) - 1:]
    model["a3b.sha256"] = np.array(sha)
    model["a3b.tokens"] = np.argmax(tail, axis=1).astype(np.int64)
    model["a3b.logits"] = tail
    np.savez_compressed(OUT_MODEL, **model)
    print(f"wrote {OUT_MODEL}: {len(model)} arrays")


if __name__ == "__main__":
    main()
