"""The qwen35moe FP64 restatement (oracle/moe_fp64.py) pinned to the
reference's own kernels.

The reference's qwen35moe path is Metal only.  Its compute kernels
(metal_llm.metal) compile as C++ (oracle/metal_shim.h) and run on the host in
the order and with the parameters the reference's MoE host encodes them
(oracle/metal_ref.py, restating moe_llm.mm); tests/golden/moe_metal_ref.npz
holds their outputs on seeded inputs (tests/golden/make_moe_metal_golden.py,
which also rebuilds the inputs here).  This checks the restatement's formulas
step by step against them, after the projections:

* the DeltaNet mixer (moe_llm.mm:2470-2635): conv + history, SiLU, L2 norms,
  decay / beta, the delta-rule recurrence, the per-head RMSNorm and the z
  gate, at the tiny width and at config 4's state size 128;
* routing (moe_llm.mm:2642-2690): softmax, top-8 of 256 with an exact
  three-way tie, renormalisation;
* routed experts (moe_llm.mm:2692-2843) over native Q4_K / Q6_K rows;
* gated attention (moe_llm.mm:2256-2428) at config 4's head size 256 and
  rotary width 64, three tokens after five cached rows;
* whole token steps of two seeded tiny qwen35moe models (embedding, every
  layer, routed and shared experts, LM head) with every product, norm and
  activation a reference kernel, in the layer order of the reference's
  forward (moe_llm.mm:2845-3039; oracle.metal_ref.MoeReference): a 6-token
  prompt and 4 greedy steps, same tokens, logits within 2e-5;
* the FP64 fixture the GPU test at config 4's layer widths uses
  (moe_a3b_width.npz: 4 layers, 256 experts top-8, hidden 2048) against the
  reference-kernel forward of the same model (stored beside the tiny models'
  runs): the same greedy tokens, logits within 2e-5.

The reference kernels compute in FP32 and the restatement in float64: values
agree within 2e-5 of the largest, expert ids and copied rows exactly.
"""
import importlib.util
import os

import numpy as np
import pytest

import oracle
from myllm_b200 import synth_gguf as sg
from oracle import metal_ref as M
from oracle import moe_fp64 as O

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
_spec = importlib.util.spec_from_file_location("make_moe_metal_golden",
                                               os.path.join(GOLDEN_DIR, "make_moe_metal_golden.py"))
G = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(G)

TOL = 2e-5
F64 = np.float64


def rel(got, ref):
    got, ref = np.asarray(got, F64), np.asarray(ref, F64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


@pytest.fixture(scope="module")
def golden():
    return np.load(os.path.join(GOLDEN_DIR, "moe_metal_ref.npz"))


@pytest.fixture(scope="module")
def model_golden():
    return np.load(os.path.join(GOLDEN_DIR, "moe_metal_ref_model.npz"))


@pytest.fixture(scope="module")
def model_dir(tmp_path_factory):
    return str(tmp_path_factory.mktemp("moe_ref_models"))


CASES = G.cases()


def by_kind(kind):
    return [pytest.param(c, id=c["name"]) for c in CASES if c["kind"] == kind]


@pytest.mark.parametrize("c", by_kind("deltanet"))
def test_deltanet_matches_reference_kernels(c, golden):
    hist, S = c["hist"].astype(F64), c["state"].astype(F64).copy()
    outs = []
    for t in range(c["qkv"].shape[0]):
        g, hist = O.deltanet_token(c["qkv"][t].astype(F64), c["z"][t].astype(F64), c["beta_raw"][t].astype(F64),
                                   c["alpha"][t].astype(F64), c["dt_bias"].astype(F64), c["a"].astype(F64),
                                   c["conv_w"].astype(F64), hist, S, c["norm"].astype(F64), c["key_heads"],
                                   c["head_dim"], c["value_heads"], G.EPS)
        outs.append(g)
    n = c["name"]
    assert rel(np.stack(outs), golden[n + ".gated"]) <= TOL
    assert rel(S, golden[n + ".state"]) <= TOL
    assert np.array_equal(hist.astype(np.float32), golden[n + ".hist"])  # the history is copied rows


@pytest.mark.parametrize("c", by_kind("route"))
def test_routing_matches_reference_kernels(c, golden):
    n = c["name"]
    for t, row in enumerate(c["logits"]):
        ids, w = O.route_probs(row.astype(F64), c["k"])
        np.testing.assert_array_equal(ids, golden[n + ".ids"][t])
        assert rel(w, golden[n + ".weights"][t]) <= TOL
    # token 0 has experts 5, 9, 40 tied at the top: lower ids first in both
    np.testing.assert_array_equal(golden[n + ".ids"][0][:3], [5, 9, 40])


@pytest.mark.parametrize("c", by_kind("experts"))
def test_routed_experts_match_reference_kernels(c, golden):
    H, F = c["x"].shape[1], c["ffn"]
    rows = {"gate": (c["gate_type"], c["gate"], F, H), "up": (c["gate_type"], c["up"], F, H),
            "down": (c["down_type"], c["down"], H, F)}

    def expert_rows(kind, e):
        t, native, r, cols = rows[kind]
        return oracle.dequant(t, native[e * r:(e + 1) * r], r, cols).astype(F64)

    out = np.stack([O.routed_experts(c["x"][t].astype(F64), c["ids"][t], c["weights"][t].astype(F64), expert_rows)
                    for t in range(c["x"].shape[0])])
    assert rel(out, golden[c["name"] + ".out"]) <= TOL


@pytest.mark.parametrize("c", by_kind("attention"))
def test_gated_attention_matches_reference_kernels(c, golden):
    hkv, d, pos = c["kv_heads"], c["head_dim"], c["position"]
    k_hist = [r.astype(F64).reshape(hkv, d) for r in c["k_cache"][:pos]]
    v_hist = [r.astype(F64).reshape(hkv, d) for r in c["v_cache"][:pos]]
    outs = [O.attention_token(c["mixed"][t].astype(F64), c["k"][t].astype(F64), c["v"][t].astype(F64),
                              c["q_norm"].astype(F64), c["k_norm"].astype(F64), pos + t, k_hist, v_hist,
                              c["q_heads"], hkv, d, c["rot"], c["theta"], G.EPS)
            for t in range(c["mixed"].shape[0])]
    n = c["name"]
    assert rel(np.stack(outs), golden[n + ".out"]) <= TOL
    # the appended cache rows: normalised, rotated keys; values as given
    assert rel(np.stack(k_hist[pos:]).reshape(-1, hkv * d), golden[n + ".k_cache"][pos:]) <= TOL
    assert np.array_equal(golden[n + ".v_cache"][pos:], c["v"])


@pytest.mark.parametrize("seed", G.MODEL_SEEDS)
def test_whole_token_steps_match_reference_kernels(seed, model_golden, model_dir):
    """The FP64 forward fed the reference run's tokens: every step's logits
    within 2e-5 of the reference kernels' and the same greedy token."""
    spec, path = G.tiny_model(seed, model_dir)
    fed, ref_logits = model_golden[f"s{seed}.tokens"], model_golden[f"s{seed}.logits"]
    np.testing.assert_array_equal(fed[:G.PROMPT], sg.prompt_ids(spec.seed, G.PROMPT, spec.vocab))
    fp64 = O.MoeFP64(path, max_sequence=32)
    for i, t in enumerate(fed):
        logits = fp64.step(int(t))
        assert rel(logits, ref_logits[i]) <= TOL, i
        assert int(np.argmax(logits)) == int(np.argmax(ref_logits[i])), i


def test_config4_width_fixture_matches_reference_kernels(model_golden):
    """The FP64 forward's fixture at config 4's widths and the reference
    kernels' forward of the same GGUF (same SHA-256) agree."""
    fp64 = np.load(os.path.join(GOLDEN_DIR, "moe_a3b_width.npz"))
    assert str(fp64["sha256"]) == str(model_golden["a3b.sha256"])
    np.testing.assert_array_equal(fp64["tokens"], model_golden["a3b.tokens"])
    for i in range(len(fp64["tokens"])):
        assert rel(fp64["logits"][i], model_golden["a3b.logits"][i]) <= TOL, i


@pytest.mark.skipif(not M.available(), reason="the reference kernels were not built here (oracle/Makefile metal)")
def test_fixture_is_what_the_reference_kernels_compute(golden, model_golden, model_dir):
    """Where the reference sources were built, the reference kernels run now
    reproduce the committed outputs bit for bit."""
    for c in CASES:
        for key, val in G.run_reference(c).items():
            assert np.array_equal(val, golden[f"{c['name']}.{key}"]), (c["name"], key)
    for seed in G.MODEL_SEEDS:
        spec, path = G.tiny_model(seed, model_dir)
        fed, logits = G.run_reference_model(path, sg.prompt_ids(spec.seed, G.PROMPT, spec.vocab),
                                            G.PROMPT + G.DECODES)
        assert np.array_equal(fed, model_golden[f"s{seed}.tokens"]) and np.array_equal(
            logits, model_golden[f"s{seed}.logits"]), seed
