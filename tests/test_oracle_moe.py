"""The qwen35moe FP64 oracle (oracle/moe_fp64.py) on the CPU.

The reference has no CPU path for qwen35moe, so GPU parity for that model is
checked against this restatement; these tests pin the restatement's own
invariants and the rules it restates: the layer-kind rule (moe_model.cpp:164),
the router's top-k tie rule and renormalisation (metal_llm.metal:1424-1474),
DeltaNet decay below one (real GGUFs store ssm_a = -exp(A_log)), and that a
prompt gives the same state whether it is prefilled at once or token by token.
"""
import numpy as np
import pytest

from myllm_b200 import synth_gguf as sg
from oracle.moe_fp64 import MoeFP64


@pytest.fixture(scope="module")
def tiny_moe_path(tmp_path_factory):
    spec = sg.tiny_moe_spec(seed=5)
    return spec, sg.cached_moe(spec, str(tmp_path_factory.mktemp("moe")))


def test_generator_is_deterministic(tmp_path):
    spec = sg.tiny_moe_spec(seed=9, layers=4)
    a = sg.write_moe(spec, str(tmp_path / "a.gguf"))
    b = sg.write_moe(spec, str(tmp_path / "b.gguf"))
    assert a == b


def test_layer_kinds_follow_the_full_attention_interval(tiny_moe_path):
    spec, path = tiny_moe_path
    ref = MoeFP64(path, max_sequence=16)
    assert [ref.is_attention(l) for l in range(spec.layers)] == [(l + 1) % 4 == 0 for l in range(spec.layers)]


def test_deltanet_decay_is_below_one(tiny_moe_path):
    spec, path = tiny_moe_path
    ref = MoeFP64(path, max_sequence=16)
    for l in range(spec.layers):
        if not ref.is_attention(l):
            assert (ref.vec(f"blk.{l}.ssm_a") < 0).all()


def test_prefill_equals_token_by_token(tiny_moe_path):
    spec, path = tiny_moe_path
    prompt = sg.prompt_ids(spec.seed, 9, spec.vocab)
    a = MoeFP64(path, max_sequence=32)
    ta, la = a.prefill(prompt)
    b = MoeFP64(path, max_sequence=32)
    b.prefill(prompt[:-1])
    tb, lb = b.decode(int(prompt[-1]))
    assert ta == tb and np.array_equal(la, lb)
    # reset clears the KV, DeltaNet state and convolution history
    a.reset()
    tc, lc = a.prefill(prompt)
    assert tc == ta and np.array_equal(lc, la)


def test_router_ties_prefer_lower_ids_and_weights_renormalise(tiny_moe_path):
    spec, path = tiny_moe_path
    ref = MoeFP64(path, max_sequence=16)
    E, K, H = spec.experts, spec.experts_used, spec.hidden
    # router rows chosen so that logits = W x are: experts 3, 9, 12 tied at the top, then 0..
    W = np.zeros((E, H))
    W[:, 0] = 0.1 * np.arange(E)[::-1]      # descending in id: lower ids larger
    W[[3, 9, 12], 0] = 5.0
    x = np.zeros(H)
    x[0] = 1.0
    orig = ref.w
    ref.w = lambda name: W if name.endswith("ffn_gate_inp.weight") else orig(name)
    ids, wts = ref.route(0, x)
    assert list(ids) == [3, 9, 12, 0][:K]
    assert abs(wts.sum() - 1.0) < 1e-12
    assert wts[0] == wts[1] == wts[2] > wts[3]
