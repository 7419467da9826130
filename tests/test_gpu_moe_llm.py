"""qwen35moe end to end: CudaMoeLLM (through the same C-ABI / Python binding
as CudaLLM) against the FP64 oracle (oracle/moe_fp64.py) on seeded tiny
models.  The reference has no CPU qwen35moe path; the oracle restates its
formulas (moe_llm.mm, metal_llm.metal) in float64.

Tokens must be identical at every step; logits within 1e-2 max-abs relative
(the north-star tolerance); the observed error is pinned tighter.  Prefill
runs token-batched by default (each layer over the whole prompt chunk: the
projections as GEMMs, the DeltaNet conv and recurrence in one launch each,
the routed experts over all (token, route) pairs); CUDALLM_MOE_PREFILL=serial
replays the one-token step per prompt token, and CUDALLM_MOE_PREFILL_CHUNK
splits the prompt into chunks that hand the conv history, recurrent state
and KV cache on to each other.
"""
import os

import numpy as np
import pytest
import torch  # noqa: F401  (a skipif condition below is evaluated in this namespace)

from myllm_b200 import CudaLLM, InvalidArgument, LengthError, OutOfRange
from myllm_b200 import synth_gguf as sg
from oracle.moe_fp64 import MoeFP64
from ranks import run_ranks

pytestmark = pytest.mark.gpu


def rel(a, b):
    return float(np.abs(a - b).max() / np.abs(b).max())


@pytest.fixture(scope="module")
def tiny_moe(model_dir, cuda):
    out = {}
    for seed in (5, 9):
        spec = sg.tiny_moe_spec(seed=seed)
        out[seed] = (spec, sg.cached_moe(spec, model_dir))
    return out


@pytest.mark.parametrize("prefill", ["batched", "serial", "chunk5"])
@pytest.mark.parametrize("seed", [5, 9])
def test_moe_parity_with_fp64_oracle(tiny_moe, seed, prefill, monkeypatch):
    if prefill == "chunk5":
        monkeypatch.setenv("CUDALLM_MOE_PREFILL_CHUNK", "5")  # 12 tokens: chunks of 5, 5, 2
    else:
        monkeypatch.setenv("CUDALLM_MOE_PREFILL", prefill)
    spec, path = tiny_moe[seed]
    prompt = sg.prompt_ids(spec.seed, 12, spec.vocab)
    ref = MoeFP64(path, max_sequence=64)
    llm = CudaLLM(path, max_sequence=64)
    assert llm.config().layer_count == spec.layers
    rt, rl = ref.prefill(prompt)
    gt = llm.prefill(prompt)
    steps = [(gt, rt, llm.last_logits(), rl)]
    for _ in range(6):
        rt2, rl2 = ref.decode(rt)
        gt = llm.decode(gt)
        rt = rt2
        steps.append((gt, rt, llm.last_logits(), rl2))
    for i, (g, r, gl, refl) in enumerate(steps):
        assert g == r, f"step {i}: token {g} != {r} (oracle margin {ref.margin(refl):.4g})"
        err = rel(gl, refl)
        assert err <= 1e-2, f"step {i}"
        assert err <= 1e-3, f"step {i}: {err:.3g}"
    llm.close()


def test_moe_reset_reproduces_and_state_is_cleared(tiny_moe):
    spec, path = tiny_moe[5]
    prompt = sg.prompt_ids(spec.seed, 10, spec.vocab)
    llm = CudaLLM(path, max_sequence=32)
    t1 = llm.prefill(prompt)
    l1 = llm.last_logits()
    d1 = llm.decode(t1)
    llm.reset()
    assert llm.position == 0
    # the DeltaNet state and conv history are zeroed by reset: same result
    assert llm.prefill(prompt) == t1
    assert np.array_equal(llm.last_logits(), l1)
    assert llm.decode(t1) == d1
    m = llm.memory_stats()
    assert m.recurrent_state_bytes > 0 and m.kv_cache_bytes > 0 and m.weight_bytes > 0
    llm.close()


def test_moe_protocol_errors(tiny_moe):
    spec, path = tiny_moe[5]
    llm = CudaLLM(path, max_sequence=8)
    with pytest.raises(InvalidArgument):
        llm.decode(1)
    with pytest.raises(InvalidArgument):
        llm.prefill([])
    with pytest.raises(OutOfRange):
        llm.prefill([spec.vocab])
    with pytest.raises(LengthError):
        llm.prefill(list(range(9)))
    t = llm.prefill([1, 2, 3])
    with pytest.raises(InvalidArgument):
        llm.prefill([1])  # prefill without reset
    for _ in range(5):
        t = llm.decode(t)
    with pytest.raises(LengthError):
        llm.decode(t)
    llm.close()


@pytest.mark.skipif("torch.cuda.device_count() < 2")
def test_moe_expert_parallel_two_gpus(tiny_moe):
    """Expert parallel over 2 GPUs (expert e on rank e % 2, one all-reduce
    per layer) gives the single-GPU result and the oracle's tokens."""
    spec, path = tiny_moe[9]
    prompt = sg.prompt_ids(spec.seed, 8, spec.vocab)
    ref = MoeFP64(path, max_sequence=64)
    rt, rl = ref.prefill(prompt)
    rtoks, rlogits = [rt], [rl]
    for _ in range(4):
        rt, rl = ref.decode(rt)
        rtoks.append(rt)
        rlogits.append(rl)
    got = run_ranks(2, path, prompt, 4)
    for r in (0, 1):
        toks, logits = got[r]
        assert toks == rtoks, r
        for i in range(len(toks)):
            assert rel(logits[i], rlogits[i]) <= 1e-3, (r, i)


def test_moe_profile_csv(tiny_moe, tmp_path):
    """The qwen35moe backend's profile CSV: the reference Profiler's format
    with the stage names of the reference's MoE GPU path."""
    import csv
    spec, path = tiny_moe[5]
    llm = CudaLLM(path, max_sequence=64)
    out = str(tmp_path / "profile.csv")
    llm.enable_profiling(out)
    tok = llm.prefill(sg.prompt_ids(spec.seed, 12, spec.vocab))
    llm.decode(tok)
    llm.disable_profiling()
    llm.close()
    with open(out, newline="") as f:
        rows = list(csv.DictReader(f))
    assert [(r["stage"], r["sequence_tokens"]) for r in rows if r["record_type"] == "forward_stage"] == \
        [("prefill.gpu_moe", "12"), ("decode.gpu_moe", "13")]
    assert sorted(r["stage"] for r in rows if r["record_type"] == "global") == \
        ["decode.gpu_moe", "forward.total", "prefill.gpu_moe"]
    for r in rows:
        assert int(r["flops"]) > 0 and int(r["read_bytes"]) > 0 and float(r["time_ms"]) > 0


def test_moe_config4_widths_against_fp64_fixture(model_dir, cuda):
    """Every config-4 width end to end: 256 experts top-8 of FFN 512 plus the
    shared expert, gated attention of 16 / 2 heads of 256 with RoPE on 64,
    DeltaNet of 16 key / 32 value heads of 128, hidden 2048, Q5_K o_proj.
    4 layers and a 4096-word vocabulary keep the FP64 restatement's fixture
    (tests/golden/make_moe_golden.py) affordable.

    The decode steps are teacher-forced with the fixture's tokens, so that a
    near-tie cannot make the rest diverge.  Logits must be within the spec's
    1e-2 at every step.  The greedy token must be equal wherever the top-1 /
    top-2 margin exceeds twice the step's observed error; a smaller margin
    is tie-ambiguous, is reported, and does not count as a match."""
    d = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "moe_a3b_width.npz"))
    spec = sg.a3b_width_spec()
    path = os.path.join(model_dir, f"{spec.name}.gguf")
    # written afresh: the hash pins the generator the fixture was made with
    assert sg.write_moe(spec, path) == str(d["sha256"])
    llm = CudaLLM(path, max_sequence=64)
    got = [(llm.prefill(d["prompt"]), llm.last_logits())]
    for i in range(1, len(d["tokens"])):
        got.append((llm.decode(int(d["tokens"][i - 1])), llm.last_logits()))
    llm.close()
    checked, ambiguous = 0, []
    for i, (tok, logits) in enumerate(got):
        ref = d["logits"][i]
        err = rel(logits, ref)
        assert err <= 1e-2, f"step {i}: {err:.3g}"
        if d["margin"][i] / np.abs(ref).max() > 2 * err:
            assert tok == int(d["tokens"][i]), f"step {i}"
            checked += 1
        else:
            ambiguous.append(i)
    assert checked >= len(got) - 1, f"tie-ambiguous steps {ambiguous}"


def test_moe_backend_queries(tiny_moe):
    """available() and MoeLLM's expert cache (moe_llm.h:49-50): every expert
    is resident, so every routed use is a hit and none is a miss."""
    spec, path = tiny_moe[5]
    llm = CudaLLM(path, max_sequence=64)
    assert llm.available() and llm.uses_gpu()
    assert llm.expert_cache_count() == spec.experts
    tok = llm.prefill(sg.prompt_ids(spec.seed, 12, spec.vocab))
    llm.decode(tok)
    st = llm.expert_cache_stats()
    assert st.misses == 0 and st.hits == 13 * spec.layers * spec.experts_used == st.requests()
    llm.close()
