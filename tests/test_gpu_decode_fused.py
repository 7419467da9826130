"""The one-launch decode step (cl_qwen2_decode_step) against the reference.

With CUDALLM_DECODE=fused, CudaLLM runs a one-GPU qwen2 decode step as a
single persistent launch (every layer matrix Q4_K / Q6_K, 128-wide heads:
the 7B and 14B shapes; construction fails if the model does not qualify,
so these tests cannot pass on a silent fallback); the default is the
per-operator graph (CUDALLM_DECODE=graph).  Both must give the reference CPULLM's greedy tokens at every
step and logits within 1e-4 (max-abs relative), on a small model with the
7B's structure (head_dim 128, 7 query heads per KV head): a short prompt
(one attention split) and a 1100-token prompt (32 key splits of 35 keys),
and the long prompt again with 4 splits forced (CUDALLM_DECODE_SPLITS): 276
keys per split in five 64-key tiles, the KV append landing in the last
split's last tile.
"""
import os

import numpy as np
import pytest

from myllm_b200 import CudaLLM
from myllm_b200 import synth_gguf as sg

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def rel(a, b):
    return float(np.abs(a - b).max() / np.abs(b).max())


@pytest.fixture(scope="module")
def small(model_dir, cuda):
    d = np.load(os.path.join(GOLDEN, "q4km_d128.npz"))
    path = os.path.join(model_dir, "q4km_d128.gguf")
    if not os.path.exists(path) or os.path.getsize(path) == 0:
        assert sg.write_qwen2(sg.q4km_small_spec(), path) == str(d["sha256"])
    return path, d


def run(path, prompt, steps, monkeypatch, mode, max_sequence=2048, prefill="tf32x3", splits=None):
    monkeypatch.setenv("CUDALLM_DECODE", mode)
    if splits is not None:
        monkeypatch.setenv("CUDALLM_DECODE_SPLITS", str(splits))
    monkeypatch.setenv("CUDALLM_PREFILL_GEMM", prefill)
    llm = CudaLLM(path, max_sequence=max_sequence)
    toks = [llm.prefill(prompt)]
    logits = [llm.last_logits()]
    for _ in range(steps):
        toks.append(llm.decode(toks[-1]))
        logits.append(llm.last_logits())
    llm.close()
    return toks, logits


@pytest.mark.parametrize("mode", ["fused", "graph"])
@pytest.mark.parametrize("n", [8, 1100])
def test_small_model_matches_reference(small, monkeypatch, mode, n):
    path, d = small
    toks, logits = run(path, d[f"prompt{n}"], 4, monkeypatch, mode)
    assert toks == list(d[f"tokens{n}"])
    for i, ref in enumerate(d[f"logits{n}"]):
        assert rel(logits[i], ref) <= 1e-4, (i, rel(logits[i], ref))


def test_small_model_multi_tile_splits(small, monkeypatch):
    """Four key splits over 1100+ keys: every split runs five key tiles
    (the first from the prefetch during the QKV phase, the rest loaded in
    attention)."""
    path, d = small
    toks, logits = run(path, d["prompt1100"], 4, monkeypatch, "fused", splits=4)
    assert toks == list(d["tokens1100"])
    for i, ref in enumerate(d["logits1100"]):
        assert rel(logits[i], ref) <= 1e-4, (i, rel(logits[i], ref))


@pytest.mark.parametrize("n", [8, 1100])
def test_small_model_default_paths(small, monkeypatch, n):
    """The default prefill (split FP16 GEMM) with the fused decode step: the
    reference's tokens, logits within 1e-4."""
    path, d = small
    monkeypatch.delenv("CUDALLM_PREFILL_GEMM", raising=False)
    monkeypatch.setenv("CUDALLM_DECODE", "fused")
    llm = CudaLLM(path, max_sequence=2048)
    toks = [llm.prefill(d[f"prompt{n}"])]
    logits = [llm.last_logits()]
    for _ in range(4):
        toks.append(llm.decode(toks[-1]))
        logits.append(llm.last_logits())
    llm.close()
    assert toks == list(d[f"tokens{n}"])
    for i, ref in enumerate(d[f"logits{n}"]):
        assert rel(logits[i], ref) <= 1e-4, (i, rel(logits[i], ref))


def test_fused_step_is_deterministic(small, monkeypatch):
    """Partial sums are added in warp order, never in arrival order: two
    runs give bit-identical logits."""
    path, d = small
    a = run(path, d["prompt8"], 3, monkeypatch, "fused")
    b = run(path, d["prompt8"], 3, monkeypatch, "fused")
    assert a[0] == b[0]
    for x, y in zip(a[1], b[1]):
        assert np.array_equal(x, y)


def test_fused_step_across_reset(small, monkeypatch):
    """The control block is re-armed by every step: a second conversation on
    the same model (reset, new prefill) decodes the same tokens."""
    path, d = small
    monkeypatch.setenv("CUDALLM_DECODE", "fused")
    monkeypatch.setenv("CUDALLM_PREFILL_GEMM", "tf32x3")
    llm = CudaLLM(path, max_sequence=2048)
    for _ in range(2):
        llm.reset()
        toks = [llm.prefill(d["prompt8"])]
        for _ in range(4):
            toks.append(llm.decode(toks[-1]))
        assert toks == list(d["tokens8"])
    llm.close()


def test_fused_refuses_models_it_does_not_support(model_dir, cuda, monkeypatch):
    """A model with 64-wide heads and 32-column formats (the tiny model) is
    refused when the fused step is insisted on, and decoded by the graph
    otherwise."""
    path = os.path.join(model_dir, "tiny_s7.gguf")
    sg.write_qwen2(sg.tiny_spec(seed=7), path)
    monkeypatch.setenv("CUDALLM_DECODE", "fused")
    with pytest.raises(Exception, match="fused decode"):
        CudaLLM(path, max_sequence=64)
    monkeypatch.delenv("CUDALLM_DECODE")
    llm = CudaLLM(path, max_sequence=64)
    llm.close()
