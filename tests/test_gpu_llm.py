"""End-to-end parity of CudaLLM with the reference CPULLM path.

Tokens must be identical at every step; logits must satisfy
max|g - r| / max|r| <= 1e-2 (the tolerance of the north-star spec).  With
the FP32-grade prefill GEMM (CUDALLM_PREFILL_GEMM=tf32x3) the observed error
is ~1e-5, which the tighter 1e-4 check pins; the default prefill rounds the
GEMM operands once to FP16 (11-bit significands) and is held to the spec's
1e-2 with identical tokens.
"""
import os

import numpy as np
import pytest

from myllm_b200 import CudaLLM, InvalidArgument, LengthError, OutOfRange
from myllm_b200 import synth_gguf as sg

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def rel(a, b):
    return float(np.abs(a - b).max() / np.abs(b).max())


# Logit tolerance per prefill GEMM path: FP32-grade paths 1e-4, the 16-bit
# paths the north-star 1e-2.
# Logit bars (max-abs relative).  The FP32-grade paths: split TF32 and the
# FP32 CUDA cores at 1e-4; split FP16 (three tcgen05 MMAs per step) at 5e-4,
# its accumulation over long K in the tensor cores' FP32 adders putting the
# 7B's logits at ~1.5e-4 of the CPU's (tokens identical); the one-pass 16-bit
# paths at the north-star 1e-2.
PREFILL_TOL = {"fp16x3": 5e-4, "tf32x3": 1e-4, "simt": 1e-4, "fp16": 1e-2, "bf16": 1e-2, "f16": 1e-2}


@pytest.fixture(scope="module")
def tiny_models(model_dir, cuda):
    paths = {}
    for seed in (7, 11):
        d = np.load(os.path.join(GOLDEN, f"tiny_s{seed}.npz"))
        path = os.path.join(model_dir, f"tiny_s{seed}.gguf")
        sha = sg.write_qwen2(sg.tiny_spec(seed=seed), path)
        assert sha == str(d["sha256"])
        paths[seed] = (path, d)
    return paths


@pytest.mark.parametrize("prefill", ["fp16x3", "tf32x3", "fp16"])
@pytest.mark.parametrize("seed", [7, 11])
@pytest.mark.parametrize("n", [8, 40])
def test_tiny_parity(tiny_models, monkeypatch, seed, n, prefill):
    monkeypatch.setenv("CUDALLM_PREFILL_GEMM", prefill)
    path, d = tiny_models[seed]
    llm = CudaLLM(path, max_sequence=64)
    toks = [llm.prefill(d[f"prompt{n}"])]
    logits = [llm.last_logits()]
    for _ in range(4):
        toks.append(llm.decode(toks[-1]))
        logits.append(llm.last_logits())
    assert toks == list(d[f"tokens{n}"])
    for got, ref in zip(logits, d[f"logits{n}"]):
        assert rel(got, ref) <= 1e-2
        assert rel(got, ref) <= PREFILL_TOL[prefill]
    llm.close()


@pytest.mark.parametrize("path_name", ["simt", "f16", "bf16"])
def test_prefill_gemm_paths(tiny_models, monkeypatch, path_name):
    """The other prefill GEMM paths: the FP32 CUDA-core kernel keeps the
    1e-4 bar; the single-pass FP16 tensor-core path over native blocks and
    the BF16 resident-weight path keep the spec's 1e-2."""
    path, d = tiny_models[11]
    monkeypatch.setenv("CUDALLM_PREFILL_GEMM", path_name)
    llm = CudaLLM(path, max_sequence=64)
    tok = llm.prefill(d["prompt40"])
    err = rel(llm.last_logits(), d["logits40"][0])
    assert err <= (1e-4 if path_name == "simt" else 1e-2)
    if path_name == "simt":
        assert tok == d["tokens40"][0]
    llm.close()


def test_prefill_gemm_path_rejects_unknown(tiny_models, monkeypatch):
    path, _ = tiny_models[7]
    monkeypatch.setenv("CUDALLM_PREFILL_GEMM", "int4")
    with pytest.raises(InvalidArgument):
        CudaLLM(path, max_sequence=16)


def test_prefill_chunking_matches_single_pass(tiny_models, monkeypatch):
    """A prompt split into several prefill chunks (later chunks attend to the
    earlier ones through the KV cache) gives the one-shot result, and a
    reset conversation reproduces it."""
    path, d = tiny_models[7]
    prompt = sg.prompt_ids(99, 150, 1024)
    one = CudaLLM(path, max_sequence=200)
    t1 = one.prefill(prompt)
    l1 = one.last_logits()
    d1 = one.decode(t1)
    one.reset()
    assert one.prefill(prompt) == t1 and np.array_equal(l1, one.last_logits())
    one.close()
    monkeypatch.setenv("CUDALLM_PREFILL_CHUNK", "48")
    chunked = CudaLLM(path, max_sequence=200)
    assert chunked.prefill(prompt) == t1
    assert rel(chunked.last_logits(), l1) <= 1e-6
    assert chunked.decode(t1) == d1
    chunked.close()


def test_protocol_errors(tiny_models):
    path, d = tiny_models[7]
    llm = CudaLLM(path, max_sequence=16)
    with pytest.raises(InvalidArgument):
        llm.decode(1)  # decode before prefill
    with pytest.raises(InvalidArgument):
        llm.prefill([])
    with pytest.raises(OutOfRange):
        llm.prefill([1, 2, 1024])
    with pytest.raises(OutOfRange):
        llm.prefill([-1])
    with pytest.raises(LengthError):
        llm.prefill(list(range(17)))
    tok = llm.prefill(list(range(15)))
    with pytest.raises(InvalidArgument):
        llm.prefill([1])  # requires reset
    with pytest.raises(OutOfRange):
        llm.decode(5000)
    tok = llm.decode(tok)
    assert llm.position == 16
    with pytest.raises(LengthError):
        llm.decode(tok)  # capacity reached
    llm.reset()
    assert llm.position == 0
    assert llm.prefill([3, 4]) >= 0
    stats = llm.memory_stats()
    assert stats.weight_bytes > 0 and stats.kv_cache_bytes == 2 * 2 * 16 * 2 * 64 * 4
    assert llm.uses_gpu() and "B200" in llm.device_name()
    llm.close()


def test_bad_model_files(tmp_path, cuda):
    with pytest.raises(RuntimeError):
        CudaLLM(str(tmp_path / "missing.gguf"))
    p = tmp_path / "trunc.gguf"
    full = tmp_path / "full.gguf"
    sg.write_qwen2(sg.tiny_spec(seed=7), str(full))
    p.write_bytes(full.read_bytes()[:5000])
    with pytest.raises(RuntimeError):
        CudaLLM(str(p))
    with pytest.raises(InvalidArgument):
        CudaLLM(str(full), max_sequence=10**6)


@pytest.mark.parametrize("prefill", ["fp16x3", "tf32x3", "fp16"])
def test_qwen2_05b_parity(model_dir, cuda, monkeypatch, prefill):
    """BASELINE config 0 against the reference's tokens and logits."""
    monkeypatch.setenv("CUDALLM_PREFILL_GEMM", prefill)
    d = np.load(os.path.join(GOLDEN, "qwen2_05b.npz"))
    spec = sg.CONFIGS["qwen2.5-0.5b"]
    path = os.path.join(model_dir, "qwen2.5-0.5b.gguf")
    if not os.path.exists(path) or os.path.getsize(path) == 0:
        sha = sg.write_qwen2(spec, path)
        assert sha == str(d["sha256"])
    llm = CudaLLM(path, max_sequence=64)
    toks = [llm.prefill(d["prompt"])]
    logits = [llm.last_logits()]
    for _ in range(4):
        toks.append(llm.decode(toks[-1]))
        logits.append(llm.last_logits())
    assert toks == list(d["tokens"])
    for i, lg in enumerate(logits):
        err_top = np.abs(lg[d["top_idx"][i]] - d["top_val"][i]).max()
        err_s = np.abs(lg[::16] - d["stride16"][i]).max()
        assert max(err_top, err_s) / d["maxabs"][i] <= 1e-2
        assert max(err_top, err_s) / d["maxabs"][i] <= PREFILL_TOL[prefill]
        assert abs(np.abs(lg).max() - d["maxabs"][i]) / d["maxabs"][i] <= PREFILL_TOL[prefill]
    llm.close()


@pytest.mark.parametrize("mode,prefill", [("fused", "fp16x3"), ("graph", "fp16x3"), ("fused", "tf32x3"),
                                          ("fused", "fp16")])
def test_qwen2_7b_parity(model_dir, cuda, monkeypatch, mode, prefill):
    """BASELINE config 2 (the bench workload's model, Qwen2.5-7B shape with the
    Q4_K_M layout) against the reference CPULLM's tokens and logits, through
    the one-launch decode step and through the per-operator graph."""
    monkeypatch.setenv("CUDALLM_DECODE", mode)
    monkeypatch.setenv("CUDALLM_PREFILL_GEMM", prefill)
    d = np.load(os.path.join(GOLDEN, "qwen2_7b.npz"))
    spec = sg.CONFIGS["qwen2.5-7b"]
    path = os.path.join(model_dir, "qwen2.5-7b.gguf")
    if not os.path.exists(path) or os.path.getsize(path) == 0:
        sha = sg.write_qwen2(spec, path)
        assert sha == str(d["sha256"])
    llm = CudaLLM(path, max_sequence=64)
    toks = [llm.prefill(d["prompt"])]
    logits = [llm.last_logits()]
    for _ in range(len(d["tokens"]) - 1):
        toks.append(llm.decode(toks[-1]))
        logits.append(llm.last_logits())
    assert toks == list(d["tokens"])
    for i, lg in enumerate(logits):
        err_top = np.abs(lg[d["top_idx"][i]] - d["top_val"][i]).max()
        err_s = np.abs(lg[::16] - d["stride16"][i]).max()
        # the north-star bar (1e-2) and the FP32-grade level observed at 0.5B
        assert max(err_top, err_s) / d["maxabs"][i] <= 1e-2
        assert max(err_top, err_s) / d["maxabs"][i] <= PREFILL_TOL[prefill]
    llm.close()


@pytest.mark.skipif(not os.path.exists(os.path.join(GOLDEN, "qwen2_7b_long.npz")),
                    reason="the full-length 7B golden has not been generated")
@pytest.mark.parametrize("decode,prefill,gemv", [("graph", "fp16x3", "head"), ("fused", "fp16x3", "head"),
                                                 ("graph", "tf32x3", "head"), ("graph", "fp16x3", "packed"),
                                                 ("graph", "fp16x3", "ring")])
def test_qwen2_7b_bench_workload_parity(model_dir, cuda, monkeypatch, decode, prefill, gemv):
    """The bench workload end to end: the 512-token prompt
    bench.py prefills, then 128 greedy decodes against a 4096-slot cache, on
    the default decode path (the per-operator graph, LM head on the packed
    GEMV) and the one-launch step, with every decode GEMV packed or none, with
    the default prefill GEMM (split FP16 on the tensor cores: what
    bench.py times) and split TF32.  Every token
    identical to CPULLM's; logits (the reference's top 64 and every 16th)
    within the path's bar.  (The one-pass FP16 prefill is not held to this:
    at decode 76 the reference's two best logits are 0.2 % of the largest
    apart, within that path's rounding.)"""
    monkeypatch.setenv("CUDALLM_PREFILL_GEMM", prefill)
    monkeypatch.setenv("CUDALLM_DECODE", decode)
    monkeypatch.setenv("CUDALLM_DECODE_GEMV", gemv)
    d = np.load(os.path.join(GOLDEN, "qwen2_7b_long.npz"))
    assert int(d["cpullm_checked"]) == 1, "fixture not cross-checked against CPULLM itself"
    spec = sg.CONFIGS["qwen2.5-7b"]
    path = os.path.join(model_dir, "qwen2.5-7b.gguf")
    if not os.path.exists(path) or os.path.getsize(path) == 0:
        assert sg.write_qwen2(spec, path) == str(d["sha256"])
    assert np.array_equal(d["prompt"], sg.prompt_ids(spec.seed, 512, spec.vocab))
    llm = CudaLLM(path, max_sequence=4096)
    toks = [llm.prefill(d["prompt"])]
    errs = []
    for i in range(len(d["tokens"])):
        lg = llm.last_logits()
        err = max(np.abs(lg[d["top_idx"][i]] - d["top_val"][i]).max(), np.abs(lg[::16] - d["stride16"][i]).max())
        errs.append(err / d["maxabs"][i])
        if i + 1 < len(d["tokens"]):
            toks.append(llm.decode(toks[-1]))
    llm.close()
    assert toks == list(d["tokens"])
    assert max(errs) <= PREFILL_TOL[prefill], (int(np.argmax(errs)), max(errs))


def test_profile_csv(tiny_models, tmp_path):
    """enable_profiling writes the reference Profiler's CSV format: one
    forward_total and one forward_stage row per call (stage names of the
    reference's resident GPU path), global rows when profiling stops."""
    import csv
    path, d = tiny_models[7]
    llm = CudaLLM(path, max_sequence=64)
    out = str(tmp_path / "profile.csv")
    llm.enable_profiling(out)
    tok = llm.prefill(d["prompt8"])
    for _ in range(2):
        tok = llm.decode(tok)
    llm.disable_profiling()
    llm.close()
    with open(out, newline="") as f:
        rows = list(csv.DictReader(f))
    stages = [(r["record_type"], r["stage"], r["sequence_tokens"]) for r in rows]
    assert stages[:6] == [("forward_total", "forward.total", "8"), ("forward_stage", "prefill.gpu_resident", "8"),
                          ("forward_total", "forward.total", "9"), ("forward_stage", "decode.gpu_resident", "9"),
                          ("forward_total", "forward.total", "10"), ("forward_stage", "decode.gpu_resident", "10")]
    assert sorted(r["stage"] for r in rows[6:]) == ["decode.gpu_resident", "forward.total", "prefill.gpu_resident"]
    for r in rows:
        assert int(r["flops"]) > 0 and int(r["read_bytes"]) > 0 and float(r["time_ms"]) > 0


def test_backend_queries(tiny_models):
    path, _ = tiny_models[7]
    llm = CudaLLM(path, max_sequence=64)
    assert llm.available() and llm.uses_gpu() and llm.device_name()
    assert llm.expert_cache_count() == 0 and llm.expert_cache_stats().requests() == 0
    llm.close()
