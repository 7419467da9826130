"""Tensor parallel (qwen2) on 2 GPUs of one box: the column/row splits with
one NCCL all-reduce after o_proj and down, and the vocab-split LM head with
the (value, index) merge, give the reference CPULLM's tokens and logits."""
import os

import numpy as np
import pytest
import torch  # noqa: F401  (the skipif condition below is evaluated in this namespace)

from myllm_b200 import synth_gguf as sg
from ranks import run_ranks

pytestmark = [pytest.mark.gpu, pytest.mark.skipif("torch.cuda.device_count() < 2")]

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def rel(a, b):
    return float(np.abs(a - b).max() / np.abs(b).max())


@pytest.mark.parametrize("n", [8, 40])
def test_tensor_parallel_two_gpus_matches_reference(model_dir, cuda, monkeypatch, n):
    monkeypatch.setenv("CUDALLM_PREFILL_GEMM", "tf32x3")  # FP32-grade prefill: the 1e-4 bar
    d = np.load(os.path.join(GOLDEN, "tiny_s7.npz"))
    path = os.path.join(model_dir, "tiny_s7.gguf")
    assert sg.write_qwen2(sg.tiny_spec(seed=7), path) == str(d["sha256"])
    got = run_ranks(2, path, d[f"prompt{n}"], 4)
    for r in (0, 1):
        toks, logits = got[r]
        assert toks == list(d[f"tokens{n}"]), r
        for i, ref in enumerate(d[f"logits{n}"]):
            assert rel(logits[i], ref) <= 1e-4, (r, i)


def test_tensor_parallel_peer_allreduce(model_dir, cuda, monkeypatch):
    """The decode all-reduces through cl_peer_allreduce (exchange buffers
    mapped by CUDA IPC, rank-order sum) instead of NCCL: the same tokens and
    logits as the reference, and bit-identical logits on both ranks."""
    monkeypatch.setenv("CUDALLM_ALLREDUCE", "p2p")  # inherited by the spawned ranks
    monkeypatch.setenv("CUDALLM_PREFILL_GEMM", "tf32x3")
    d = np.load(os.path.join(GOLDEN, "tiny_s7.npz"))
    path = os.path.join(model_dir, "tiny_s7.gguf")
    assert sg.write_qwen2(sg.tiny_spec(seed=7), path) == str(d["sha256"])
    got = run_ranks(2, path, d["prompt8"], 4)
    for r in (0, 1):
        toks, logits = got[r]
        assert toks == list(d["tokens8"]), r
        for i, ref in enumerate(d["logits8"]):
            assert rel(logits[i], ref) <= 1e-4, (r, i)
    assert np.array_equal(got[0][1], got[1][1])
