"""CPU tests: the oracle is pinned to the reference, the generator is stable."""
import os

import numpy as np
import pytest

import oracle
from myllm_b200 import synth_gguf as sg

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.mark.parametrize("name,gtype", [("Q4_K", sg.Q4_K), ("Q6_K", sg.Q6_K), ("Q5_0", sg.Q5_0), ("Q8_0", sg.Q8_0)])
def test_port_dequant_matches_reference_blocks(name, gtype):
    """Known-answer vectors: the reference GgufDequantizer's values, bit-exact."""
    d = np.load(os.path.join(GOLDEN, "blocks.npz"))
    raw, ref = d[f"raw_{name}"], d[f"ref_{name}"]
    got = oracle.dequant(gtype, raw, ref.shape[0], ref.shape[1])
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("seed", [7, 11])
def test_generator_reproduces_fixture_model(seed, tmp_path):
    d = np.load(os.path.join(GOLDEN, f"tiny_s{seed}.npz"))
    sha = sg.write_qwen2(sg.tiny_spec(seed=seed), str(tmp_path / "m.gguf"))
    assert sha == str(d["sha256"])


def test_quantizers_round_trip_within_format_error():
    x = sg.normal(64 * 512, sg.stream_key(3, "x"), 0.0, 0.02).reshape(64, 512)
    for gtype, tol in ((sg.Q8_0, 0.002), (sg.Q6_K, 0.004), (sg.Q5_0, 0.006), (sg.Q5_K, 0.006), (sg.Q4_K, 0.012)):
        q = sg.quantize(x, gtype)
        y = oracle.dequant(gtype, q, 64, 512)
        assert np.abs(y - x).max() < tol, sg.TYPE_NAMES[gtype]


def test_q5k_decoder_matches_independent_numpy():
    """Q5_K has no CPU decoder in the reference; check the C port against a
    vectorised restatement of metal_llm.metal:447-496."""
    x = sg.normal(8 * 512, sg.stream_key(5, "q5k"), 0.0, 0.02).reshape(8, 512)
    q = sg.quantize(x, sg.Q5_K)
    got = oracle.dequant(sg.Q5_K, q, 8, 512)
    blocks = q.reshape(8, 2, 176)
    d = blocks[..., 0:2].copy().view(np.float16).astype(np.float32)[..., 0]
    dmin = blocks[..., 2:4].copy().view(np.float16).astype(np.float32)[..., 0]
    s = blocks[..., 4:16].astype(np.int32)
    qh = blocks[..., 16:48].astype(np.int32)
    qs = blocks[..., 48:176].astype(np.int32)
    out = np.zeros((8, 2, 256), dtype=np.float32)
    for i in range(8):
        if i < 4:
            sc, m = s[..., i] & 63, s[..., i + 4] & 63
        else:
            sc = (s[..., i + 4] & 15) | ((s[..., i - 4] >> 6) << 4)
            m = (s[..., i + 4] >> 4) | ((s[..., i] >> 6) << 4)
        g, hi = i // 2, i % 2
        nib = (qs[..., g * 32:(g + 1) * 32] >> (4 * hi)) & 15
        bit = (qh >> i) & 1
        qv = nib + 16 * bit
        out[..., i * 32:(i + 1) * 32] = ((d * sc)[..., None] * qv - (dmin * m)[..., None]).astype(np.float32)
    np.testing.assert_allclose(got, out.reshape(8, 512), rtol=0, atol=1e-7)


def test_oracle_gemm_matches_numpy():
    x = sg.normal(4 * 256, sg.stream_key(9, "x"), 0.0, 1.0).reshape(4, 256)
    w = sg.fill(sg.Q4_K, 64, 256, sg.stream_key(9, "w"), 0.0, 0.02)
    ref = x.astype(np.float64) @ oracle.dequant(sg.Q4_K, w, 64, 256).astype(np.float64).T
    got = oracle.gemm(sg.Q4_K, w, 64, 256, x)
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5)


@pytest.mark.skipif(not oracle.ref_available(), reason="reference CPU path not built here")
def test_reference_tokens_match_fixture(tmp_path):
    d = np.load(os.path.join(GOLDEN, "tiny_s7.npz"))
    path = str(tmp_path / "m.gguf")
    sg.write_qwen2(sg.tiny_spec(seed=7), path)
    ref = oracle.ReferenceCPU(path)
    tok, lg = ref.prefill(d["prompt8"])
    assert tok == d["tokens8"][0]
    assert np.array_equal(lg, d["logits8"][0])
    ref.close()


@pytest.mark.skipif(not oracle.ref_available(), reason="reference CPU path not built here")
def test_port_dequant_matches_reference_on_every_tensor(tmp_path):
    spec = sg.tiny_spec(seed=11)
    path = str(tmp_path / "m.gguf")
    sg.write_qwen2(spec, path)
    ref = oracle.ReferenceCPU(path)
    for l in range(spec.layers):
        for name in ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"):
            want = ref.tensor(l, name)
            rows, cols = want.shape
            raw = sg.fill(spec.types(l, name), rows, cols, sg.stream_key(spec.seed, f"blk.{l}.{name}.weight"),
                          0.0, spec.weight_std)
            got = oracle.dequant(spec.types(l, name), raw, rows, cols)
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (l, name)
    ref.close()
