"""The oracle's block decoders (oracle/quant_oracle.c) against the
reference's own Metal decoders.

The reference's CPU path pins Q4_K, Q6_K, Q8_0 and Q5_0 already
(tests/golden/blocks.npz); Q5_K is decoded only by its Metal kernels
(metal_llm.metal:447-496).  tests/golden/metal_quant_ref.npz holds what those
kernels decode (read out of the one-row product kernels with one-hot
activations, tests/golden/make_metal_quant_golden.py) for seeded rows of all
five formats, and their products with one activation row.  The decoders
must agree bit for bit; the oracle's FP32 product (dequantize, then a
sequential sum) agrees with the reference's blockwise sums within 1e-5 of
the largest output.
"""
import importlib.util
import os

import numpy as np
import pytest

import oracle
from myllm_b200 import synth_gguf as sg
from oracle import metal_ref as M

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
_spec = importlib.util.spec_from_file_location("make_metal_quant_golden",
                                               os.path.join(GOLDEN_DIR, "make_metal_quant_golden.py"))
G = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(G)


@pytest.fixture(scope="module")
def golden():
    return np.load(os.path.join(GOLDEN_DIR, "metal_quant_ref.npz"))


@pytest.mark.parametrize("gtype", G.TYPES, ids=[sg.TYPE_NAMES[t] for t in G.TYPES])
def test_decoders_match_reference_metal_decoders(gtype, golden):
    got = oracle.dequant(gtype, G.weights(gtype), G.ROWS, G.COLS)
    assert np.array_equal(got, golden[f"{sg.TYPE_NAMES[gtype]}.values"])


@pytest.mark.parametrize("gtype", G.TYPES, ids=[sg.TYPE_NAMES[t] for t in G.TYPES])
def test_products_match_reference_metal_products(gtype, golden):
    got = oracle.gemm(gtype, G.weights(gtype), G.ROWS, G.COLS, G.activation()[None, :])[0]
    ref = golden[f"{sg.TYPE_NAMES[gtype]}.product"].astype(np.float64)
    assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max()


@pytest.mark.skipif(not M.available(), reason="the reference kernels were not built here (oracle/Makefile metal)")
def test_fixture_is_what_the_reference_kernels_decode(golden):
    for gtype in G.TYPES:
        vals, prod = G.reference_values(gtype)
        name = sg.TYPE_NAMES[gtype]
        assert np.array_equal(vals, golden[name + ".values"]) and np.array_equal(prod, golden[name + ".product"])
