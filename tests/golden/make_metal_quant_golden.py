"""Golden values of the reference's own Metal block decoders.

The reference decodes Q5_K only on Metal (metal_llm.metal:447-496; its CPU
path has no Q5_K decoder).  Its one-row product kernels (metal_gevm_*_f32,
compiled as C++ into oracle/_ref/libref_metal.so, see oracle/metal_ref.py)
are run here with one-hot activations: for x = e_j the dot of a row is that
row's decoded value at column j (every other term is an exact zero), so the
product kernel reads out the reference's decoding of every weight.  For each
of Q4_K, Q5_K, Q6_K, Q8_0 and Q5_0, eight seeded rows of 512 columns
(myllm_b200.synth_gguf, rebuilt from the seed in the test) give the decoded
values and the products with one seeded activation row; both are stored in
tests/golden/metal_quant_ref.npz.

    python tests/golden/make_metal_quant_golden.py    # needs the built library
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from myllm_b200 import synth_gguf as sg  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "metal_quant_ref.npz")
TYPES = (sg.Q4_K, sg.Q5_K, sg.Q6_K, sg.Q8_0, sg.Q5_0)
ROWS, COLS = 8, 512


def weights(gtype):
    return sg.fill(gtype, ROWS, COLS, sg.stream_key(7, f"mq{gtype}"), 0.0, 0.02)


def activation():
    return sg.normal(COLS, sg.stream_key(7, "mqx"), 0.0, 1.0).astype(np.float32)


def reference_product(gtype, w, x):
    """The reference's one-row product of rows w with x."""
    from oracle import metal_ref as M
    w = np.ascontiguousarray(w)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(w.shape[0], np.float32)
    if M.lib().mref_gevm(gtype, M._ptr(w), M._ptr(x), M._ptr(y), w.shape[0], COLS, w.shape[1]) != 0:
        raise ValueError(f"no reference product kernel for type {gtype}")
    return y


def reference_values(gtype):
    """(decoded values [ROWS, COLS], product with activation()) of the
    reference's kernel on weights(gtype)."""
    w = weights(gtype)
    vals = np.zeros((ROWS, COLS), np.float32)
    for j in range(COLS):
        e = np.zeros(COLS, np.float32)
        e[j] = 1.0
        vals[:, j] = reference_product(gtype, w, e)
    return vals, reference_product(gtype, w, activation())


def main():
    from oracle import metal_ref as M
    if not M.available():
        raise SystemExit("build oracle/_ref/libref_metal.so first (make -C oracle metal REF=<reference checkout>)")
    arrays = {}
    for gtype in TYPES:
        vals, prod = reference_values(gtype)
        arrays[f"{sg.TYPE_NAMES[gtype]}.values"] = vals
        arrays[f"{sg.TYPE_NAMES[gtype]}.product"] = prod
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT}: {len(arrays)} arrays")


if __name__ == "__main__":
    main()
