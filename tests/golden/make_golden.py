"""Generates tests/golden/golden.npz and tests/golden/table_traces.json from the
reference's own CPU library (oracle/_ref/libhlkv_ref.so, compiled from the
reference sources by oracle/build.py).  Run where the reference tree exists:

    python tests/golden/make_golden.py

The fixtures let the oracle be checked against the reference on machines that
do not have the reference tree (the GPU machines).
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle.oracle import Ref, table_trace  # noqa: E402

# The kernel-test scale set of the reference (tests/project2/test_dequant_cuda.cpp:76-79).
K_SCALES = np.array([1.0, 0.5, 2.0, 1.0 / 448.0, 3.7e-3, 12.5, -1.0, 0.0, 2.0 ** -20, 2.0 ** -30,
                     1e-6, 150.0, 1e4, 0.1, 65504.0 / 448.0, np.finfo(np.float32).tiny],
                    dtype=np.float32)
TRACE_CASES = [(20261011, 20000, 96, (48, 48, 64)), (1, 5000, 8, (4, 4, 4)),
               (7, 30000, 300, (100, 200, 50)), (99, 3000, 2000, (3000, 3000, 3000))]


def encode_inputs() -> np.ndarray:
    rng = np.random.default_rng(20261011)
    bits = rng.integers(0, 2 ** 32, size=1 << 16, dtype=np.uint64).astype(np.uint32)
    special = np.array([0.0, -0.0, 65504.0, 65519.996, 65520.0, 1e10, np.inf, -np.inf, np.nan,
                        448.0, 464.0, 465.0, 3e38, 57344.0, 61440.0, -1e30, 2.0 ** -10,
                        1.5 * 2.0 ** -10, -(2.0 ** -30), 2.0 ** -17, 2.0 ** -16, 1e-40, -1e-40],
                       dtype=np.float32)
    return np.concatenate([bits.view(np.float32), special])


def main() -> None:
    ref = Ref()
    g = {}
    for fmt, n in ((0, 65536), (1, 256), (2, 256)):
        g[f"decode_{fmt}"] = ref.decode(fmt, np.arange(n, dtype=np.uint16)).view(np.uint32)
    x = encode_inputs()
    g["encode_in"] = x.view(np.uint32)
    for fmt in (0, 1, 2):
        g[f"encode_{fmt}"] = ref.encode(fmt, x)
    # dequantize_reference_to_fp16 of every FP8 code under every kernel-test scale.
    codes = np.arange(256, dtype=np.uint8)
    for fmt in (1, 2):
        rows = []
        for s in K_SCALES:
            st, out = ref.dequantize_to_fp16(fmt, codes, 256, np.array([[s, 0.0]], np.float32), 256)
            assert st == 0
            rows.append(out)
        g[f"fp8_scales_{fmt}"] = np.stack(rows)
    g["k_scales"] = K_SCALES
    # quantize_reference on seeded data (with signed zeros and ties) for every format and group.
    rng = np.random.default_rng(7)
    for fmt, groups in ((0, (0,)), (1, (1, 16, 128)), (2, (16, 128)), (3, (2, 16, 128))):
        for gs in groups:
            v = (rng.standard_normal(1031) * 3).astype(np.float32)
            v[5:9] = [0.0, -0.0, 0.0, -0.0]
            v[40:44] = [-0.0, 0.0, -0.0, 0.0]
            st, p, packed = ref.quantize(fmt, v, gs)
            assert st == 0
            _, deq = ref.dequantize_to_fp16(fmt, packed, v.size, p, gs)
            g[f"q_in_{fmt}_{gs}"] = v
            g[f"q_params_{fmt}_{gs}"] = p
            g[f"q_packed_{fmt}_{gs}"] = packed
            g[f"q_fp16_{fmt}_{gs}"] = deq
    np.savez_compressed(os.path.join(HERE, "golden.npz"), **g)
    traces = {}
    for seed, steps, mb, slots in TRACE_CASES:
        t = table_trace(ref.lib, seed, steps, mb, slots)
        traces[f"{seed}:{steps}:{mb}:{','.join(map(str, slots))}"] = {
            "words": int(t.size), "sha256": hashlib.sha256(t.tobytes()).hexdigest()}
    with open(os.path.join(HERE, "table_traces.json"), "w") as f:
        json.dump(traces, f, indent=1)
    print("wrote golden.npz and table_traces.json")


if __name__ == "__main__":
    main()
