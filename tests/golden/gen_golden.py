"""Generate the committed golden fixtures (tests/golden/*.npz).

Run from the repository root:  python tests/golden/gen_golden.py

Each fixture holds seeded inputs (qw_b200.synth; the fp16 weights are not
stored, they regenerate from the seed), the quantized triple and
dequantized weights produced by the C oracle, and the oracle's matmul output.
The fixtures pin the oracle over time (tests/test_oracle.py regenerates and
compares) and are the golden vectors for the GPU parity tests.  Shapes cover
M = 1 / 4 / 16 / 64, K that is and is not a multiple of 512, and N that is
not a multiple of 128.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402
from qw_b200 import synth  # noqa: E402

CASES = {
    # name: (M, N, K, seed)
    "m1_n40_k576": (1, 40, 576, 1),
    "m1_n136_k1024": (1, 136, 1024, 2),
    "m4_n72_k1536": (4, 72, 1536, 3),
    "m16_n200_k512": (16, 200, 512, 4),
    "m7_n129_k192": (7, 129, 192, 5),
    "m64_n96_k1024": (64, 96, 1024, 6),
}


def make_case(M, N, K, seed):
    w = synth.weight_fp16(N, K, seed=seed, layer=0, tid=0)
    x = synth.activations(M, K, seed=seed)
    wq, s, b = oracle.quantize(w)
    deq0 = oracle.dequantize(wq, s, b, rounding=oracle.ROUND_TWICE)
    deq1 = oracle.dequantize(wq, s, b, rounding=oracle.ROUND_ONCE)
    y, y32 = oracle.quantized_matmul(x, wq, s, b, want_f32=True)
    return dict(x=x, wq=wq, scales=s, biases=b, deq_twice=deq0, deq_once=deq1, y=y, y32=y32)


def main():
    for name, (M, N, K, seed) in CASES.items():
        d = make_case(M, N, K, seed)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **d)
        print(f"wrote {path} ({os.path.getsize(path)} bytes)")


if __name__ == "__main__":
    main()
