"""Generate the committed golden fixtures (tests/golden/*.npz).

Run from the repository root:  python tests/golden/gen_golden.py

Each fixture holds seeded inputs (qw_b200.synth; the fp16 weights are not
stored, they regenerate from the seed), the quantized triple and
dequantized weights produced by the C oracle, and the oracle's matmul output.
The fixtures pin the oracle over time (tests/test_oracle.py regenerates and
compares) and are the golden vectors for the GPU parity tests.  Shapes cover
M = 1 / 4 / 16 / 64, K that is and is not a multiple of 512, and N that is
not a multiple of 128.

BASELINE's single configuration (17408 x 5120, M = 1 and 16) and an 8-bit,
group-128 override shape are too large to store; their oracle outputs are
pinned by SHA-256 digests in baseline_digests.json instead (the inputs
regenerate from the seeds).
"""
from __future__ import annotations

import hashlib
import json
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


DIGEST_CASES = {
    # name: (M, N, K, bits, group_size, seed)
    "single_m1_n17408_k5120": (1, 17408, 5120, 4, 64, 0),
    "single_m16_n17408_k5120": (16, 17408, 5120, 4, 64, 0),
    "override_b8_g128_m1_n5120_k17408": (1, 5120, 17408, 8, 128, 0),
}
DIGEST_FILE = os.path.join(HERE, "baseline_digests.json")


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def digest_cases():
    """{name: {array: sha256}} of the oracle's quantized triple and outputs."""
    out, weights = {}, {}
    for name, (M, N, K, bits, gs, seed) in DIGEST_CASES.items():
        key = (N, K, bits, gs, seed)
        if key not in weights:
            w = synth.weight_fp16(N, K, seed=seed, layer=0, tid=0)
            weights[key] = oracle.quantize(w, group_size=gs, bits=bits)
        wq, s, b = weights[key]
        x = synth.activations(M, K, seed=seed)
        y, y32 = oracle.quantized_matmul(x, wq, s, b, group_size=gs, bits=bits, want_f32=True)
        out[name] = {"wq": _sha(wq), "scales": _sha(s), "biases": _sha(b), "x": _sha(x), "y": _sha(y),
                     "y32": _sha(y32)}
    return out


def main():
    for name, (M, N, K, seed) in CASES.items():
        d = make_case(M, N, K, seed)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **d)
        print(f"wrote {path} ({os.path.getsize(path)} bytes)")
    with open(DIGEST_FILE, "w") as f:
        json.dump(digest_cases(), f, indent=1, sort_keys=True)
        f.write("\n")
    print(f"wrote {DIGEST_FILE}")


if __name__ == "__main__":
    main()
