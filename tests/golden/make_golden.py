"""Generate tests/golden/golden.npz from the reference's own code.

Runs the UNMODIFIED reference hot path (cllm_inference src/core/quant.cpp,
built into oracle/_ref/libcllm_ref.so by oracle/Makefile) on seeded inputs and
stores inputs and outputs, so that the oracle and the GPU kernels are pinned to
the reference on machines where the reference tree is absent.

Cases per hot-path type T:
  T/seeded   synthetic blocks (cllm_inference_b200.synth), N(0,1) activations,
             K=512, N=24 rows, M=3, with a bias
  T/odd      K=96 (3 blocks; 32-value types) or K=768 (K types), N=7, M=2
  T/reftest  the input generators of the reference's tests/quant_test.cpp:
             d=1.0 at offset 0, other bytes (k+blk+j)%7 (:244-256),
             x = ((i+t)%5-2)*0.5 (:343-347); K=64 or 256, N=40, M=3
  T/special  activations with NaN, +-inf, zeros, subnormals and huge values
Each case stores w (uint8), x, bias (may be empty), y = matmul_quant_batch,
and the quantized activations (scales, qs, bsums) of quantize_row_q8_0.

Usage: python tests/golden/make_golden.py   (needs oracle/_ref; run from the repo root)
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from cllm_inference_b200 import synth  # noqa: E402
from oracle.oracle import HOT_TYPES, TYPE_NAMES, Reference, build  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")


def reftest_weights(t, k, n):
    bs, ts = synth.BLOCK[t], synth.TSIZE[t]
    w = np.zeros((n, k // bs, ts), np.uint8)
    for j in range(n):
        for blk in range(k // bs):
            w[j, blk, 0:2] = (0x00, 0x3C)
            for kk in range(2, ts):
                w[j, blk, kk] = (kk + blk + j) % 7
    return w.reshape(-1)


def special_x(m, k, seed):
    x = synth.make_activations(m, k, seed)
    x[0, 3] = np.nan
    x[0, 40] = np.nan
    x[0, 70:102] = 0.0
    x[1 % m, 5] = np.inf
    x[1 % m, 200] = -np.inf
    if k >= 512:
        x[0, 300:332] = np.float32(1e-41)   # a block of subnormals
        x[0, 400] = np.float32(3e38)
    return x


def main():
    build()
    ref = Reference()
    out = {}
    for t in HOT_TYPES:
        name = TYPE_NAMES[t]
        big = synth.BLOCK[t] == 256
        cases = {
            "seeded": (synth.make_weights(t, 24, 512, seed=1000 + t), synth.make_activations(3, 512, 2000 + t),
                       np.random.default_rng(t).standard_normal(24).astype(np.float32), 512, 24),
            "odd": (synth.make_weights(t, 7, 768 if big else 96, seed=3000 + t),
                    synth.make_activations(2, 768 if big else 96, 4000 + t), None, 768 if big else 96, 7),
            "reftest": (reftest_weights(t, 256 if big else 64, 40),
                        np.array([[((i + r) % 5 - 2) * 0.5 for i in range(256 if big else 64)] for r in range(3)],
                                 np.float32), None, 256 if big else 64, 40),
            "special": (synth.make_weights(t, 16, 512, seed=5000 + t), special_x(2, 512, 6000 + t), None, 512, 16),
        }
        for cname, (w, x, bias, k, n) in cases.items():
            y = ref.matmul(x, w, t, k, n, bias=bias)
            sc, qs, bs = ref.quantize(x)
            key = f"{name}/{cname}"
            out[key + "/w"] = w
            out[key + "/x"] = x
            out[key + "/bias"] = bias if bias is not None else np.zeros(0, np.float32)
            out[key + "/y"] = y
            out[key + "/scales"] = sc
            out[key + "/qs"] = qs
            out[key + "/bsums"] = bs
            out[key + "/shape"] = np.array([k, n, x.shape[0], t], np.int64)
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    main()
