"""CPU tests of the oracle: pinned to the reference's known answers, to golden
vectors produced by the reference build, and (when oracle/_ref is present) to
the reference live, bitwise."""
import os

import numpy as np
import pytest

from cllm_inference_b200 import synth
from oracle.oracle import HOT_TYPES, TYPE_NAMES
from tests.golden.known_answers import CASES

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden.npz")


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_known_answer_dequant(oracle, case):
    _, t, block, n, expect = case
    y = oracle.dequantize(np.frombuffer(block, np.uint8), t, n)
    for i, v in expect.items():
        assert abs(y[i] - v) <= 1e-4, (i, y[i], v)


def golden_cases():
    g = np.load(GOLDEN)
    keys = sorted({k.rsplit("/", 1)[0] for k in g.files})
    return g, keys


@pytest.mark.parametrize("key", golden_cases()[1])
def test_oracle_matches_golden_bitwise(oracle, key):
    g = np.load(GOLDEN)
    k, n, m, t = (int(v) for v in g[key + "/shape"])
    x, w = g[key + "/x"], g[key + "/w"]
    bias = g[key + "/bias"]
    bias = bias if bias.size else None
    sc, qs, bs = oracle.quantize(x)
    assert np.array_equal(bits(sc), bits(g[key + "/scales"]))
    assert np.array_equal(qs, g[key + "/qs"])
    assert np.array_equal(bs, g[key + "/bsums"])
    y = oracle.matmul(x, w, t, k, n, bias=bias)
    assert np.array_equal(bits(y), bits(g[key + "/y"])), np.abs(y - g[key + "/y"]).max()


@pytest.mark.parametrize("t", HOT_TYPES, ids=[TYPE_NAMES[t] for t in HOT_TYPES])
def test_oracle_matches_reference_live(oracle, reference, t):
    for k, n, m in [(256, 40, 3), (1024, 33, 2), (4096, 16, 1)]:
        if k % synth.BLOCK[t]:
            continue
        w = synth.make_weights(t, n, k, seed=77 + t + k)
        x = synth.make_activations(m, k, seed=k + m)
        yo = oracle.matmul(x, w, t, k, n)
        yr = reference.matmul(x, w, t, k, n)
        yp = reference.matmul(x, w, t, k, n, n_threads=3)
        assert np.array_equal(bits(yo), bits(yr))
        assert np.array_equal(bits(yp), bits(yr))


def test_partials_reaccumulate(oracle):
    """The exact partials are consistent with the float row sums: summing
    them with the block scales in double lands within float error of y."""
    t, k, n = synth.Q8_0, 512, 8
    w = synth.make_weights(t, n, k, 5)
    x = synth.make_activations(1, k, 6)
    sc, qs, bs = oracle.quantize(x)
    P = oracle.partials(w, t, k, n, qs)[0]
    d = np.frombuffer(w.reshape(n, k // 32, 34)[:, :, 0:2].tobytes(), np.float16).astype(np.float64).reshape(n, -1)
    y64 = (d * sc[0][None, :] * P).sum(1)
    y = oracle.matmul(x, w, t, k, n)[0]
    assert np.allclose(y, y64, rtol=1e-5, atol=1e-5)


def test_quantize_special_values(oracle, reference):
    x = np.zeros((3, 128), np.float32)
    x[0, 1] = np.nan                       # NaN -> -128 on x86
    x[1, :32] = np.float32(1e-40)          # subnormal block: d underflows to a subnormal, id = inf
    x[2, 33] = np.inf
    x[2, 64:96] = np.linspace(-3, 3, 32, dtype=np.float32)
    so, qo, bo = oracle.quantize(x)
    sr, qr, br = reference.quantize(x)
    assert np.array_equal(bits(so), bits(sr)) and np.array_equal(qo, qr) and np.array_equal(bo, br)
    assert qo[0, 1] == -128


def test_errors(oracle):
    with pytest.raises(RuntimeError, match="not divisible by 32"):
        oracle.quantize(np.zeros((1, 33), np.float32))
    with pytest.raises(RuntimeError, match="in_dim not divisible by block size"):
        oracle.matmul(np.zeros((1, 100), np.float32), np.zeros(1000, np.uint8), synth.Q4_K, 100, 2)
