"""Batched prefill (matmul_quant_batch, n_rows >= 32) on the tcgen05 GEMM
against the oracle, with the same row tolerance as the decode path:
|y_gpu - y_ref| <= 1e-5 * sum over the row's per-block float terms of |term|."""
import ctypes

import numpy as np
import pytest
import torch

from cllm_inference_b200 import _lib, synth
from tests import gpu_helpers as G

pytestmark = pytest.mark.gpu
REL_TOL = 1e-5

# (K, N, M): a single tile, ragged token and row tiles, several super-blocks
SHAPES = [(256, 128, 32), (1024, 136, 48), (256, 128, 64), (256, 200, 100), (1024, 300, 129), (4096, 256, 128),
          (4096, 300, 257)]


def plan(lib, w_ptr, t, k, n, m):
    info = (ctypes.c_int * 8)()
    _lib.check(lib.cllm_cuda_matmul_plan(w_ptr, t, k, n, m, info, 8))
    return list(info)


@pytest.mark.parametrize("k,n,m", SHAPES)
def test_prefill_q4k_tcgen05(cuda, lib, oracle, k, n, m):
    t = synth.Q4_K
    w = synth.make_weights(t, n, k, seed=k + n + m)
    x = synth.make_activations(m, k, seed=m)
    bias = np.linspace(-2, 2, n, dtype=np.float32) if m % 2 else None
    _, wp = G.dev_bytes(w)
    assert plan(lib, wp, t, k, n, m)[1] == 2, "expected the tcgen05 path"
    y = G.matmul(lib, x, w, t, k, n, bias=bias)
    yo, ab = oracle.matmul(x, w, t, k, n, bias=bias, with_abs=True)
    G.assert_rows_close(y, yo, ab, REL_TOL, f"prefill {k}x{n} m={m}")


def test_prefill_threshold(cuda, lib):
    """31 rows run the GEMV in chunks, 32 rows the tensor-core GEMM."""
    for t, k in ((synth.Q4_K, 4096), (synth.Q6_K, 4096)):
        w = torch.empty(synth.row_bytes(t, k) * 64, dtype=torch.uint8, device="cuda")
        assert plan(lib, G.dptr(w), t, k, 64, 31)[1] != 2
        assert plan(lib, G.dptr(w), t, k, 64, 32)[1] == 2


def test_prefill_matches_decode_rows(cuda, lib):
    """Rows of a 64-row prefill equal 1-row calls within the row tolerance."""
    from oracle.oracle import Oracle

    t, k, n, m = synth.Q4_K, 4096, 160, 64
    w = synth.make_weights(t, n, k, seed=3)
    x = synth.make_activations(m, k, seed=4)
    y = G.matmul(lib, x, w, t, k, n)
    _, ab = Oracle().matmul(x[:8], w, t, k, n, with_abs=True)
    for r in range(8):
        y1 = G.matmul(lib, x[r:r + 1], w, t, k, n)
        G.assert_rows_close(y[r:r + 1], y1, ab[r:r + 1], 2 * REL_TOL, f"row {r}")


def _tile_samples(count: int, tile: int, rng) -> np.ndarray:
    """Indices covering every tile of `tile` entries: its first and last entry
    and one seeded entry inside it."""
    out = []
    for b in range(0, count, tile):
        e = min(count, b + tile) - 1
        out += [b, e, int(rng.integers(b, e + 1))]
    return np.unique(np.array(out))


@pytest.mark.parametrize("m", [64, 512, 2048])
def test_prefill_config3_exact_shape(cuda, lib, oracle, m):
    """BASELINE config 3 itself: Q4_K 14336x4096 at M = 64, 512, 2048 on the
    tcgen05 GEMM.  Every output row tile and every token tile is checked
    against the oracle (three rows per 128-row tile; all tokens up to M=512,
    three per 128-token tile at M=2048)."""
    t, k, n = synth.Q4_K, 4096, 14336
    w = synth.make_weights(t, n, k, seed=31337)
    x = synth.make_activations(m, k, seed=m + 1)
    _, wp = G.dev_bytes(w)
    assert plan(lib, wp, t, k, n, m)[1] == 2, "expected the tcgen05 path"
    y = G.matmul(lib, x, w, t, k, n)
    rng = np.random.default_rng(m)
    rows = _tile_samples(n, 128, rng)
    toks = np.arange(m) if m <= 512 else _tile_samples(m, 128, rng)
    yo, ab = oracle.matmul(x[toks], G.row_subset(w, synth.row_bytes(t, k), rows), t, k, len(rows),
                           with_abs=True)
    G.assert_rows_close(y[np.ix_(toks, rows)], yo, ab, REL_TOL, f"config 3 M={m}")


# Q6_K: K a multiple of 2048 keeps its 210-byte-per-super-block rows 16-byte
# multiples (the tensor map's row pitch); the full int8 scale range makes
# sc * (q6 - 32) exceed fp16's exact integers, which the kernel must not need.
Q6_SHAPES = [(2048, 128, 32), (4096, 200, 47), (2048, 128, 64), (2048, 200, 100), (4096, 300, 129),
             (4096, 256, 257), (6144, 136, 192)]


@pytest.mark.parametrize("k,n,m", Q6_SHAPES)
def test_prefill_q6k_tcgen05(cuda, lib, oracle, k, n, m):
    t = synth.Q6_K
    w = synth.make_weights(t, n, k, seed=k + n + m, q6_scale_max=128)
    x = synth.make_activations(m, k, seed=m + 7)
    bias = np.linspace(-2, 2, n, dtype=np.float32) if m % 2 else None
    _, wp = G.dev_bytes(w)
    assert plan(lib, wp, t, k, n, m)[1] == 2, "expected the tcgen05 path"
    y = G.matmul(lib, x, w, t, k, n, bias=bias)
    yo, ab = oracle.matmul(x, w, t, k, n, bias=bias, with_abs=True)
    G.assert_rows_close(y, yo, ab, REL_TOL, f"Q6_K prefill {k}x{n} m={m}")


def test_prefill_q6k_nan_tokens(cuda, lib, oracle):
    """Tokens with NaN inputs: the NaN quantizes to -128 and the AVX2 sign
    trick turns -128 * w (w < 0) into 128 * w; the fix-up kernel must
    reproduce it.  Tokens with one NaN, a NaN in every block, and all-NaN."""
    t, k, n, m = synth.Q6_K, 2048, 256, 96
    w = synth.make_weights(t, n, k, seed=5, q6_scale_max=128)
    x = synth.make_activations(m, k, seed=6)
    x[3, 17] = np.nan
    x[40, ::32] = np.nan
    x[41, 5::32] = np.nan
    x[95, :] = np.nan
    _, wp = G.dev_bytes(w)
    assert plan(lib, wp, t, k, n, m)[1] == 2
    y = G.matmul(lib, x, w, t, k, n)
    yo, ab = oracle.matmul(x, w, t, k, n, with_abs=True)
    assert np.isfinite(yo[[3, 40, 41, 95]]).all()
    G.assert_rows_close(y, yo, ab, REL_TOL, "Q6_K prefill, NaN tokens")


def test_prefill_q6k_ineligible_rows_take_gemv(cuda, lib):
    """K = 1024 gives 840-byte rows (not 16-byte multiples): the plan keeps the GEMV path."""
    t, k, n, m = synth.Q6_K, 1024, 64, 128
    w = synth.make_weights(t, n, k, seed=1)
    _, wp = G.dev_bytes(w)
    assert plan(lib, wp, t, k, n, m)[1] != 2


@pytest.mark.parametrize("m", [64, 512])
def test_prefill_q6k_config3_down_shape(cuda, lib, oracle, m):
    """The config-3 FFN down projection as Q6_K (4096 rows x 14336 in) at
    M = 64 (32 tiles: split-K over four CTAs per tile) and M = 512 on the
    tcgen05 GEMM: three rows per 128-row tile, every token."""
    t, k, n = synth.Q6_K, 14336, 4096
    w = synth.make_weights(t, n, k, seed=4242, q6_scale_max=128)
    x = synth.make_activations(m, k, seed=77 + m)
    _, wp = G.dev_bytes(w)
    assert plan(lib, wp, t, k, n, m)[1] == 2, "expected the tcgen05 path"
    y = G.matmul(lib, x, w, t, k, n)
    rows = _tile_samples(n, 128, np.random.default_rng(9))
    yo, ab = oracle.matmul(x, G.row_subset(w, synth.row_bytes(t, k), rows), t, k, len(rows), with_abs=True)
    G.assert_rows_close(y[:, rows], yo, ab, REL_TOL, f"config 3 down as Q6_K, M={m}")


@pytest.mark.parametrize("t,k", [(synth.Q4_K, 1024), (synth.Q6_K, 2048)])
def test_prefill_unaligned_activations(cuda, lib, oracle, t, k):
    """x 4 bytes past a 16-byte boundary: the activation preparation falls
    back to scalar loads; the tensor-core GEMM itself is unaffected."""
    n, m = 136, 70
    w = synth.make_weights(t, n, k, seed=k + 3, q6_scale_max=128)
    x = synth.make_activations(m, k, seed=k + 4)
    wt, wp = G.dev_bytes(w)
    assert plan(lib, wp, t, k, n, m)[1] == 2
    xb = torch.zeros(m * k + 4, dtype=torch.float32, device="cuda")
    xb[1:1 + m * k] = torch.from_numpy(x.reshape(-1)).cuda()
    y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    _lib.check(lib.cllm_cuda_matmul_quant(ctypes.c_void_p(xb.data_ptr() + 4), wp, t, None, k, n, m, G.dptr(y), 0,
                                          G.stream()))
    torch.cuda.synchronize()
    yo, ab = oracle.matmul(x, w, t, k, n, with_abs=True)
    G.assert_rows_close(y.cpu().numpy(), yo, ab, REL_TOL, f"unaligned x {synth.NAMES[t]}")
