"""GPU parity tests: the CUDA path (through the C ABI) against the oracle.

Bars (from the hot path's contract):
  * Q8_0 activation quantization: bit-exact (scales, int8 values, block sums);
  * per-block int32 partial dot products: bit-exact;
  * row outputs: |y_gpu - y_ref| <= 1e-5 * sum over the row's per-block float
    terms of |term| (the tree-ordered GPU sum vs the reference's sequential sum).
"""
import os

import numpy as np
import pytest
import torch

from cllm_inference_b200 import _lib, synth
from oracle.oracle import HOT_TYPES, TYPE_NAMES
from tests import gpu_helpers as G

pytestmark = pytest.mark.gpu
REL_TOL = 1e-5
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden.npz")
IDS = [TYPE_NAMES[t] for t in HOT_TYPES]


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_quantize_bit_exact(cuda, lib, oracle):
    x = synth.make_activations(5, 4096, 11) * np.float32(3.0)
    x[0, 7] = np.nan
    x[1, :32] = np.float32(1e-40)
    x[2, 64] = np.inf
    x[3, 96:128] = 0.0
    x[4, 5] = np.float32(-3e38)
    sc, qs, bs = G.quantize(lib, x)
    so, qo, bo = oracle.quantize(x)
    assert np.array_equal(bits(sc), bits(so))
    assert np.array_equal(qs, qo)
    assert np.array_equal(bs, bo)


SHAPES = [(256, 40, 1), (512, 37, 3), (4096, 300, 1), (4096, 129, 4), (4096, 64, 8), (768, 70, 9),
          (1024, 33, 2)]
SHAPES32 = [(96, 50, 2), (32, 9, 1)]


def _shapes(t):
    out = [s for s in SHAPES if s[0] % synth.BLOCK[t] == 0]
    if synth.BLOCK[t] == 32:
        out += SHAPES32
    if t == synth.Q6_K:
        out.append((14336, 40, 1))
    return out


@pytest.mark.parametrize("t", HOT_TYPES, ids=IDS)
@pytest.mark.parametrize("misalign", [0, 2], ids=["aligned", "misaligned"])
def test_partials_bit_exact(cuda, lib, oracle, t, misalign):
    for k, n, m in _shapes(t):
        w = synth.make_weights(t, n, k, seed=k * 7 + n + t)
        x = synth.make_activations(m, k, seed=k + 13 * m)
        _, qs, _ = oracle.quantize(x)
        P = G.partials(lib, qs, w, t, k, n, misalign)
        Po = oracle.partials(w, t, k, n, qs)
        assert np.array_equal(P, Po), (k, n, m, int(np.sum(P != Po)))


@pytest.mark.parametrize("t", HOT_TYPES, ids=IDS)
@pytest.mark.parametrize("misalign", [0, 2], ids=["aligned", "misaligned"])
def test_matmul_rows_within_tolerance(cuda, lib, oracle, t, misalign):
    for k, n, m in _shapes(t):
        w = synth.make_weights(t, n, k, seed=k * 3 + n + t)
        x = synth.make_activations(m, k, seed=k + 5 * m)
        bias = np.random.default_rng(n).standard_normal(n).astype(np.float32) if m == 3 else None
        y = G.matmul(lib, x, w, t, k, n, bias=bias, misalign=misalign)
        yo, ab = oracle.matmul(x, w, t, k, n, bias=bias, with_abs=True)
        G.assert_rows_close(y, yo, ab, REL_TOL, f"{TYPE_NAMES[t]} {k}x{n} m={m}")


@pytest.mark.parametrize("t", HOT_TYPES, ids=IDS)
def test_golden_fixtures(cuda, lib, t):
    """The committed vectors produced by the reference build itself."""
    g = np.load(GOLDEN)
    for case in ("seeded", "odd", "reftest", "special"):
        key = f"{TYPE_NAMES[t]}/{case}"
        k, n, m, tt = (int(v) for v in g[key + "/shape"])
        x, w = g[key + "/x"], g[key + "/w"]
        bias = g[key + "/bias"]
        bias = bias if bias.size else None
        sc, qs, bs = G.quantize(lib, x)
        assert np.array_equal(bits(sc), bits(g[key + "/scales"])), key
        assert np.array_equal(qs, g[key + "/qs"]), key
        assert np.array_equal(bs, g[key + "/bsums"]), key
        from oracle.oracle import Oracle
        _, ab = Oracle().matmul(x, w, tt, k, n, bias=bias, with_abs=True)
        for mis in (0, 2):
            y = G.matmul(lib, x, w, tt, k, n, bias=bias, misalign=mis)
            G.assert_rows_close(y, g[key + "/y"], ab, REL_TOL, key)


@pytest.mark.parametrize("t", HOT_TYPES, ids=IDS)
def test_nan_activation_sign_trick(cuda, lib, oracle, t):
    """A NaN activation quantizes to -128; the reference's AVX2 Q8_0/Q6_K dots
    then form the sign-trick product, which the GPU reproduces exactly."""
    for k, n in ((512, 64), (4096, 96)):  # direct-load path and TMA path with fused quantization
        w = synth.make_weights(t, n, k, seed=99)
        x = synth.make_activations(2, k, 3)
        x[0, [1, 2, 50, 300, 301]] = np.nan
        _, qs, _ = oracle.quantize(x)
        assert (qs == -128).sum() == 5
        assert np.array_equal(G.partials(lib, qs, w, t, k, n), oracle.partials(w, t, k, n, qs))
        y = G.matmul(lib, x, w, t, k, n)
        yo, ab = oracle.matmul(x, w, t, k, n, with_abs=True)
        assert np.all(np.isfinite(yo))
        G.assert_rows_close(y, yo, ab, REL_TOL, f"nan rows k={k}")


@pytest.mark.parametrize("t", HOT_TYPES, ids=IDS)
def test_matmul_q8_prequantized(cuda, lib, oracle, t):
    k, n, m = 1024, 77, 3
    w = synth.make_weights(t, n, k, seed=5)
    x = synth.make_activations(m, k, 6)
    x[1, 9] = np.nan
    sc, qs, bs = oracle.quantize(x)
    bias = np.arange(n, dtype=np.float32)
    y = G.matmul_q8(lib, sc, qs, bs, w, t, k, n, bias=bias)
    yo, ab = oracle.matmul(x, w, t, k, n, bias=bias, with_abs=True)
    G.assert_rows_close(y, yo, ab, REL_TOL, "matmul_q8")


@pytest.mark.parametrize("t", HOT_TYPES, ids=IDS)
def test_dequantize_bit_exact(cuda, lib, oracle, t):
    nrow, k = 9, 512
    w = synth.make_weights(t, nrow, k, seed=8)
    _, wp = G.dev_bytes(w)
    out = torch.empty(nrow * k, dtype=torch.float32, device="cuda")
    _lib.check(lib.cllm_cuda_dequantize(wp, t, nrow * k, G.dptr(out), G.stream()))
    torch.cuda.synchronize()
    assert np.array_equal(bits(out.cpu().numpy()), bits(oracle.dequantize(w, t, nrow * k)))


def test_host_io_and_registry(cuda, lib, oracle):
    """matmul_quant with host x/bias/y and a host weight pointer resolved through
    the registry (the path the quant.hpp shim uses)."""
    import ctypes

    t, k, n, m = synth.Q4_K, 4096, 500, 3
    w = synth.make_weights(t, n, k, seed=21)
    x = synth.make_activations(m, k, 22)
    bias = np.linspace(-1, 1, n, dtype=np.float32)
    y = np.full((m, n), np.nan, np.float32)
    base = w.ctypes.data
    dev = ctypes.c_void_p()
    _lib.check(lib.cllm_cuda_register_weights(ctypes.c_void_p(base), w.nbytes, ctypes.byref(dev)))
    try:
        assert (dev.value - base) % 256 == 0, "device copy keeps the host offset modulo 256"
        _lib.check(lib.cllm_cuda_matmul_quant(x.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(base), t,
                                              bias.ctypes.data_as(ctypes.c_void_p), k, n, m,
                                              y.ctypes.data_as(ctypes.c_void_p),
                                              _lib.HOST_IO | _lib.W_HOST, None))
        yo, ab = oracle.matmul(x, w, t, k, n, bias=bias, with_abs=True)
        G.assert_rows_close(y, yo, ab, REL_TOL, "host io")
        # a pointer past the range is rejected
        assert lib.cllm_cuda_matmul_quant(x.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(base + 144), t,
                                          None, k, n, m, y.ctypes.data_as(ctypes.c_void_p),
                                          _lib.HOST_IO | _lib.W_HOST, None) == _lib.ERR_INVALID_ARG
        assert lib.cllm_cuda_register_weights(ctypes.c_void_p(base + 100), 10, None) == _lib.ERR_INVALID_ARG
    finally:
        _lib.check(lib.cllm_cuda_unregister_weights(ctypes.c_void_p(base)))
    assert lib.cllm_cuda_matmul_quant(x.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(base), t, None, k, n,
                                      m, y.ctypes.data_as(ctypes.c_void_p), _lib.HOST_IO | _lib.W_HOST,
                                      None) == _lib.ERR_NOT_REGISTERED


@pytest.mark.parametrize("t,k,n,m,xoff,yoff", [(synth.Q4_K, 4096, 500, 1, 0, 0), (synth.Q4_K, 4096, 500, 3, 0, 1),
                                                (synth.Q4_K, 4096, 300, 9, 1, 0), (synth.Q6_K, 14336, 300, 1, 0, 0),
                                                (synth.Q8_0, 4096, 200, 2, 0, 0)])
def test_host_io_pinned_in_place(cuda, lib, oracle, t, k, n, m, xoff, yoff):
    """Pinned (mapped) host x and y are used in place by the GEMV path: x read
    by the quantization kernel, y written by the GEMV -- including x at a
    4-byte offset (not 16-byte aligned: the unfused quantize kernel reads it)
    and M = 9 (two row chunks)."""
    import ctypes

    w = synth.make_weights(t, n, k, seed=23)
    x = synth.make_activations(m, k, 24)
    bias = np.linspace(-1, 1, n, dtype=np.float32)
    wt, wp = G.dev_bytes(w)  # wt keeps the device copy alive
    xh = torch.empty(m * k + 4, dtype=torch.float32, pin_memory=True)
    yh = torch.full((m * n + 4,), float("nan"), dtype=torch.float32, pin_memory=True)
    xh[xoff:xoff + m * k] = torch.from_numpy(x.reshape(-1))
    bias_pinned = torch.from_numpy(bias).pin_memory()
    # a repeated call with the same pointers replays a cached graph: new x contents
    # must be seen; a pageable bias takes the direct path
    for b, bptr, xs in ((None, None, x), (bias, bias_pinned.data_ptr(), x),
                        (bias, bias_pinned.data_ptr(), -0.5 * x), (bias, bias.ctypes.data, x)):
        x = xs
        xh[xoff:xoff + m * k] = torch.from_numpy(x.reshape(-1))
        yh.fill_(float("nan"))
        _lib.check(lib.cllm_cuda_matmul_quant(ctypes.c_void_p(xh.data_ptr() + 4 * xoff), wp, t,
                                              None if bptr is None else ctypes.c_void_p(bptr), k, n, m,
                                              ctypes.c_void_p(yh.data_ptr() + 4 * yoff), _lib.HOST_IO, None))
        y = yh[yoff:yoff + m * n].numpy().reshape(m, n)
        yo, ab = oracle.matmul(x, w, t, k, n, bias=b, with_abs=True)
        G.assert_rows_close(y, yo, ab, REL_TOL, f"pinned host io {synth.NAMES[t]} m={m}")
        assert np.isnan(yh[:yoff].numpy()).all() and np.isnan(yh[yoff + m * n:].numpy()).all()


def test_host_io_graph_rebuilt_after_memory_moves(cuda, lib, oracle):
    """A cached host-I/O call graph points at the workspace and, with
    CLLM_W_HOST, at the registered weight copy.  When the workspace grows (a
    large prefill call in between) or the registration is replaced, the next
    call with the same arguments must rebuild its graph and stay correct."""
    import ctypes

    t, k, n = synth.Q4_K, 4096, 256
    w = synth.make_weights(t, n, k, seed=41)
    x = synth.make_activations(1, k, 42)
    xh = torch.from_numpy(x.reshape(-1).copy()).pin_memory()
    yh = torch.empty(n, dtype=torch.float32).pin_memory()
    yo, ab = oracle.matmul(x, w, t, k, n, with_abs=True)
    base = w.ctypes.data

    def call():
        yh.fill_(float("nan"))
        _lib.check(lib.cllm_cuda_matmul_quant(ctypes.c_void_p(xh.data_ptr()), ctypes.c_void_p(base), t, None, k, n, 1,
                                              ctypes.c_void_p(yh.data_ptr()), _lib.HOST_IO | _lib.W_HOST, None))
        G.assert_rows_close(yh.numpy().reshape(1, n), yo, ab, REL_TOL, "host io graph")

    _lib.check(lib.cllm_cuda_register_weights(ctypes.c_void_p(base), w.nbytes, None))
    try:
        call()
        call()  # replayed
        # grow the workspace: a 2048-token tcgen05 prefill over in_dim 14336
        wb = synth.make_weights_torch(synth.Q6_K, 128, 14336, seed=43)
        xb = torch.from_numpy(synth.make_activations(2048, 14336, 44)).cuda()
        yb = torch.empty(2048 * 128, device="cuda")
        _lib.check(lib.cllm_cuda_matmul_quant(G.dptr(xb), G.dptr(wb), synth.Q6_K, None, 14336, 128, 2048, G.dptr(yb),
                                              0, G.stream()))
        torch.cuda.synchronize()
        call()
        # replace the registration of the same host range
        _lib.check(lib.cllm_cuda_unregister_weights(ctypes.c_void_p(base)))
        _lib.check(lib.cllm_cuda_register_weights(ctypes.c_void_p(base), w.nbytes, None))
        call()
        call()
    finally:
        _lib.check(lib.cllm_cuda_unregister_weights(ctypes.c_void_p(base)))


def test_empty_and_degenerate(cuda, lib, oracle):
    t = synth.Q4_K
    w = synth.make_weights(t, 8, 256, 1)
    # in_dim == 0: every row is just the bias (quant.cpp: empty dot)
    bias = np.arange(8, dtype=np.float32)
    y = G.matmul(lib, np.zeros((2, 0), np.float32), np.zeros(0, np.uint8), t, 0, 8, bias=bias)
    assert np.array_equal(y, np.stack([bias, bias]))
    # all-zero activations: d = 0, id = 0, every q = 0
    y = G.matmul(lib, np.zeros((1, 256), np.float32), w, t, 256, 8)
    assert np.array_equal(y, np.zeros((1, 8), np.float32))


# the 8B decode layer shapes at M=1 and M=4, and the extra Q8_0 / Q5_K pass.
LAYER_SHAPES = [("q/o", synth.Q4_K, 4096, 4096), ("k/v", synth.Q4_K, 4096, 1024),
                ("gate/up", synth.Q4_K, 4096, 14336), ("down", synth.Q6_K, 14336, 4096),
                ("lm_head", synth.Q6_K, 4096, 128256), ("q8_0", synth.Q8_0, 4096, 4096),
                ("q5_k", synth.Q5_K, 4096, 4096)]


# BASELINE config 5 (70B) projections whose in_dim exceeds the 8B ones: the
# fused quantization holds up to 32768 activation values per row.
LAYER_SHAPES_70B = [("70b-gate/up", synth.Q4_K, 8192, 28672), ("70b-down", synth.Q6_K, 28672, 8192)]


@pytest.mark.parametrize("name,t,k,n", LAYER_SHAPES + LAYER_SHAPES_70B,
                         ids=[s[0] for s in LAYER_SHAPES + LAYER_SHAPES_70B])
def test_baseline_layer_shapes(cuda, lib, oracle, name, t, k, n):
    w = synth.make_weights(t, n, k, seed=n + k + t)
    x = synth.make_activations(4, k, seed=k)
    y4 = G.matmul(lib, x, w, t, k, n)
    yo, ab = oracle.matmul(x, w, t, k, n, with_abs=True)
    worst = G.assert_rows_close(y4, yo, ab, REL_TOL, name)
    assert worst < 1.0
    # size-independent properties: M=4 rows agree with four M=1 calls (bit for bit
    # where both run the same loop; Q4_K at M=1 has its own lane-per-super-block
    # loop, whose sums are ordered differently), and reruns are deterministic
    same_loop = not (t == synth.Q4_K and 4096 <= k <= 8192)
    for r in range(4):
        y1 = G.matmul(lib, x[r:r + 1], w, t, k, n)
        if same_loop:
            assert np.array_equal(bits(y1[0]), bits(y4[r]))
        else:
            G.assert_rows_close(y1, y4[r:r + 1], ab[r:r + 1], 2 * REL_TOL, f"{name} M=1 vs M=4 row {r}")
    assert np.array_equal(bits(G.matmul(lib, x, w, t, k, n)), bits(y4))


def test_plan_uses_tma_ring_and_fused_quantization(cuda, lib):
    """The aligned BASELINE layer shapes run on the bulk-copy ring with the
    activation quantization fused (one launch per call)."""
    import ctypes

    info = (ctypes.c_int * 8)()
    w = torch.empty(1 << 20, dtype=torch.uint8, device="cuda")
    for name, t, k, n in LAYER_SHAPES:
        for m in (1, 4):
            _lib.check(lib.cllm_cuda_matmul_plan(G.dptr(w), t, k, n, m, info, 8))
            assert info[1] == 1, (name, m, list(info))
            if not (m == 4 and k == 14336):
                assert info[2] == 1 and info[0] == 1, (name, m, list(info))


# The production loops (fused quantization; q4k_row_fused / q6k_row_fused for
# Q4_K and Q6_K; the activation image for in_dim >= 8192) must form exactly the
# reference's integer partials: checked through the parity build of the same
# launch plan (cllm_cuda_matmul_partials) on the BASELINE config-2 and 70B shapes.
@pytest.mark.parametrize("name,t,k,n", LAYER_SHAPES + LAYER_SHAPES_70B,
                         ids=[s[0] for s in LAYER_SHAPES + LAYER_SHAPES_70B])
@pytest.mark.parametrize("m", [1, 4])
def test_production_partials_bit_exact(cuda, lib, oracle, name, t, k, n, m):
    w = synth.make_weights(t, n, k, seed=n + 3 * k + t)
    x = synth.make_activations(m, k, seed=k + m)
    if m == 4:
        x[2, 33] = np.nan  # a -128 activation: the sign-trick correction path
    P = G.matmul_partials(lib, x, w, t, k, n)
    rows = G.sample_rows(n, 1024, seed=n)
    _, qs, _ = oracle.quantize(x)
    Po = oracle.partials(G.row_subset(w, synth.row_bytes(t, k), rows), t, k, len(rows), qs)
    assert np.array_equal(P[:, rows], Po), (name, m, int(np.sum(P[:, rows] != Po)))


def test_production_partials_small_and_unaligned(cuda, lib, oracle):
    """Every hot type on the direct-load and TMA paths, ragged row counts."""
    for t in HOT_TYPES:
        for k, n, m in ((256, 37, 1), (512, 70, 4), (4096, 129, 1)):
            if k % synth.BLOCK[t]:
                continue
            w = synth.make_weights(t, n, k, seed=k + n + t)
            x = synth.make_activations(m, k, seed=n)
            _, qs, _ = oracle.quantize(x)
            P = G.matmul_partials(lib, x, w, t, k, n)
            assert np.array_equal(P, oracle.partials(w, t, k, n, qs)), (TYPE_NAMES[t], k, n, m)


@pytest.mark.parametrize("k,n", [(4096, 2500), (6144, 2400), (8192, 300), (4096, 8)])
def test_q4k_superblock_loop_partials_and_rows(cuda, lib, oracle, k, n):
    """Q4_K with 16..32 super-blocks per row runs the lane-per-super-
    block loop: 16-row tiles with a ragged last tile (2500 rows), two
    super-blocks on some lanes (K = 6144), 32 lanes per row (K = 8192), and
    8-row tiles for few rows.  Partials bit-exact, rows within tolerance."""
    import ctypes

    t = synth.Q4_K
    w = synth.make_weights(t, n, k, seed=k + n)
    x = synth.make_activations(1, k, seed=k)
    info = (ctypes.c_int * 8)()
    wt, wp = G.dev_bytes(w)
    _lib.check(lib.cllm_cuda_matmul_plan(wp, t, k, n, 1, info, 8))
    assert info[2] == 1, list(info)
    _, qs, _ = oracle.quantize(x)
    P = G.matmul_partials(lib, x, w, t, k, n)
    assert np.array_equal(P, oracle.partials(w, t, k, n, qs))
    bias = np.linspace(-1, 1, n, dtype=np.float32)
    y = G.matmul(lib, x, w, t, k, n, bias=bias)
    yo, ab = oracle.matmul(x, w, t, k, n, bias=bias, with_abs=True)
    G.assert_rows_close(y, yo, ab, REL_TOL, f"Q4_K sb loop {k}x{n}")


# ---- the seven types without an integer dot kernel (quant.cpp:28-336, :1404-1430)
from oracle.oracle import ALL_TYPES, OTHER_TYPES  # noqa: E402


@pytest.mark.parametrize("t", ALL_TYPES, ids=[TYPE_NAMES[t] for t in ALL_TYPES])
def test_dequantize_all_types_bit_exact(cuda, lib, oracle, t):
    k, nrow = 512, 5
    w = synth.make_weights(t, nrow, k, seed=30 + t)
    _, wp = G.dev_bytes(w)
    out = torch.empty(nrow * k, dtype=torch.float32, device="cuda")
    _lib.check(lib.cllm_cuda_dequantize(wp, t, nrow * k, G.dptr(out), G.stream()))
    out16 = torch.empty(nrow * k, dtype=torch.int16, device="cuda")
    _lib.check(lib.cllm_cuda_dequantize_f16(wp, t, nrow * k, G.dptr(out16), G.stream()))
    torch.cuda.synchronize()
    ref = oracle.dequantize(w, t, nrow * k)
    assert np.array_equal(bits(out.cpu().numpy()), bits(ref))
    want16 = (np.ascontiguousarray(w).view(np.uint16) if t == synth.F16 else
              np.array([oracle.float_to_half(float(v)) for v in ref], np.uint16))
    assert np.array_equal(out16.cpu().numpy().view(np.uint16), want16)


@pytest.mark.parametrize("t", OTHER_TYPES, ids=[TYPE_NAMES[t] for t in OTHER_TYPES])
def test_fallback_matmul_bit_exact(cuda, lib, oracle, t):
    """matmul_quant for the fallback types sums in the reference's order: bit-exact."""
    for k, n, m in ((512, 37, 1), (4096, 300, 3), (1024, 129, 9)):
        w = synth.make_weights(t, n, k, seed=k + n + t)
        x = synth.make_activations(m, k, seed=m + t)
        bias = np.linspace(-1, 1, n, dtype=np.float32) if m == 3 else None
        y = G.matmul(lib, x, w, t, k, n, bias=bias)
        yo = oracle.matmul_fallback(x, w, t, k, n, bias=bias)
        assert np.array_equal(bits(y), bits(yo)), (TYPE_NAMES[t], k, n, m)


def test_fallback_matches_reference_build(cuda, lib, reference):
    for t in OTHER_TYPES:
        k, n, m = 768, 50, 2
        w = synth.make_weights(t, n, k, seed=7 * t)
        x = synth.make_activations(m, k, seed=t)
        assert np.array_equal(bits(G.matmul(lib, x, w, t, k, n)), bits(reference.matmul(x, w, t, k, n)))
