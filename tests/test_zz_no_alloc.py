"""The allocation-free entry point, cllm_cuda_matmul_quant_noalloc.

It exists for callers that cannot let the library allocate device memory
during a call: a decode step being recorded into a CUDA graph (allocations
are not capturable), an engine whose own allocator already owns the GPU's
memory, or a latency-critical loop that cannot absorb the device-wide
synchronisation a growing workspace costs.  It keeps its scratch (the
quantized activations) in one fixed array inside the library instead.

This file is named to be collected last: if it fails, a run that stops at the
first failure has already run every other test.  It passes on its own in a
fresh process too (it needs only the session fixtures).
"""
import ctypes

import numpy as np
import pytest
import torch

from cllm_inference_b200 import _lib, synth
from tests import gpu_helpers as G

pytestmark = pytest.mark.gpu
REL_TOL = 1e-5  # the row tolerance of the GPU parity tests

MAX_ROWS, MAX_IN_DIM = 8, 32768  # CLLM_NOALLOC_MAX_ROWS / _IN_DIM in include/cllm_cuda.h


def _both(lib, x, w, t, k, n, bias):
    """Outputs of the regular and of the allocation-free entry point, same device inputs."""
    m = x.shape[0]
    xd = G.to_dev(x)
    _, wp = G.dev_bytes(w)
    bd = G.to_dev(bias)
    y_ref = torch.full((m, n), float("nan"), device="cuda")
    y_na = torch.full((m, n), float("nan"), device="cuda")
    _lib.check(lib.cllm_cuda_matmul_quant(G.dptr(xd), wp, t, G.dptr(bd), k, n, m, G.dptr(y_ref), 0, G.stream()))
    _lib.check(lib.cllm_cuda_matmul_quant_noalloc(G.dptr(xd), wp, t, G.dptr(bd), k, n, m, G.dptr(y_na),
                                                  G.stream()))
    torch.cuda.synchronize()
    _lib.check(lib.cllm_cuda_check_device_status())
    return y_ref.cpu().numpy(), y_na.cpu().numpy()


def test_noalloc_matches_regular_entry_on_two_calls(cuda, lib, oracle):
    # two calls in a row with different shapes, types and inputs: the second
    # reuses the scratch the first one left behind
    cases = [(synth.Q4_K, 4096, 1000, 1, 41), (synth.Q6_K, 4096, 777, 3, 42)]
    for t, k, n, m, seed in cases:
        w = synth.make_weights(t, n, k, seed=seed)
        x = synth.make_activations(m, k, seed + 100)
        bias = np.random.default_rng(seed).standard_normal(n).astype(np.float32)
        y_ref, y_na = _both(lib, x, w, t, k, n, bias)
        _, abs_terms = oracle.matmul(x, w, t, k, n, bias=bias, with_abs=True)
        G.assert_rows_close(y_na, y_ref, abs_terms, REL_TOL, f"noalloc {synth.NAMES[t]} m={m}")


# Every loader and unit code the entry point can reach, and the exact-fit
# limit: 8 rows x 32768 values fill the scratch array to its last byte.
EDGE_CASES = [
    (synth.Q4_K, MAX_IN_DIM, 300, MAX_ROWS),  # the limit case
    (synth.Q6_K, 8192, 257, 2),               # in_dim >= 8192
    (synth.Q6_K, 256, 45, 3),                 # 210-byte rows: the direct-load kernel
    (synth.Q8_0, 1024, 70, 5),                # 32-value block types
    (synth.Q5_0, 512, 33, 1),
]


@pytest.mark.parametrize("t,k,n,m", EDGE_CASES, ids=lambda c: str(c))
def test_noalloc_edge_cases_against_oracle(cuda, lib, oracle, t, k, n, m):
    w = synth.make_weights(t, n, k, seed=k + n)
    x = synth.make_activations(m, k, seed=m + n)
    bias = np.linspace(-1, 1, n, dtype=np.float32)
    y_o, abs_terms = oracle.matmul(x, w, t, k, n, bias=bias, with_abs=True)
    for call in range(2):  # twice: the second call starts from the first one's scratch contents
        y_ref, y_na = _both(lib, x, w, t, k, n, bias)
        G.assert_rows_close(y_na, y_o, abs_terms, REL_TOL, f"noalloc vs oracle {synth.NAMES[t]} call {call}")
        G.assert_rows_close(y_na, y_ref, abs_terms, 2 * REL_TOL, f"noalloc vs regular {synth.NAMES[t]}")


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda, lib):
    dummy = ctypes.c_void_p(256)
    rc = lib.cllm_cuda_matmul_quant_noalloc(dummy, dummy, synth.Q4_K, None, 4096, 16, MAX_ROWS + 1, dummy, None)
    assert rc == _lib.ERR_TOO_LARGE and "at most" in _lib.last_error()
    rc = lib.cllm_cuda_matmul_quant_noalloc(dummy, dummy, synth.Q4_K, None, MAX_IN_DIM + 256, 16, 1, dummy, None)
    assert rc == _lib.ERR_TOO_LARGE
