"""Helpers for the GPU tests: device buffers from torch (plumbing only) and
calls through the C ABI of libcllm_cuda.so."""
import ctypes

import numpy as np
import torch

from cllm_inference_b200 import _lib


def dptr(t: torch.Tensor):
    return ctypes.c_void_p(t.data_ptr())


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def to_dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def dev_bytes(w: np.ndarray, misalign: int = 0) -> tuple[torch.Tensor, ctypes.c_void_p]:
    """Weight bytes on the device, optionally starting `misalign` bytes past a
    256-byte boundary (to exercise the unaligned loader)."""
    buf = torch.zeros(w.size + 256 + misalign, dtype=torch.uint8, device="cuda")
    base = buf.data_ptr()
    start = ((base + 255) // 256) * 256 + misalign - base
    buf[start:start + w.size] = torch.from_numpy(np.ascontiguousarray(w).view(np.uint8))
    return buf, ctypes.c_void_p(base + start)


def quantize(lib, x: np.ndarray):
    m, k = x.shape
    xd = to_dev(x.astype(np.float32))
    sc = torch.empty((m, k // 32), dtype=torch.float32, device="cuda")
    qs = torch.empty((m, k), dtype=torch.int8, device="cuda")
    bs = torch.empty((m, k // 32), dtype=torch.int32, device="cuda")
    _lib.check(lib.cllm_cuda_quantize_q8_0(dptr(xd), k, m, dptr(sc), dptr(qs), dptr(bs), stream()))
    torch.cuda.synchronize()
    return sc.cpu().numpy(), qs.cpu().numpy(), bs.cpu().numpy()


def matmul(lib, x: np.ndarray, w: np.ndarray, t: int, k: int, n: int, bias=None, misalign=0):
    m = x.shape[0]
    xd = to_dev(x.astype(np.float32))
    _, wp = dev_bytes(w, misalign)
    bd = to_dev(bias.astype(np.float32)) if bias is not None else None
    y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    _lib.check(lib.cllm_cuda_matmul_quant(dptr(xd), wp, t, dptr(bd) if bd is not None else None,
                                          k, n, m, dptr(y), 0, stream()))
    torch.cuda.synchronize()
    _lib.check(lib.cllm_cuda_check_device_status())
    return y.cpu().numpy()


def matmul_q8(lib, sc, qs, bsums, w, t, k, n, bias=None):
    m = qs.shape[0]
    scd, qsd, bsd = to_dev(sc), to_dev(qs), to_dev(bsums)
    _, wp = dev_bytes(w)
    bd = to_dev(bias.astype(np.float32)) if bias is not None else None
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    _lib.check(lib.cllm_cuda_matmul_q8(dptr(scd), dptr(qsd), dptr(bsd), wp, t,
                                       dptr(bd) if bd is not None else None, k, n, m, dptr(y), stream()))
    torch.cuda.synchronize()
    return y.cpu().numpy()


def partials(lib, qs: np.ndarray, w: np.ndarray, t: int, k: int, n: int, misalign=0):
    m = qs.shape[0]
    ppr = (2 if t == 14 else 1) * (k // 32)
    qd = to_dev(qs.astype(np.int8))
    _, wp = dev_bytes(w, misalign)
    out = torch.full((m, n, ppr), -7777777, dtype=torch.int32, device="cuda")
    _lib.check(lib.cllm_cuda_row_partials(dptr(qd), wp, t, k, n, m, dptr(out), stream()))
    torch.cuda.synchronize()
    return out.cpu().numpy()


def matmul_partials(lib, x: np.ndarray, w: np.ndarray, t: int, k: int, n: int):
    """Partials of the production kernels (cllm_cuda_matmul_partials): the
    launch plan of matmul_quant on fp32 x, int32 partials instead of y."""
    m = x.shape[0]
    ppr = (2 if t == 14 else 1) * (k // 32)
    xd = to_dev(x.astype(np.float32))
    _, wp = dev_bytes(w)
    out = torch.full((m, n, ppr), -7777777, dtype=torch.int32, device="cuda")
    _lib.check(lib.cllm_cuda_matmul_partials(dptr(xd), wp, t, k, n, m, dptr(out), stream()))
    torch.cuda.synchronize()
    _lib.check(lib.cllm_cuda_check_device_status())
    return out.cpu().numpy()


def sample_rows(n: int, limit: int, seed: int = 0) -> np.ndarray:
    """All rows when n <= limit, else the first and last 8 rows plus a seeded
    sample (sorted, distinct)."""
    if n <= limit:
        return np.arange(n)
    rng = np.random.default_rng(seed)
    mid = rng.choice(np.arange(8, n - 8), size=limit - 16, replace=False)
    return np.unique(np.concatenate([np.arange(8), mid, np.arange(n - 8, n)]))


def row_subset(w: np.ndarray, rb: int, rows: np.ndarray) -> np.ndarray:
    """The weight bytes of the given rows, back to back."""
    w2 = np.ascontiguousarray(w).view(np.uint8).reshape(-1, rb)
    return np.ascontiguousarray(w2[rows]).reshape(-1)


def assert_rows_close(y_gpu, y_ref, abs_terms, rel=1e-5, what=""):
    """The north-star row tolerance: |y_gpu - y_ref| <= rel * sum|partial*scale|.

    Non-finite reference values must be matched in kind (NaN vs +-inf)."""
    y_gpu = np.asarray(y_gpu, np.float64)
    y_ref = np.asarray(y_ref, np.float64)
    fin = np.isfinite(y_ref)
    assert np.array_equal(np.isnan(y_gpu), np.isnan(y_ref)), f"{what}: NaN pattern differs"
    inf = np.isinf(y_ref)
    assert np.array_equal(y_gpu[inf], y_ref[inf]), f"{what}: inf values differ"
    err = np.abs(y_gpu[fin] - y_ref[fin])
    tol = rel * abs_terms[fin] + 1e-30
    worst = np.max(err / tol) if err.size else 0.0
    assert np.all(err <= tol), f"{what}: worst err/tol = {worst:.3f}"
    return worst
