"""Seeded synthetic GGML weight blocks and activations.

There are no model files in this build; every weight matrix is generated from
a seed with the value distributions below.  The byte layouts are GGML's
(cllm_inference include/cllm/core/quant.hpp:13-27, src/core/quant.cpp:340-369):

=====  =====  ==========================================================
type   bytes  fields and synthetic distribution
=====  =====  ==========================================================
Q4_K   144    d f16 ~U(1e-3,2e-2), dmin f16 ~U(0,1e-2), 12 packed 6-bit
              scale/min bytes ~U{0..255} (each unpacks to U{0..63}),
              128 B of nibbles ~U{0..15}
Q5_K   176    as Q4_K plus 32 B of high bits ~U
Q6_K   210    128 B low nibbles, 64 B high pairs ~U; 16 int8 scales
              ~U{-32..31}; d f16 ~U(1e-3,2e-2) at offset 208
Q8_0   34     d f16 ~U(1e-3,2e-2), 32 int8 ~U
Q4_0   18     d f16 ~U(1e-3,2e-2), 16 B nibbles ~U
Q5_0   22     d f16 ~U(1e-3,2e-2), 4 B high bits, 16 B nibbles ~U
=====  =====  ==========================================================

Activations are fp32 ~N(0, 1).  ``make_weights`` (numpy) feeds the CPU checks;
``make_weights_torch`` builds the same distributions directly in device memory
for the benchmark, where only throughput is measured.
"""
from __future__ import annotations

import numpy as np

Q4_0, Q5_0, Q8_0, Q4_K, Q5_K, Q6_K = 2, 6, 8, 12, 13, 14
F32, F16, Q4_1, Q5_1, Q8_1, Q2_K, Q3_K = 0, 1, 3, 7, 9, 10, 11
BLOCK = {Q4_0: 32, Q5_0: 32, Q8_0: 32, Q4_K: 256, Q5_K: 256, Q6_K: 256,
         F32: 1, F16: 1, Q4_1: 32, Q5_1: 32, Q8_1: 32, Q2_K: 256, Q3_K: 256}
TSIZE = {Q4_0: 18, Q5_0: 22, Q8_0: 34, Q4_K: 144, Q5_K: 176, Q6_K: 210,
         F32: 4, F16: 2, Q4_1: 20, Q5_1: 24, Q8_1: 36, Q2_K: 84, Q3_K: 110}
NAMES = {Q4_0: "Q4_0", Q5_0: "Q5_0", Q8_0: "Q8_0", Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K",
         F32: "F32", F16: "F16", Q4_1: "Q4_1", Q5_1: "Q5_1", Q8_1: "Q8_1", Q2_K: "Q2_K", Q3_K: "Q3_K"}
# fp16 fields of the fallback types: (byte offset, low, high) of a uniform draw
_F16_FIELDS = {Q4_1: [(0, 1e-3, 2e-2), (2, -0.1, 0.1)], Q5_1: [(0, 1e-3, 2e-2), (2, -0.1, 0.1)],
               Q8_1: [(0, 1e-3, 2e-2), (2, -1.0, 1.0)], Q2_K: [(80, 1e-3, 2e-2), (82, 0.0, 1e-2)],
               Q3_K: [(108, 1e-3, 2e-2)]}
BY_NAME = {v: k for k, v in NAMES.items()}


def row_bytes(t: int, k: int) -> int:
    return (k // BLOCK[t]) * TSIZE[t]


def _f16_bytes(vals: np.ndarray) -> np.ndarray:
    return vals.astype(np.float16).view(np.uint8).reshape(-1, 2)


def pack_scale_min_k4(sc: np.ndarray, m: np.ndarray) -> np.ndarray:
    """The 12 packed bytes of 8 six-bit (scale, min) pairs per super-block, as
    get_scale_min_k4 (quant.cpp:72-80) unpacks them: sc, m [nblk, 8] in 0..63."""
    sc = sc.astype(np.uint8)
    m = m.astype(np.uint8)
    out = np.empty((sc.shape[0], 12), np.uint8)
    out[:, 0:4] = (sc[:, 0:4] & 63) | ((sc[:, 4:8] >> 4) << 6)
    out[:, 4:8] = (m[:, 0:4] & 63) | ((m[:, 4:8] >> 4) << 6)
    out[:, 8:12] = (sc[:, 4:8] & 0xF) | ((m[:, 4:8] & 0xF) << 4)
    return out


def make_weights(t: int, n_rows: int, k: int, seed: int, centered: bool = False, d_range=(1e-3, 2e-2),
                 q6_scale_max: int = 32) -> np.ndarray:
    """[n_rows * row_bytes] uint8 of seeded synthetic blocks of type t.

    centered=True (Q4_K/Q5_K only) draws every sub-block's min so that its
    values average about zero, as trained weights do: dmin = 8 d and
    m = round(sc * mean(q) / 8), mean(q) = 7.5 (Q4_K) or 15.5 (Q5_K, with
    dmin = 16 d).  The engine's synthetic models use it; the GEMV benchmarks
    keep the uniform scale/min bytes of the BASELINE distributions.
    d_range: the uniform range of the block scale d (BASELINE: 1e-3..2e-2);
    q6_scale_max: Q6_K sub-block scales are drawn from [-q6_scale_max, q6_scale_max)."""
    if k % BLOCK[t]:
        raise ValueError("k must be a multiple of the block size")
    rng = np.random.default_rng(seed)
    nblk = n_rows * (k // BLOCK[t])
    if t == F32:
        return rng.standard_normal(nblk, dtype=np.float32).view(np.uint8)
    if t == F16:
        return rng.standard_normal(nblk).astype(np.float16).view(np.uint8)
    ts = TSIZE[t]
    w = rng.integers(0, 256, size=(nblk, ts), dtype=np.uint8)
    if nblk == 0:
        return w.reshape(-1)
    if t in _F16_FIELDS:
        for off, lo, hi in _F16_FIELDS[t]:
            w[:, off:off + 2] = _f16_bytes(rng.uniform(lo, hi, size=nblk))
        return w.reshape(-1)
    d = rng.uniform(d_range[0], d_range[1], size=nblk)
    if t == Q6_K:
        w[:, 192:208] = rng.integers(-q6_scale_max, q6_scale_max, size=(nblk, 16), dtype=np.int8).view(np.uint8)
        w[:, 208:210] = _f16_bytes(d)
    else:
        w[:, 0:2] = _f16_bytes(d)
        if t in (Q4_K, Q5_K):
            if centered:
                mean_q, ratio = (7.5, 8.0) if t == Q4_K else (15.5, 16.0)
                sc = rng.integers(0, 64, size=(nblk, 8))
                m = np.rint(sc * mean_q / ratio)
                w[:, 2:4] = _f16_bytes(d.astype(np.float16).astype(np.float64) * ratio)
                w[:, 4:16] = pack_scale_min_k4(sc, m)
            else:
                w[:, 2:4] = _f16_bytes(rng.uniform(0.0, 1e-2, size=nblk))
    return w.reshape(-1)


def make_activations(m: int, k: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).standard_normal((m, k), dtype=np.float32)


def make_weights_torch(t: int, n_rows: int, k: int, seed: int, device="cuda"):
    """Same distributions as make_weights, generated in device memory (torch uint8 [bytes])."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    nblk = n_rows * (k // BLOCK[t])
    ts = TSIZE[t]
    w = torch.randint(0, 256, (nblk, ts), dtype=torch.uint8, device=device, generator=g)
    d = (torch.rand(nblk, device=device, generator=g) * (2e-2 - 1e-3) + 1e-3).half()
    d = d.view(torch.uint8).view(nblk, 2)
    if t == Q6_K:
        w[:, 192:208] = torch.randint(-32, 32, (nblk, 16), dtype=torch.int8, device=device,
                                      generator=g).view(torch.uint8)
        w[:, 208:210] = d
    else:
        w[:, 0:2] = d
        if t in (Q4_K, Q5_K):
            dm = (torch.rand(nblk, device=device, generator=g) * 1e-2).half()
            w[:, 2:4] = dm.view(torch.uint8).view(nblk, 2)
    return w.view(-1)
