"""TEST INFRASTRUCTURE ONLY — Python front end of the CPU oracle.

Only tests/, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` leg of
``bench.py`` may import this module, and only as the checker.  The product
library never imports it.

Two CPU implementations of the quantized-matmul hot path are exposed:

* ``Oracle`` — the plain-C restatement in ``oracle/quant_oracle.c``
  (``oracle/_build/liboracle.so``).  It returns the exact int32 per-block
  partial dot products as well as the float row sums.
* ``Reference`` — the reference's own ``src/core/quant.cpp`` and
  ``src/core/thread_pool.cpp`` compiled unmodified by ``oracle/Makefile``
  into ``oracle/_ref/libcllm_ref.so`` (wrapper: ``oracle/ref_capi.cpp``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libcllm_ref.so")

Q4_0, Q5_0, Q8_0, Q4_K, Q5_K, Q6_K = 2, 6, 8, 12, 13, 14
F32, F16, Q4_1, Q5_1, Q8_1, Q2_K, Q3_K = 0, 1, 3, 7, 9, 10, 11
HOT_TYPES = (Q4_0, Q5_0, Q8_0, Q4_K, Q5_K, Q6_K)
OTHER_TYPES = (F32, F16, Q4_1, Q5_1, Q8_1, Q2_K, Q3_K)  # dequantize + float-dot fallback (quant.cpp:1404-1430)
ALL_TYPES = OTHER_TYPES + HOT_TYPES
TYPE_NAMES = {Q4_0: "Q4_0", Q5_0: "Q5_0", Q8_0: "Q8_0", Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K", F32: "F32",
              F16: "F16", Q4_1: "Q4_1", Q5_1: "Q5_1", Q8_1: "Q8_1", Q2_K: "Q2_K", Q3_K: "Q3_K"}

_P = ctypes.c_void_p
_I64 = ctypes.c_int64


def build() -> None:
    """Compile the oracle (and, where the reference tree exists, oracle/_ref)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(_P)


class Oracle:
    """ctypes binding of oracle/quant_oracle.c."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build()
        lib = ctypes.CDLL(path)
        lib.orc_block_size.argtypes = [ctypes.c_int]
        lib.orc_type_size.argtypes = [ctypes.c_int]
        lib.orc_type_size.restype = _I64
        lib.orc_has_vec_dot.argtypes = [ctypes.c_int]
        lib.orc_half_to_float.argtypes = [ctypes.c_uint16]
        lib.orc_half_to_float.restype = ctypes.c_float
        lib.orc_float_to_half.argtypes = [ctypes.c_float]
        lib.orc_float_to_half.restype = ctypes.c_uint16
        lib.orc_quantize_row_q8_0.argtypes = [_P, _I64, _P, _P, _P]
        lib.orc_partials_per_row.argtypes = [ctypes.c_int, _I64]
        lib.orc_partials_per_row.restype = _I64
        lib.orc_row_partials.argtypes = [_P, ctypes.c_int, _P, _I64, _P]
        lib.orc_vec_dot_row.argtypes = [_P, ctypes.c_int, _P, _P, _P, _I64, _P]
        lib.orc_matmul_quant_batch.argtypes = [_P, _P, ctypes.c_int, _P, ctypes.c_int, ctypes.c_int,
                                               ctypes.c_int, _P, _P, _P, _P, _P]
        lib.orc_dequantize.argtypes = [_P, ctypes.c_int, _I64, _P]
        lib.orc_matmul_fallback.argtypes = [_P, _P, ctypes.c_int, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                            _P, _P]
        self.lib = lib

    def block_size(self, t: int) -> int:
        return self.lib.orc_block_size(t)

    def type_size(self, t: int) -> int:
        return self.lib.orc_type_size(t)

    def row_bytes(self, t: int, k: int) -> int:
        return (k // self.block_size(t)) * self.type_size(t)

    def quantize(self, x: np.ndarray):
        """quantize_row_q8_0 of each row of x [M, K] -> (scales [M,K/32] f32, qs [M,K] i8, bsums i32)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        x2 = x.reshape(-1, x.shape[-1])
        m, k = x2.shape
        if k % 32:
            raise RuntimeError("quantize_row_q8_0: n not divisible by 32")
        sc = np.empty((m, k // 32), np.float32)
        qs = np.empty((m, k), np.int8)
        bs = np.empty((m, k // 32), np.int32)
        for r in range(m):
            self.lib.orc_quantize_row_q8_0(_ptr(x2[r]), k, _ptr(sc[r]), _ptr(qs[r]), _ptr(bs[r]))
        return sc, qs, bs

    def partials(self, w: np.ndarray, t: int, k: int, n: int, qs: np.ndarray) -> np.ndarray:
        """Exact int32 partials [M, N, parts_per_row] of W [N rows] against qs [M, K]."""
        rb = self.row_bytes(t, k)
        w = np.ascontiguousarray(w, dtype=np.uint8).reshape(-1)
        qs = np.ascontiguousarray(qs, dtype=np.int8).reshape(-1, k)
        npr = self.lib.orc_partials_per_row(t, k)
        out = np.empty((qs.shape[0], n, npr), np.int32)
        base = w.ctypes.data
        for r in range(qs.shape[0]):
            for j in range(n):
                rc = self.lib.orc_row_partials(ctypes.c_void_p(base + j * rb), t, _ptr(qs[r]), k,
                                               out[r, j].ctypes.data_as(_P))
                if rc:
                    raise RuntimeError("orc_row_partials failed")
        return out

    def matmul(self, x: np.ndarray, w: np.ndarray, t: int, k: int, n: int,
               bias: np.ndarray | None = None, with_abs: bool = False):
        """matmul_quant_batch: y [M, N] = x [M, K] . W^T (+bias), AVX2 float order.

        with_abs=True also returns, per output, the double sum of |term| over
        the per-block float terms (plus |bias|): the tolerance denominator."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        m = x.shape[0] if x.ndim == 2 else (x.size // k if k else 1)
        x = x.reshape(m, k)
        w = np.ascontiguousarray(w, dtype=np.uint8)
        y = np.empty((m, n), np.float32)
        sc = np.empty(max(m * (k // 32), 1), np.float32)
        qs = np.empty(max(m * k, 1), np.int8)
        bs = np.empty(max(m * (k // 32), 1), np.int32)
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        a = np.empty((m, n), np.float64) if with_abs else None
        rc = self.lib.orc_matmul_quant_batch(_ptr(x), _ptr(w), t, _ptr(b), k, n, m, _ptr(y),
                                             _ptr(sc), _ptr(qs), _ptr(bs), _ptr(a))
        if rc == -1:
            raise RuntimeError("matmul_quant: in_dim not divisible by block size")
        if rc:
            raise RuntimeError(f"oracle matmul failed ({rc})")
        return (y, a) if with_abs else y

    def matmul_fallback(self, x: np.ndarray, w: np.ndarray, t: int, k: int, n: int,
                        bias: np.ndarray | None = None, with_abs: bool = False):
        """matmul_quant(_batch) for a type without an integer dot kernel (the
        reference's dequantize-then-float-dot path): y [M, N] (and the |term| sums)."""
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, k)
        m = x.shape[0]
        y = np.empty((m, n), np.float32)
        a = np.empty((m, n), np.float64)
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        rc = self.lib.orc_matmul_fallback(_ptr(x), _ptr(np.ascontiguousarray(w, np.uint8)), t, _ptr(b), k, n, m,
                                          _ptr(y), _ptr(a))
        if rc:
            raise RuntimeError(f"oracle fallback matmul failed ({rc})")
        return (y, a) if with_abs else y

    def dequantize(self, w: np.ndarray, t: int, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        w = np.ascontiguousarray(w, dtype=np.uint8)
        if self.lib.orc_dequantize(_ptr(w), t, n, _ptr(out)):
            raise RuntimeError("unsupported ggml type for dequantize")
        return out

    def half_to_float(self, h: int) -> float:
        return self.lib.orc_half_to_float(h)

    def float_to_half(self, f: float) -> int:
        return self.lib.orc_float_to_half(f)


class Reference:
    """ctypes binding of the reference's own quant.cpp (oracle/_ref/libcllm_ref.so)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        lib = ctypes.CDLL(path)
        lib.ref_last_error.restype = ctypes.c_char_p
        lib.ref_block_size.argtypes = [ctypes.c_int]
        lib.ref_type_size.argtypes = [ctypes.c_int]
        lib.ref_type_size.restype = _I64
        lib.ref_pool_create.argtypes = [ctypes.c_int]
        lib.ref_pool_create.restype = _P
        lib.ref_pool_destroy.argtypes = [_P]
        lib.ref_pool_size.argtypes = [_P]
        lib.ref_pool_size.restype = _I64
        lib.ref_dequantize_block.argtypes = [_P, _P, ctypes.c_int, _I64]
        lib.ref_quantize_row_q8_0.argtypes = [_P, _I64, _P, _P, _P]
        lib.ref_vec_dot_row.argtypes = [_P, ctypes.c_int, _P, _P, _P, _I64, _P]
        lib.ref_matmul_quant.argtypes = [_P, _P, ctypes.c_int, _P, ctypes.c_int, ctypes.c_int, _P, _P]
        lib.ref_matmul_quant_batch.argtypes = [_P, _P, ctypes.c_int, _P, ctypes.c_int, ctypes.c_int,
                                               ctypes.c_int, _P, _P]
        self.lib = lib
        self._pool = None

    def _check(self, rc: int) -> None:
        if rc:
            raise RuntimeError(self.lib.ref_last_error().decode())

    def pool(self, n_threads: int):
        """A reference ThreadPool of n_threads workers (kept for reuse)."""
        if self._pool is None or self._pool[0] != n_threads:
            if self._pool is not None:
                self.lib.ref_pool_destroy(self._pool[1])
            self._pool = (n_threads, self.lib.ref_pool_create(n_threads))
        return self._pool[1]

    def pool_size(self, n_threads: int) -> int:
        return self.lib.ref_pool_size(self.pool(n_threads))

    def quantize(self, x: np.ndarray):
        x = np.ascontiguousarray(x, dtype=np.float32)
        x2 = x.reshape(-1, x.shape[-1])
        m, k = x2.shape
        sc = np.empty((m, max(k // 32, 0)), np.float32)
        qs = np.empty((m, k), np.int8)
        bs = np.empty((m, max(k // 32, 0)), np.int32)
        for r in range(m):
            self._check(self.lib.ref_quantize_row_q8_0(_ptr(x2[r]), k, _ptr(sc[r]), _ptr(qs[r]),
                                                       _ptr(bs[r])))
        return sc, qs, bs

    def matmul(self, x, w, t, k, n, bias=None, n_threads: int = 0, m: int | None = None):
        """matmul_quant_batch (n_threads=0: no pool, the reference's serial path)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        if m is None:
            m = x.size // k if k else 1
        y = np.empty((m, n), np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        pool = self.pool(n_threads) if n_threads > 0 else None
        w = np.ascontiguousarray(w, dtype=np.uint8)
        self._check(self.lib.ref_matmul_quant_batch(_ptr(x), _ptr(w), t, _ptr(b), k, n, m, _ptr(y),
                                                    pool))
        return y

    def matmul_ptr(self, x_ptr: int, w_ptr: int, t: int, k: int, n: int, m: int, y_ptr: int,
                   n_threads: int) -> None:
        """Same as matmul() on raw host addresses (used by the timed CPU baseline)."""
        pool = self.pool(n_threads) if n_threads > 0 else None
        self._check(self.lib.ref_matmul_quant_batch(_P(x_ptr), _P(w_ptr), t, None, k, n, m,
                                                    _P(y_ptr), pool))

    def dequantize(self, w, t, n):
        out = np.empty(n, np.float32)
        w = np.ascontiguousarray(w, dtype=np.uint8)
        self._check(self.lib.ref_dequantize_block(_ptr(w), _ptr(out), t, n))
        return out


def reference_available() -> bool:
    return os.path.exists(REF_SO)


REF_ENGINE_SO = os.path.join(HERE, "_ref", "libcllm_ref_engine.so")


def reference_engine_available() -> bool:
    return os.path.exists(REF_ENGINE_SO)


class ReferenceEngine:
    """The reference's own TransformerEngine (engine.cpp, gguf.cpp, quant.cpp),
    built unmodified into oracle/_ref/libcllm_ref_engine.so (wrapper:
    oracle/ref_engine_capi.cpp), on a GGUF file."""

    def __init__(self, path: str, n_threads: int = 0, ctx_limit: int = 0, so: str = REF_ENGINE_SO):
        if not os.path.exists(so):
            raise FileNotFoundError(so)
        lib = ctypes.CDLL(so)
        lib.ref_engine_last_error.restype = ctypes.c_char_p
        lib.ref_engine_create.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.POINTER(_P)]
        lib.ref_engine_destroy.argtypes = [_P]
        lib.ref_engine_config.argtypes = [_P, _P]
        lib.ref_engine_prefill.argtypes = [_P, _P, ctypes.c_int, _P, _P]
        lib.ref_engine_forward.argtypes = [_P, ctypes.c_int, _P, _P]
        lib.ref_engine_greedy.argtypes = [_P, _P, ctypes.c_int, ctypes.c_int, _P, _P, _P]
        lib.ref_engine_reset.argtypes = [_P]
        lib.ref_engine_seq_len.argtypes = [_P]
        self.lib = lib
        h = _P()
        n_threads = n_threads or (os.cpu_count() or 1)
        self._check(lib.ref_engine_create(path.encode(), n_threads, ctx_limit, ctypes.byref(h)))
        self.h = h
        cfg = np.zeros(8, np.int32)
        lib.ref_engine_config(h, _ptr(cfg))
        (self.n_layers, self.n_embd, self.n_head, self.n_head_kv, self.head_dim, self.n_ff, self.vocab,
         self.n_ctx) = (int(v) for v in cfg)

    def _check(self, rc: int) -> None:
        if rc:
            raise RuntimeError(self.lib.ref_engine_last_error().decode())

    def prefill(self, tokens) -> np.ndarray:
        ids = np.ascontiguousarray(tokens, np.int32)
        logits = np.empty(self.vocab, np.float32)
        tok = ctypes.c_int()
        self._check(self.lib.ref_engine_prefill(self.h, _ptr(ids), len(ids), _ptr(logits), ctypes.byref(tok)))
        return logits

    def forward(self, token: int) -> np.ndarray:
        logits = np.empty(self.vocab, np.float32)
        nxt = ctypes.c_int()
        self._check(self.lib.ref_engine_forward(self.h, int(token), _ptr(logits), ctypes.byref(nxt)))
        return logits

    def greedy(self, prompt, steps: int, with_scales: bool = False):
        """(tokens, top-1 minus top-2 margins[, largest |logit|]) of greedy decoding after prefill(prompt)."""
        ids = np.ascontiguousarray(prompt, np.int32)
        toks = np.empty(steps, np.int32)
        margins = np.empty(steps, np.float32)
        scales = np.empty(steps, np.float32)
        self._check(self.lib.ref_engine_greedy(self.h, _ptr(ids), len(ids), steps, _ptr(toks), _ptr(margins),
                                               _ptr(scales)))
        return (toks, margins, scales) if with_scales else (toks, margins)

    def reset(self) -> None:
        self._check(self.lib.ref_engine_reset(self.h))

    def seq_len(self) -> int:
        return self.lib.ref_engine_seq_len(self.h)

    def close(self) -> None:
        if self.h:
            self.lib.ref_engine_destroy(self.h)
            self.h = None


REF_OPS_SO = os.path.join(HERE, "_ref", "libcllm_ref_ops.so")


class ReferenceOps:
    """The reference engine's internal operators (engine.cpp compiled whole into
    oracle/ref_engine_ops.cpp -> oracle/_ref/libcllm_ref_ops.so)."""

    def __init__(self, so: str = REF_OPS_SO):
        if not os.path.exists(so):
            raise FileNotFoundError(so)
        lib = ctypes.CDLL(so)
        lib.ref_op_rms_norm.argtypes = [_P, _P, ctypes.c_int, ctypes.c_float, _P]
        lib.ref_op_silu.argtypes = [_P, _I64, _P]
        lib.ref_op_rope.argtypes = [_P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float]
        lib.ref_op_attention.argtypes = [_P, _P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P]
        self.lib = lib

    def rms_norm(self, x, w, eps):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        self.lib.ref_op_rms_norm(_ptr(x), _ptr(np.ascontiguousarray(w, np.float32)), x.size, eps, _ptr(out))
        return out

    def silu(self, x):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        self.lib.ref_op_silu(_ptr(x), x.size, _ptr(out))
        return out

    def rope(self, q, n_head, head_dim, pos, theta):
        q = np.array(q, np.float32, copy=True)
        self.lib.ref_op_rope(_ptr(q), n_head, head_dim, pos, theta)
        return q

    def attention(self, q, kc, vc, seq, n_head, n_kv, head_dim):
        out = np.empty(n_head * head_dim, np.float32)
        self.lib.ref_op_attention(_ptr(np.ascontiguousarray(q, np.float32)), _ptr(np.ascontiguousarray(kc, np.float32)),
                                  _ptr(np.ascontiguousarray(vc, np.float32)), seq, n_head, n_kv, head_dim, _ptr(out))
        return out


def reference_ops_available() -> bool:
    return os.path.exists(REF_OPS_SO)
