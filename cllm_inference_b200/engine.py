"""Python front end of the device-resident engine (include/cllm_cuda.h,
``cllm_cuda_engine_*``): the reference's TransformerEngine API
(include/cllm/core/engine.hpp:27-56 -- forward, prefill, reset_kv_cache,
seq_len, config) on a GGUF file, every activation in HBM.

There is no fallback: without the CUDA library the constructor fails.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


class Engine:
    """TransformerEngine(model, pool, WeightMode::Quant, ctx_limit) on the GPU."""

    def __init__(self, gguf_path: str, ctx_limit: int = 0, device: int = 0):
        self.lib = _lib.load()
        _lib.check(self.lib.cllm_cuda_init(device))
        h = ctypes.c_void_p()
        _lib.check(self.lib.cllm_cuda_engine_create(gguf_path.encode(), ctx_limit, ctypes.byref(h)))
        self.h = h
        v = (ctypes.c_int * 11)()
        _lib.check(self.lib.cllm_cuda_engine_config(h, v, 11))
        (self.n_layers, self.n_embd, self.n_head, self.n_head_kv, self.head_dim, self.n_ff, self.vocab,
         self.n_ctx, self.launches_per_step) = (int(x) for x in v[:9])
        self.fused = bool(v[10])

    def forward(self, token: int, logits: bool = True):
        """forward(token): (logits or None, greedy next token)."""
        out = np.empty(self.vocab, np.float32) if logits else None
        nxt = ctypes.c_int()
        _lib.check(self.lib.cllm_cuda_engine_forward(self.h, int(token), _ptr(out), ctypes.byref(nxt)))
        return out, nxt.value

    def prefill(self, tokens, logits: bool = True):
        ids = np.ascontiguousarray(tokens, np.int32)
        out = np.empty(self.vocab, np.float32) if logits else None
        nxt = ctypes.c_int()
        _lib.check(self.lib.cllm_cuda_engine_prefill(self.h, _ptr(ids), len(ids), _ptr(out), ctypes.byref(nxt)))
        return out, nxt.value

    def generate(self, prompt, steps: int):
        """Greedy decoding on the device: (tokens [steps], margins [steps])."""
        ids = np.ascontiguousarray(prompt, np.int32)
        toks = np.empty(steps, np.int32)
        margins = np.empty(steps, np.float32)
        _lib.check(self.lib.cllm_cuda_engine_generate(self.h, _ptr(ids), len(ids), steps, _ptr(toks),
                                                      _ptr(margins)))
        return toks, margins

    def reset(self) -> None:
        _lib.check(self.lib.cllm_cuda_engine_reset(self.h))

    def seq_len(self) -> int:
        return self.lib.cllm_cuda_engine_seq_len(self.h)

    def stream(self) -> int:
        s = ctypes.c_void_p()
        _lib.check(self.lib.cllm_cuda_engine_stream(self.h, ctypes.byref(s)))
        return s.value or 0

    def close(self) -> None:
        if self.h:
            self.lib.cllm_cuda_engine_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
