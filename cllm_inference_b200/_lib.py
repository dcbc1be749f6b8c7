"""ctypes binding of lib/libcllm_cuda.so (C ABI: include/cllm_cuda.h).

There is no fallback: if the library is missing or a symbol is absent,
loading fails loudly.  Build it with ``python -m cllm_inference_b200.build``
or ``__graft_entry__.build()``.
"""
from __future__ import annotations

import ctypes
import os
import re

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
LIB_PATH = os.path.join(PKG, "lib", "libcllm_cuda.so")
HEADER = os.path.join(ROOT, "include", "cllm_cuda.h")

OK = 0
ERR_INVALID_ARG = -1
ERR_UNSUPPORTED_TYPE = -2
ERR_BLOCK_MULTIPLE = -3
ERR_CUDA = -4
ERR_NOT_REGISTERED = -5
ERR_NO_DEVICE = -6
ERR_KERNEL_TIMEOUT = -7
ERR_TOO_LARGE = -8

X_HOST, Y_HOST, W_HOST = 1, 2, 4
SHARD_WAIT_PREV = 1
SHARD_NO_SIGNAL = 2
SHARD_PAD_WORDS = 16
IPC_HANDLE_BYTES = 64
HOST_IO = X_HOST | Y_HOST

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_U = ctypes.c_uint
_SZ = ctypes.c_size_t

# name -> (restype, argtypes); must cover every entry point of the header.
SIGNATURES = {
    "cllm_cuda_init": (_I, [_I]),
    "cllm_cuda_block_size": (_I, [_I]),
    "cllm_cuda_type_size": (_I64, [_I]),
    "cllm_cuda_has_vec_dot": (_I, [_I]),
    "cllm_cuda_register_weights": (_I, [_P, _SZ, ctypes.POINTER(_P)]),
    "cllm_cuda_unregister_weights": (_I, [_P]),
    "cllm_cuda_lookup_weights": (_I, [_P, ctypes.POINTER(_P)]),
    "cllm_cuda_quantize_q8_0": (_I, [_P, _I64, _I, _P, _P, _P, _P]),
    "cllm_cuda_matmul_quant": (_I, [_P, _P, _I, _P, _I, _I, _I, _P, _U, _P]),
    "cllm_cuda_matmul_q8": (_I, [_P, _P, _P, _P, _I, _P, _I, _I, _I, _P, _P]),
    "cllm_cuda_row_partials": (_I, [_P, _P, _I, _I, _I, _I, _P, _P]),
    "cllm_cuda_matmul_partials": (_I, [_P, _P, _I, _I, _I, _I, _P, _P]),
    "cllm_cuda_dequantize": (_I, [_P, _I, _I64, _P, _P]),
    "cllm_cuda_dequantize_f16": (_I, [_P, _I, _I64, _P, _P]),
    "cllm_cuda_matmul_plan": (_I, [_P, _I, _I, _I, _I, ctypes.POINTER(_I), _I]),
    "cllm_cuda_matmul_quant_noalloc": (_I, [_P, _P, _I, _P, _I, _I, _I, _P, _P]),
    "cllm_cuda_shard_rows": (_I, [_I, _I, _I, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]),
    "cllm_cuda_matmul_quant_rowshard": (_I, [_P, _P, _I, _P, _I, _I, _I, _I, _I, ctypes.POINTER(_P),
                                             ctypes.POINTER(_P), _P, _U, _P]),
    "cllm_cuda_shard_wait": (_I, [_P, _P, _I, _P]),
    "cllm_cuda_shard_barrier": (_I, [ctypes.POINTER(_P), _P, _I, _I, _P]),
    "cllm_cuda_ipc_alloc": (_I, [ctypes.c_size_t, ctypes.POINTER(_P), _P]),
    "cllm_cuda_ipc_open": (_I, [_P, ctypes.POINTER(_P)]),
    "cllm_cuda_ipc_close": (_I, [_P]),
    "cllm_cuda_ipc_free": (_I, [_P]),
    "cllm_cuda_engine_create": (_I, [ctypes.c_char_p, _I, ctypes.POINTER(_P)]),
    "cllm_cuda_engine_destroy": (_I, [_P]),
    "cllm_cuda_engine_config": (_I, [_P, ctypes.POINTER(ctypes.c_int), _I]),
    "cllm_cuda_engine_forward": (_I, [_P, _I, _P, ctypes.POINTER(ctypes.c_int)]),
    "cllm_cuda_engine_prefill": (_I, [_P, _P, _I, _P, ctypes.POINTER(ctypes.c_int)]),
    "cllm_cuda_engine_generate": (_I, [_P, _P, _I, _I, _P, _P]),
    "cllm_cuda_engine_reset": (_I, [_P]),
    "cllm_cuda_engine_seq_len": (_I, [_P]),
    "cllm_cuda_engine_stream": (_I, [_P, ctypes.POINTER(_P)]),
    "cllm_cuda_rms_norm": (_I, [_P, _P, _I, _I, ctypes.c_float, _P, _P]),
    "cllm_cuda_silu_mul": (_I, [_P, _P, _I64, _P]),
    "cllm_cuda_rope_table": (_I, [ctypes.c_float, _I, _I, _P]),
    "cllm_cuda_rope_kv": (_I, [_P, _P, _P, _I, _I, _I, _I, _P, _I, _P, _P, _P]),
    "cllm_cuda_attention": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _P, _P]),
    "cllm_cuda_check_device_status": (_I, []),
    "cllm_cuda_last_error": (_I, [ctypes.c_char_p, _SZ]),
}


def header_symbols(path: str = HEADER) -> list[str]:
    """Every function the C header declares (used by the export test)."""
    text = open(path).read()
    return sorted(set(re.findall(r"^\s*(?:int|int64_t|void)\s+(cllm_cuda_\w+)\s*\(", text, re.M)))


class CudaError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


_lib = None


def load(path: str = LIB_PATH):
    """Load libcllm_cuda.so once and bind every signature."""
    global _lib
    if _lib is None:
        if not os.path.exists(path):
            raise ImportError(f"{path} is missing: build it with cllm_inference_b200.build.build()")
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def last_error() -> str:
    lib = load()
    buf = ctypes.create_string_buffer(1024)
    lib.cllm_cuda_last_error(buf, len(buf))
    return buf.value.decode()


def check(rc: int) -> None:
    if rc != OK:
        raise CudaError(rc, last_error())
