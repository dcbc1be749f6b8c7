"""CPU tests of the C ABI: the library loads, exports every symbol the header
declares, and answers the calls that need no device (type tables, argument
errors, which return before any CUDA call)."""
import ctypes

import pytest

from cllm_inference_b200 import _lib


def test_exports_every_header_symbol(lib):
    declared = _lib.header_symbols()
    assert len(declared) >= 13
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, missing
    assert set(declared) == set(_lib.SIGNATURES), "binding table out of sync with the header"


def test_type_tables(lib, oracle):
    for t in list(range(0, 16)) + [999, -1]:
        assert lib.cllm_cuda_block_size(t) == oracle.block_size(t)
        assert lib.cllm_cuda_type_size(t) == oracle.type_size(t)
        assert lib.cllm_cuda_has_vec_dot(t) == oracle.lib.orc_has_vec_dot(t)


def _err(lib, rc, code, text):
    assert rc == code
    assert text in _lib.last_error()


def test_argument_errors_before_device(lib):
    dummy = ctypes.c_void_p(16)
    _err(lib, lib.cllm_cuda_matmul_quant(dummy, dummy, 12, None, 100, 4, 1, dummy, 0, None),
         _lib.ERR_BLOCK_MULTIPLE, "matmul_quant: in_dim not divisible by block size")
    _err(lib, lib.cllm_cuda_matmul_quant(dummy, dummy, 12, None, 100, 4, 2, dummy, 0, None),
         _lib.ERR_BLOCK_MULTIPLE, "matmul_quant_batch: in_dim not divisible by block size")
    # the thirteen GGML types are accepted (the seven without an integer dot
    # kernel on the dequantize fallback); other ids fail as the reference's
    # fallback does, in dequantize_block (quant.cpp:387)
    _err(lib, lib.cllm_cuda_matmul_quant(dummy, dummy, 4, None, 64, 4, 1, dummy, 0, None),
         _lib.ERR_UNSUPPORTED_TYPE, "unsupported ggml type for dequantize")
    _err(lib, lib.cllm_cuda_matmul_q8(dummy, dummy, dummy, dummy, 3, None, 64, 4, 1, dummy, None),
         _lib.ERR_UNSUPPORTED_TYPE, "vec_dot_row: no kernel for this type")
    _err(lib, lib.cllm_cuda_quantize_q8_0(dummy, 33, 1, dummy, dummy, dummy, None),
         _lib.ERR_BLOCK_MULTIPLE, "quantize_row_q8_0: n not divisible by 32")
    _err(lib, lib.cllm_cuda_matmul_quant(dummy, dummy, 12, None, 256, 4, 1, dummy, 64, None),
         _lib.ERR_INVALID_ARG, "unknown flags")
    _err(lib, lib.cllm_cuda_matmul_quant(dummy, dummy, 12, None, -256, 4, 1, dummy, 0, None),
         _lib.ERR_INVALID_ARG, "negative")
    _err(lib, lib.cllm_cuda_dequantize(dummy, 5, 32, dummy, None),
         _lib.ERR_UNSUPPORTED_TYPE, "unsupported ggml type for dequantize")
    _err(lib, lib.cllm_cuda_dequantize_f16(dummy, 99, 32, dummy, None),
         _lib.ERR_UNSUPPORTED_TYPE, "unsupported ggml type for dequantize")
    _err(lib, lib.cllm_cuda_register_weights(None, 0, None), _lib.ERR_INVALID_ARG, "empty range")
    # n_rows <= 0 and out_dim == 0 are no-ops (quant.cpp:1436); nothing is touched
    assert lib.cllm_cuda_matmul_quant(None, None, 12, None, 256, 4, 0, None, 0, None) == 0
    assert lib.cllm_cuda_matmul_quant(None, None, 12, None, 256, 0, 1, None, 0, None) == 0


def test_lookup_unregistered(lib):
    out = ctypes.c_void_p()
    assert lib.cllm_cuda_lookup_weights(ctypes.c_void_p(0x1234), ctypes.byref(out)) == _lib.ERR_NOT_REGISTERED


def test_last_error_truncates(lib):
    lib.cllm_cuda_quantize_q8_0(None, 33, 1, None, None, None, None)
    buf = ctypes.create_string_buffer(8)
    n = lib.cllm_cuda_last_error(buf, 8)
    assert n > 8 and len(buf.value) == 7


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(ImportError):
        _lib._lib_saved = _lib._lib
        try:
            _lib._lib = None
            _lib.load(str(tmp_path / "nope.so"))
        finally:
            _lib._lib = _lib._lib_saved
