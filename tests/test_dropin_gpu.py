"""The C++ drop-in (cllm_inference_b200/csrc/shim: the reference's quant.hpp
API on the GPU library) under the reference's own code, built unmodified by
oracle/Makefile against the shim headers and linked to libcllm_quant.so:

* the reference's tests/quant_test.cpp (known answers for all thirteen
  types, F32/F16 included, the differential matmul tests, bias, batch ==
  single) must report no failure;
* the reference's TransformerEngine and GGUF loader (engine.cpp, gguf.cpp)
  must construct on the shim -- it dequantizes the F32 norm weights at
  construction (engine.cpp:201-225) -- and follow the reference built on its
  own quant.cpp, teacher-forced, within the Q8_0 re-quantization noise band.
"""
import ctypes
import json
import os
import subprocess

import numpy as np
import pytest

from cllm_inference_b200 import gguf

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.path.join(ROOT, "oracle", "_ref")
QUANT_TEST = os.path.join(REF_DIR, "quant_test_on_shim")
ENGINE_ON_SHIM = os.path.join(REF_DIR, "libcllm_ref_engine_on_shim.so")


def test_reference_quant_test_passes_on_the_shim(cuda):
    if not os.path.exists(QUANT_TEST):
        pytest.skip("oracle/_ref/quant_test_on_shim was not built (needs the reference tree at build time)")
    r = subprocess.run([QUANT_TEST], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert "FAIL" not in r.stdout


def test_reference_engine_on_the_shim_matches_reference(cuda, tmp_path):
    """The reference engine constructs and runs on the shim; its logits follow the
    reference-on-quant.cpp logits within the Q8_0 re-quantization noise band
    (5 % of the logit scale, see tests/test_engine_gpu.py), teacher-forced on the
    reference's greedy tokens, and its greedy choice agrees on every step whose
    margin exceeds that band."""
    from oracle.oracle import ReferenceEngine, reference_engine_available

    if not (os.path.exists(ENGINE_ON_SHIM) and reference_engine_available()):
        pytest.skip("the reference engine builds in oracle/_ref are not present")
    g = json.load(open(os.path.join(ROOT, "tests", "golden", "engine_greedy.json")))
    path = str(tmp_path / "small.gguf")
    gguf.write_llama(path, gguf.SMALL, seed=g["seed"])
    c = g["cases"]["short"]
    on_shim = ReferenceEngine(path, so=ENGINE_ON_SHIM)
    ref = ReferenceEngine(path)
    ls, lr = on_shim.prefill(c["prompt"]), ref.prefill(c["prompt"])
    decisive = agree = 0
    for tok in c["tokens"][:12]:
        scale = float(np.max(np.abs(lr)))
        assert float(np.max(np.abs(ls - lr))) <= 0.05 * scale
        top = np.sort(lr)[-2:]
        if top[1] - top[0] > 0.05 * scale:
            decisive += 1
            agree += int(np.argmax(ls) == np.argmax(lr))
        ls, lr = on_shim.forward(tok), ref.forward(tok)
    on_shim.close()
    ref.close()
    assert decisive > 0 and agree == decisive
