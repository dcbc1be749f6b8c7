"""The quant.hpp drop-in (C++20, libcllm_quant.so) driven by its C++ test
program, which mirrors the reference's tests/quant_test.cpp checks."""
import os
import subprocess

import pytest

from cllm_inference_b200 import build

pytestmark = pytest.mark.gpu


def test_quant_shim_program(cuda):
    build.build()
    exe = build.SHIM_TEST
    assert os.path.exists(exe), exe
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failed" in r.stdout
