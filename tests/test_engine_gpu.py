"""The device-resident engine step (cllm_cuda_engine_*) against the
reference's own TransformerEngine on the same synthetic GGUF model.

Bars:
  * greedy decoding produces the reference's tokens for 128 steps (the
    committed sequences in tests/golden/engine_greedy.json, made by the
    reference build; live against oracle/_ref when it is present), after a
    16-token prefill (GEMV path) and an 80-token prefill (tcgen05 GEMM path);
  * logits agree with the reference's within 2e-3 of the logit scale
    (max |logit|): the matmul rows, norms and softmax sums are reduced in a
    different order than the reference's loops;
  * prefix reuse, context limits and errors follow engine.cpp:520-545, :340-344.
"""
import json
import os

import numpy as np
import pytest

from cllm_inference_b200 import gguf

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "engine_greedy.json")
LOGIT_TOL = 2e-3


@pytest.fixture(scope="module")
def small_model(tmp_path_factory):
    g = json.load(open(GOLDEN))
    path = str(tmp_path_factory.mktemp("model") / "small.gguf")
    gguf.write_llama(path, gguf.SMALL, seed=g["seed"])
    return path, g


@pytest.fixture(scope="module")
def engine(cuda, small_model):
    from cllm_inference_b200.engine import Engine

    e = Engine(small_model[0])
    yield e
    e.close()


def _reference(path):
    from oracle.oracle import ReferenceEngine, reference_engine_available

    return ReferenceEngine(path) if reference_engine_available() else None


def test_config(engine):
    s = gguf.SMALL
    assert (engine.n_layers, engine.n_embd, engine.n_head, engine.n_head_kv, engine.head_dim, engine.n_ff,
            engine.vocab, engine.n_ctx) == (s.n_layers, s.n_embd, s.n_head, s.n_head_kv, s.head_dim, s.n_ff,
                                            s.vocab, s.n_ctx)
    assert engine.launches_per_step > 10 * s.n_layers  # the captured decode step


@pytest.mark.parametrize("case", ["short", "long"])
def test_greedy_128_steps_match_reference(engine, small_model, case):
    path, g = small_model
    c = g["cases"][case]
    engine.reset()
    toks, margins = engine.generate(c["prompt"], g["steps"])
    want = np.array(c["tokens"])
    first_diff = int(np.argmax(toks != want)) if np.any(toks != want) else -1
    assert first_diff == -1, (f"{case}: first differing step {first_diff}: gpu {toks[first_diff]} vs reference "
                              f"{want[first_diff]} (reference margin {c['margins'][first_diff]})")
    np.testing.assert_allclose(margins, np.array(c["margins"]), rtol=0.05, atol=0.05)
    assert engine.seq_len() == len(c["prompt"]) + g["steps"] - 1


def test_greedy_live_reference(engine, small_model):
    """The same comparison against the reference build run here and now."""
    path, g = small_model
    ref = _reference(path)
    if ref is None:
        pytest.skip("oracle/_ref/libcllm_ref_engine.so is not present")
    prompt = [5, 17, 300, 4000, 123]
    rt, _ = ref.greedy(prompt, 64)
    engine.reset()
    gt, _ = engine.generate(prompt, 64)
    assert np.array_equal(gt, rt)
    ref.close()


def test_logits_close_to_reference(engine, small_model):
    path, g = small_model
    ref = _reference(path)
    if ref is None:
        pytest.skip("oracle/_ref/libcllm_ref_engine.so is not present")
    prompt = g["cases"]["long"]["prompt"]
    engine.reset()
    ref.reset()
    lg, nxt = engine.prefill(prompt)
    lr = ref.prefill(prompt)
    scale = float(np.max(np.abs(lr)))
    assert np.max(np.abs(lg - lr)) <= LOGIT_TOL * scale
    assert nxt == int(np.argmax(lr))
    tok = nxt
    for _ in range(6):
        lg, nxt = engine.forward(tok)
        lr = ref.forward(tok)
        assert np.max(np.abs(lg - lr)) <= LOGIT_TOL * float(np.max(np.abs(lr)))
        tok = int(np.argmax(lr))
        assert nxt == tok
    ref.close()


def test_prefix_reuse_and_truncation(engine, small_model):
    """prefill(a) then prefill(a + b) computes only b (engine.cpp:530-545) and
    equals a fresh prefill(a + b); prefill(a) again re-runs only its last token."""
    a = [7, 8, 9, 10, 11, 12, 13, 14]
    b = [20, 21, 22, 23]
    engine.reset()
    engine.prefill(a)
    l_reuse, t_reuse = engine.prefill(a + b)
    assert engine.seq_len() == len(a) + len(b)
    engine.reset()
    l_fresh, t_fresh = engine.prefill(a + b)
    assert t_reuse == t_fresh
    assert np.max(np.abs(l_reuse - l_fresh)) <= LOGIT_TOL * float(np.max(np.abs(l_fresh)))
    l_again, _ = engine.prefill(a + b)  # the whole prompt is cached: only its last token re-runs
    assert engine.seq_len() == len(a) + len(b)
    assert np.max(np.abs(l_again - l_fresh)) <= LOGIT_TOL * float(np.max(np.abs(l_fresh)))


def test_context_limit_and_errors(cuda, small_model):
    from cllm_inference_b200 import _lib
    from cllm_inference_b200.engine import Engine

    e = Engine(small_model[0], ctx_limit=8)
    assert e.n_ctx == 8
    e.prefill([1, 2, 3, 4, 5, 6, 7])
    e.forward(9)
    with pytest.raises(_lib.CudaError, match="context length exceeded"):
        e.forward(9)
    with pytest.raises(_lib.CudaError, match="empty tokens"):
        e.prefill([])
    with pytest.raises(_lib.CudaError, match="out of range"):
        e.forward(gguf.SMALL.vocab)
    e.close()
    with pytest.raises(_lib.CudaError, match="cannot open model file"):
        Engine("/nonexistent/model.gguf")
