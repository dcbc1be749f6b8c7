"""CPU tests of the synthetic GGUF writer (cllm_inference_b200.gguf): the
header round-trips, and the reference's own GGUF loader and engine
(oracle/_ref/libcllm_ref_engine.so) read the file it writes."""
import os

import numpy as np
import pytest

from cllm_inference_b200 import gguf, synth

TINY = gguf.LlamaShape(n_layers=2, n_embd=256, n_head=2, n_head_kv=1, n_ff=512, vocab=300, n_ctx=64)


def test_header_roundtrip(tmp_path):
    path = str(tmp_path / "tiny.gguf")
    size = gguf.write_llama(path, TINY, seed=3)
    assert os.path.getsize(path) == size
    meta, infos, data_start = gguf.read_header(path)
    assert meta["general.architecture"] == "llama"
    assert meta["llama.block_count"] == 2 and meta["llama.embedding_length"] == 256
    assert meta["llama.attention.head_count_kv"] == 1 and meta["llama.vocab_size"] == 300
    assert abs(meta["llama.rope.freq_base"] - 500000.0) < 1e-3
    assert data_start % gguf.ALIGN == 0
    plan = gguf.tensor_plan(TINY)
    assert [i[0] for i in infos] == [p[0] for p in plan]
    raw = open(path, "rb").read()
    for (name, t, dims, off), (_, pt, rows, cols) in zip(infos, plan):
        assert t == pt and off % gguf.ALIGN == 0
        assert dims == ([cols] if rows == 1 else [cols, rows])
        want = gguf.tensor_data(name, t, rows, cols, 3).tobytes()
        assert raw[data_start + off:data_start + off + len(want)] == want, name


def test_centred_kquant_blocks():
    """The engine models' Q4_K blocks average about zero per sub-block."""
    from oracle.oracle import Oracle

    w = synth.make_weights(synth.Q4_K, 64, 256, seed=4, centered=True)
    deq = Oracle().dequantize(w, synth.Q4_K, 64 * 256).reshape(64, 8, 32)
    assert np.abs(deq.mean(axis=(0, 2))).max() < 0.5 * deq.std()


def test_reference_engine_loads_the_file(tmp_path):
    from oracle.oracle import ReferenceEngine, reference_engine_available

    if not reference_engine_available():
        pytest.skip("oracle/_ref/libcllm_ref_engine.so (the reference build) is not present")
    path = str(tmp_path / "tiny.gguf")
    gguf.write_llama(path, TINY, seed=3)
    eng = ReferenceEngine(path, n_threads=2)
    assert (eng.n_layers, eng.n_embd, eng.n_head, eng.n_head_kv, eng.head_dim, eng.n_ff, eng.vocab, eng.n_ctx) == \
        (2, 256, 2, 1, 128, 512, 300, 64)
    toks, margins = eng.greedy([1, 2, 3, 4], 8)
    assert toks.shape == (8,) and np.all((toks >= 0) & (toks < 300)) and np.all(margins >= 0)
    eng.close()
