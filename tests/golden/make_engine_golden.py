"""Generate tests/golden/engine_greedy.json: greedy token sequences of the
reference's own TransformerEngine (oracle/_ref/libcllm_ref_engine.so, built
from the reference sources by oracle/Makefile) on the seeded synthetic GGUF
model cllm_inference_b200.gguf.SMALL.  The model file itself is not committed:
the GPU tests rewrite it from the same seed (the writer is deterministic).

Run from the repository root:  python tests/golden/make_engine_golden.py
"""
import json
import os
import sys
import tempfile

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

from cllm_inference_b200 import gguf  # noqa: E402
from oracle.oracle import ReferenceEngine  # noqa: E402

SEED = 1
STEPS = 128
PROMPTS = {
    # 16 tokens: prefill on the GEMV (fewer than 64 rows)
    "short": [int(v) for v in np.random.default_rng(11).integers(3, gguf.SMALL.vocab, 16)],
    # 80 tokens: prefill on the tcgen05 GEMM for the Q4_K matrices
    "long": [int(v) for v in np.random.default_rng(12).integers(3, gguf.SMALL.vocab, 80)],
}


def main():
    out = {"model": "cllm_inference_b200.gguf.SMALL", "seed": SEED, "steps": STEPS, "cases": {}}
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "small.gguf")
        gguf.write_llama(path, gguf.SMALL, seed=SEED)
        eng = ReferenceEngine(path)
        for name, prompt in PROMPTS.items():
            eng.reset()
            toks, margins, scales = eng.greedy(prompt, STEPS, with_scales=True)
            out["cases"][name] = {"prompt": prompt, "tokens": [int(t) for t in toks],
                                  "margins": [round(float(m), 5) for m in margins],
                                  "scales": [round(float(m), 4) for m in scales]}
            print(name, "min margin", float(np.min(margins)), "distinct tokens", len(set(toks.tolist())))
        eng.close()
    with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "engine_greedy.json"), "w") as f:
        json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
