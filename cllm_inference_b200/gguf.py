"""Synthetic GGUF model files in the format the reference loader reads.

The reference loads models with ``GgufLoader::load`` (cllm_inference
src/core/gguf.cpp:120-275): magic ``GGUF``, version 2 or 3, tensor and
metadata counts (u64), metadata key/value pairs, one info record per tensor
(name, dims innermost first, GGML type id, data offset), then the data
section at the next 32-byte boundary, which it maps read-only and points every
tensor into (gguf.cpp:171-189).  The model hyper-parameters come from the
``<arch>.*`` keys (gguf.cpp:218-245).

There are no model files in this build, so the engine tests and the decode
benchmark write Llama-architecture files with seeded synthetic weights:

* linear weights in GGML blocks (``synth.make_weights``) with centred Q4_K
  mins and block scales that give each matrix a value spread of about
  1/sqrt(in_dim), as trained weights have, in a Q4_K_M-style mix: attn_q/k/v/output, ffn_gate/up and token_embd Q4_K,
  ffn_down and output Q6_K (the shapes of BASELINE configs 2 and 4);
* norm weights F32 ~ N(1, 0.1).

Tensor data starts at 32-byte-aligned offsets, so every row of the K-quant
types above starts 16-byte aligned in the file and in its device copy.
"""
from __future__ import annotations

import dataclasses
import struct

import numpy as np

from . import synth

F32, F16 = 0, 1
ALIGN = 32

# GGUF metadata value types (gguf.cpp:16-19)
_U32, _I32, _F32, _BOOL, _STR, _ARR = 4, 5, 6, 7, 8, 9


@dataclasses.dataclass(frozen=True)
class LlamaShape:
    """ModelConfig fields of a Llama-architecture model (gguf.hpp:13-33)."""
    n_layers: int
    n_embd: int
    n_head: int
    n_head_kv: int
    n_ff: int
    vocab: int
    n_ctx: int = 4096
    rope_theta: float = 500000.0
    norm_eps: float = 1e-5

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_head


# BASELINE config 4 (Llama-3-8B shapes) and config 5 (Llama-3-70B shapes)
LLAMA3_8B = LlamaShape(32, 4096, 32, 8, 14336, 128256, 4096)
LLAMA3_70B = LlamaShape(80, 8192, 64, 8, 28672, 128256, 4096)
# A reduced model for the engine tests: the 8B proportions at a size the
# reference CPU engine runs in seconds (n_ff a multiple of 2048, so the Q6_K
# down-projection rows are 16-byte multiples and the fused decode step applies).
SMALL = LlamaShape(4, 2048, 16, 4, 6144, 32000, 1024)


def tensor_plan(cfg: LlamaShape, down_type: int = synth.Q6_K):
    """(name, type, rows, cols) of every tensor, in file order."""
    q_dim = cfg.n_head * cfg.head_dim
    kv_dim = cfg.n_head_kv * cfg.head_dim
    out = [("token_embd.weight", synth.Q4_K, cfg.vocab, cfg.n_embd)]
    for layer in range(cfg.n_layers):
        p = f"blk.{layer}."
        out += [(p + "attn_norm.weight", F32, 1, cfg.n_embd),
                (p + "attn_q.weight", synth.Q4_K, q_dim, cfg.n_embd),
                (p + "attn_k.weight", synth.Q4_K, kv_dim, cfg.n_embd),
                (p + "attn_v.weight", synth.Q4_K, kv_dim, cfg.n_embd),
                (p + "attn_output.weight", synth.Q4_K, cfg.n_embd, q_dim),
                (p + "ffn_norm.weight", F32, 1, cfg.n_embd),
                (p + "ffn_gate.weight", synth.Q4_K, cfg.n_ff, cfg.n_embd),
                (p + "ffn_up.weight", synth.Q4_K, cfg.n_ff, cfg.n_embd),
                (p + "ffn_down.weight", down_type, cfg.n_embd, cfg.n_ff)]
    out += [("output_norm.weight", F32, 1, cfg.n_embd), ("output.weight", synth.Q6_K, cfg.vocab, cfg.n_embd)]
    return out


def tensor_bytes(t: int, rows: int, cols: int) -> int:
    if t == F32:
        return 4 * rows * cols
    if t == F16:
        return 2 * rows * cols
    return rows * synth.row_bytes(t, cols)


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _kv(key: str, vtype: int, value) -> bytes:
    out = _str(key) + struct.pack("<I", vtype)
    if vtype == _U32:
        return out + struct.pack("<I", value)
    if vtype == _F32:
        return out + struct.pack("<f", value)
    if vtype == _BOOL:
        return out + struct.pack("<B", 1 if value else 0)
    if vtype == _STR:
        return out + _str(value)
    raise ValueError(vtype)


def header_bytes(cfg: LlamaShape, plan) -> tuple[bytes, list[int], int]:
    """(header incl. padding to the data section, data offsets, data size)."""
    kvs = [("general.architecture", _STR, "llama"),
           ("general.name", _STR, "synthetic"),
           ("llama.block_count", _U32, cfg.n_layers),
           ("llama.context_length", _U32, cfg.n_ctx),
           ("llama.embedding_length", _U32, cfg.n_embd),
           ("llama.feed_forward_length", _U32, cfg.n_ff),
           ("llama.attention.head_count", _U32, cfg.n_head),
           ("llama.attention.head_count_kv", _U32, cfg.n_head_kv),
           ("llama.rope.freq_base", _F32, cfg.rope_theta),
           ("llama.attention.layer_norm_rms_epsilon", _F32, cfg.norm_eps),
           ("llama.vocab_size", _U32, cfg.vocab),
           ("tokenizer.ggml.model", _STR, "llama"),
           ("tokenizer.ggml.bos_token_id", _U32, 1),
           ("tokenizer.ggml.eos_token_id", _U32, 2),
           ("tokenizer.ggml.add_bos_token", _BOOL, True)]
    head = b"GGUF" + struct.pack("<IQQ", 3, len(plan), len(kvs))
    head += b"".join(_kv(*kv) for kv in kvs)
    offsets, off = [], 0
    for (name, t, rows, cols) in plan:
        dims = [cols] if rows == 1 else [cols, rows]  # innermost first
        head += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", t, off)
        offsets.append(off)
        off += tensor_bytes(t, rows, cols)
        off = (off + ALIGN - 1) // ALIGN * ALIGN
    pad = (-len(head)) % ALIGN
    return head + b"\0" * pad, offsets, off


def weight_scale_range(t: int, cols: int):
    """Block-scale range that gives a linear weight of `cols` inputs a value
    spread of about 1/sqrt(cols), as in trained models, so activations stay
    O(1) through the layers (the GEMV benchmarks' BASELINE scales are about
    70x larger, which makes a stack of layers numerically chaotic: the
    rounding differences of two correct implementations would decide the
    greedy tokens).  Q4_K (centred): value ~ d * sc * (q - 7.5), spread about
    145 d; Q6_K with |sc| <= 8: spread about 85 d."""
    target = 1.0 / np.sqrt(cols)
    mid = target / (145.0 if t == synth.Q4_K else 85.0)
    return (0.5 * mid, 1.5 * mid)


def tensor_data(name: str, t: int, rows: int, cols: int, seed: int) -> np.ndarray:
    """Seeded bytes of one tensor (a tensor's seed depends only on its name)."""
    s = (seed * 1000003 + sum((i + 1) * ord(c) for i, c in enumerate(name))) % (2 ** 63)
    if t == F32:
        v = 1.0 + 0.1 * np.random.default_rng(s).standard_normal(rows * cols, dtype=np.float32)
        return v.astype(np.float32).view(np.uint8)
    return synth.make_weights(t, rows, cols, seed=s, centered=True, d_range=weight_scale_range(t, cols),
                              q6_scale_max=8)


def write_llama(path: str, cfg: LlamaShape, seed: int = 0, down_type: int = synth.Q6_K) -> int:
    """Write a synthetic Llama GGUF file; returns its size in bytes."""
    plan = tensor_plan(cfg, down_type)
    head, offsets, data_size = header_bytes(cfg, plan)
    with open(path, "wb") as f:
        f.write(head)
        pos = 0
        for (name, t, rows, cols), off in zip(plan, offsets):
            if off > pos:
                f.write(b"\0" * (off - pos))
                pos = off
            data = tensor_data(name, t, rows, cols, seed)
            f.write(data.tobytes())
            pos += data.size
        if data_size > pos:
            f.write(b"\0" * (data_size - pos))
    return len(head) + data_size


def read_header(path: str):
    """Parse a GGUF header (the subset this module writes): returns
    (metadata dict, [(name, type, dims innermost-first, offset)], data start)."""
    with open(path, "rb") as f:
        buf = f.read(1 << 20)
    if buf[:4] != b"GGUF":
        raise ValueError("invalid GGUF magic")
    ver, nt, nkv = struct.unpack_from("<IQQ", buf, 4)
    p = 24

    def rd_str(p):
        (n,) = struct.unpack_from("<Q", buf, p)
        return buf[p + 8:p + 8 + n].decode(), p + 8 + n

    meta = {}
    for _ in range(nkv):
        k, p = rd_str(p)
        (vt,) = struct.unpack_from("<I", buf, p)
        p += 4
        if vt in (_U32, _I32, _F32):
            meta[k] = struct.unpack_from({_U32: "<I", _I32: "<i", _F32: "<f"}[vt], buf, p)[0]
            p += 4
        elif vt == _BOOL:
            meta[k] = bool(buf[p])
            p += 1
        elif vt == _STR:
            meta[k], p = rd_str(p)
        else:
            raise ValueError(f"value type {vt} not written by this module")
    infos = []
    for _ in range(nt):
        name, p = rd_str(p)
        (nd,) = struct.unpack_from("<I", buf, p)
        dims = list(struct.unpack_from(f"<{nd}Q", buf, p + 4))
        p += 4 + 8 * nd
        t, off = struct.unpack_from("<IQ", buf, p)
        p += 12
        infos.append((name, t, dims, off))
    return meta, infos, (p + ALIGN - 1) // ALIGN * ALIGN
