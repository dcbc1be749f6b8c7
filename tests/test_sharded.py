"""Row sharding across GPUs, host side (CPU): the row partition of
cllm_cuda_shard_rows, the byte slices of a sharded weight, and the all-gather
that reassembles the output, run as two gloo ranks.  Each rank computes its
slice with the oracle (test infrastructure), so the assembled result must equal
the unsharded oracle matmul bit for bit: rows are independent and row sharding
never splits a block."""
import os
import socket

import numpy as np
import pytest

from cllm_inference_b200 import _lib, sharded, synth


def test_shard_rows_partition():
    for out in (0, 1, 7, 37, 1024, 4096, 14336, 28672, 128256, 1000003):
        for world in range(1, 9):
            spans = [sharded.shard_rows(out, world, r) for r in range(world)]
            pos = 0
            for b, r in spans:
                assert b == pos and r >= 0
                pos += r
            assert pos == out
            sizes = [r for _, r in spans]
            assert max(sizes) - min(sizes) <= 1
            assert sizes == sorted(sizes, reverse=True)  # the first out % world ranks get one more
    # the 70B shapes split evenly over 8 GPUs: one KV head (128 rows) per rank
    assert sharded.shard_rows(1024, 8, 3) == (384, 128)
    assert sharded.shard_rows(128256, 8, 7) == (7 * 16032, 16032)


def test_shard_rows_rejects_bad_groups():
    lib = _lib.load()
    import ctypes

    b, r = ctypes.c_int(), ctypes.c_int()
    for args in ((10, 0, 0), (10, 9, 0), (10, 2, 2), (10, 2, -1), (-1, 2, 0)):
        assert lib.cllm_cuda_shard_rows(*args, ctypes.byref(b), ctypes.byref(r)) == _lib.ERR_INVALID_ARG


def test_shard_weight_bytes_are_whole_rows():
    k, n = 512, 37
    w = synth.make_weights(synth.Q4_K, n, k, seed=3)
    rb = synth.row_bytes(synth.Q4_K, k)
    parts = [sharded.shard_weight_bytes(w, synth.Q4_K, k, n, 3, r) for r in range(3)]
    assert [p.size // rb for p in parts] == [13, 12, 12]
    assert np.array_equal(np.concatenate(parts), w)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_worker(rank, world, port, cases, result_q):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from oracle.oracle import Oracle

        orc = Oracle()
        out = []
        for (t, k, n, m, seed) in cases:
            w = synth.make_weights(t, n, k, seed=seed)
            x = synth.make_activations(m, k, seed + 1)
            part = sharded.shard_weight_bytes(w, t, k, n, world, rank)
            b, r = sharded.shard_rows(n, world, rank)
            local = orc.matmul(x, part, t, k, r) if r else np.zeros((m, 0), np.float32)
            full = sharded.gather_rows(torch.from_numpy(np.ascontiguousarray(local)), n)
            out.append(full.numpy())
        if rank == 0:
            result_q.put(out)
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_gather_rows_two_gloo_ranks(oracle):
    import torch.multiprocessing as mp

    cases = [(synth.Q4_K, 512, 37, 1, 11), (synth.Q6_K, 512, 64, 3, 12), (synth.Q8_0, 256, 5, 2, 13),
             (synth.Q4_0, 64, 1, 1, 14)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, cases, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for (t, k, n, m, seed), y in zip(cases, got):
        w = synth.make_weights(t, n, k, seed=seed)
        x = synth.make_activations(m, k, seed + 1)
        assert np.array_equal(y, oracle.matmul(x, w, t, k, n))


class _FakeIpcLib:
    """Stands in for the C ABI's cllm_cuda_ipc_alloc / _open on a CPU-only
    host: rank r's buffer is address 0x10000 * (r + 1), its handle 64 bytes of
    r + 1; opening a handle returns 0x7000_0000 + that address."""

    def __init__(self, rank):
        self.rank = rank
        self.opened = []

    def cllm_cuda_ipc_alloc(self, nbytes, ptr_ref, handle):
        ptr_ref._obj.value = 0x10000 * (self.rank + 1)
        for i in range(len(handle)):
            handle[i] = self.rank + 1
        return 0

    def cllm_cuda_ipc_open(self, handle, ptr_ref):
        owner = handle[0] - 1
        assert all(b == owner + 1 for b in handle) and owner != self.rank
        ptr_ref._obj.value = 0x70000000 + 0x10000 * (owner + 1)
        self.opened.append(owner)
        return 0


def _ipc_worker(rank, world, port, result_q):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        lib = _FakeIpcLib(rank)
        own, ptrs, opened = sharded.open_peer_buffers(lib, 4096, rank, world, sharded._torch_allgather(None))
        result_q.put((rank, own, ptrs, opened, lib.opened))
    finally:
        dist.destroy_process_group()


def test_peer_buffer_exchange_two_gloo_ranks():
    """The handle exchange of RowShardGroup (open_peer_buffers) over gloo:
    each rank's own slot is its own allocation, every other slot the mapping
    of that rank's published handle, and a process never opens its own."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ipc_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = sorted(q.get(timeout=240) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, own, ptrs, opened, opened_owners in got:
        assert own == 0x10000 * (rank + 1)
        assert ptrs[rank] == own
        other = 1 - rank
        assert ptrs[other] == 0x70000000 + 0x10000 * (other + 1)
        assert opened == [ptrs[other]] and opened_owners == [other]
