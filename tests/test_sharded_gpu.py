"""Row-sharded matmul_quant on the GPU: the peer-store GEMV
(cllm_cuda_matmul_quant_rowshard) and the completion barrier
(cllm_cuda_shard_barrier).

On one GPU the ranks are emulated: every "rank's" y buffer is local memory,
the rank calls run one after another, and a barrier is only run when its
peers' signals are already in place (or never come: the bounded wait then
expires and reports a status, with no GPU fault).  Barriers that wait on each
other are never launched on one GPU.  The 2-GPU test runs real ranks, one
process per GPU, when the box has two GPUs."""
import ctypes
import os
import socket

import numpy as np
import pytest
import torch

from cllm_inference_b200 import _lib, sharded, synth
from gpu_helpers import dptr, stream, to_dev

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = _lib.load()
    _lib.check(lib.cllm_cuda_init(0))
    return lib


def _ptrs(ts):
    return (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])


def _full(lib, xd, wd, t, k, n, m, bias=None):
    y = torch.full((m, n), float("nan"), device="cuda")
    _lib.check(lib.cllm_cuda_matmul_quant(dptr(xd), dptr(wd), t, dptr(bias) if bias is not None else None,
                                          k, n, m, dptr(y), 0, stream()))
    return y


CASES = [(synth.Q4_K, 4096, 1024, 1), (synth.Q4_K, 4096, 1000, 3), (synth.Q6_K, 4096, 515, 1),
         (synth.Q8_0, 1024, 96, 2), (synth.Q5_K, 2048, 77, 4),
         # in_dim >= 8192: activations quantized once per call (activation image)
         (synth.Q6_K, 8192, 130, 1), (synth.Q4_K, 8192, 200, 2)]


@pytest.mark.parametrize("world", [1, 2, 3, 8])
@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{synth.NAMES[c[0]]}-{c[1]}x{c[2]}-m{c[3]}")
def test_rowshard_emulated_ranks(lib, case, world):
    t, k, n, m = case
    w = synth.make_weights(t, n, k, seed=k + n)
    x = to_dev(synth.make_activations(m, k, 5))
    bias = to_dev(np.linspace(-1, 1, n).astype(np.float32))
    ref = _full(lib, x, to_dev(w), t, k, n, m, bias)
    ys = [torch.full((m, n), float("nan"), device="cuda") for _ in range(world)]
    for rank in range(world):
        part = to_dev(np.ascontiguousarray(sharded.shard_weight_bytes(w, t, k, n, world, rank)))
        _lib.check(lib.cllm_cuda_matmul_quant_rowshard(dptr(x), dptr(part), t, dptr(bias), k, n, rank, world, m,
                                                       _ptrs(ys), None, None, 0, stream()))
    torch.cuda.synchronize()
    _lib.check(lib.cllm_cuda_check_device_status())
    for y in ys:  # every rank's buffer holds every slice, bit-identical to one GPU
        assert torch.equal(y, ref)


def test_barrier_single_rank_advances_epoch(lib):
    pad = torch.zeros(64, dtype=torch.int32, device="cuda")
    epoch = torch.zeros(1, dtype=torch.int32, device="cuda")
    for _ in range(3):
        _lib.check(lib.cllm_cuda_shard_barrier(_ptrs([pad]), dptr(epoch), 1, 0, stream()))
    torch.cuda.synchronize()
    _lib.check(lib.cllm_cuda_check_device_status())
    assert int(epoch.item()) == 3 and int(pad[0].item()) == 3


def test_barrier_with_peer_already_signalled(lib):
    pads = [torch.zeros(64, dtype=torch.int32, device="cuda") for _ in range(2)]
    epoch = torch.zeros(1, dtype=torch.int32, device="cuda")
    pads[0][1] = 1  # rank 1 reached epoch 1 before rank 0 arrives
    _lib.check(lib.cllm_cuda_shard_barrier(_ptrs(pads), dptr(epoch), 2, 0, stream()))
    torch.cuda.synchronize()
    _lib.check(lib.cllm_cuda_check_device_status())
    assert int(epoch.item()) == 1
    assert int(pads[1][0].item()) == 1  # rank 0 announced itself to rank 1
    assert int(pads[0][0].item()) == 1


def test_barrier_missing_rank_times_out_without_fault(lib):
    """A rank that never arrives: the wait expires after its bound (about 1 s),
    the kernel returns, the status word reports it, and the context stays
    usable."""
    pads = [torch.zeros(64, dtype=torch.int32, device="cuda") for _ in range(2)]
    epoch = torch.zeros(1, dtype=torch.int32, device="cuda")
    _lib.check(lib.cllm_cuda_shard_barrier(_ptrs(pads), dptr(epoch), 2, 0, stream()))
    torch.cuda.synchronize()
    assert lib.cllm_cuda_check_device_status() == _lib.ERR_KERNEL_TIMEOUT
    assert lib.cllm_cuda_check_device_status() == _lib.OK  # the status was cleared
    # the device still works
    t, k, n = synth.Q4_K, 512, 64
    w = to_dev(synth.make_weights(t, n, k, seed=1))
    x = to_dev(synth.make_activations(1, k, 2))
    y = _full(lib, x, w, t, k, n, 1)
    torch.cuda.synchronize()
    assert torch.isfinite(y).all()


def test_rowshard_rejects_bad_groups(lib):
    y = torch.zeros(8, device="cuda")
    x = torch.zeros(256, device="cuda")
    w = torch.zeros(144, dtype=torch.uint8, device="cuda")
    for rank, world in ((0, 0), (0, 9), (2, 2)):
        assert lib.cllm_cuda_matmul_quant_rowshard(dptr(x), dptr(w), synth.Q4_K, None, 256, 1, rank, world, 1,
                                                   _ptrs([y] * max(world, 1)), None, None, 0,
                                                   stream()) == _lib.ERR_INVALID_ARG
    assert lib.cllm_cuda_matmul_quant_rowshard(dptr(x), dptr(w), synth.Q4_K, None, 256, 1, 0, 1, 9,
                                               _ptrs([y]), None, None, 0, stream()) == _lib.ERR_TOO_LARGE
    # waiting on the previous round needs the signal pads
    assert lib.cllm_cuda_matmul_quant_rowshard(dptr(x), dptr(w), synth.Q4_K, None, 256, 1, 0, 1, 1,
                                               _ptrs([y]), None, None, _lib.SHARD_WAIT_PREV,
                                               stream()) == _lib.ERR_INVALID_ARG


def _pads(world):
    return [torch.zeros(_lib.SHARD_PAD_WORDS, dtype=torch.int32, device="cuda") for _ in range(world)]


@pytest.mark.parametrize("k", [4096, 8192])
@pytest.mark.parametrize("world", [2, 3])
def test_rowshard_signals_every_rank(lib, world, k):
    """Each emulated rank's call announces its round into every pad and
    resets its arrival count; once all ranks have run, each rank's wait
    passes, and the next round (CLLM_SHARD_WAIT_PREV) sees the previous one
    complete.  Ranks run one after another: nothing waits on a later launch."""
    t, n, m = synth.Q4_K, 300, 1
    w = synth.make_weights(t, n, k, seed=9)
    x = to_dev(synth.make_activations(m, k, 3))
    ref = _full(lib, x, to_dev(w), t, k, n, m)
    pads = _pads(world)
    epochs = [torch.zeros(1, dtype=torch.int32, device="cuda") for _ in range(world)]
    parts = [to_dev(np.ascontiguousarray(sharded.shard_weight_bytes(w, t, k, n, world, r))) for r in range(world)]
    for rnd in range(1, 3):
        ys = [torch.full((m, n), float("nan"), device="cuda") for _ in range(world)]
        for r in range(world):
            _lib.check(lib.cllm_cuda_matmul_quant_rowshard(dptr(x), dptr(parts[r]), t, None, k, n, r, world, m,
                                                           _ptrs(ys), _ptrs(pads), dptr(epochs[r]),
                                                           _lib.SHARD_WAIT_PREV, stream()))
        for r in range(world):
            _lib.check(lib.cllm_cuda_shard_wait(dptr(pads[r]), dptr(epochs[r]), world, stream()))
        torch.cuda.synchronize()
        _lib.check(lib.cllm_cuda_check_device_status())
        for r in range(world):
            assert int(epochs[r].item()) == rnd
            assert pads[r][:world].tolist() == [rnd] * world
            assert int(pads[r][_lib.SHARD_PAD_WORDS // 2].item()) == 0  # arrival count reset
            assert torch.equal(ys[r], ref)


def test_rowshard_no_signal_calls_leave_the_round(lib):
    """CLLM_SHARD_NO_SIGNAL: a call that nobody waits on (k after q, up after
    gate) neither advances the epoch nor touches the pads; the following
    signalling call announces the round for both, and a later
    CLLM_SHARD_WAIT_PREV sees both complete.  Emulated ranks run one after
    another: every wait depends only on earlier launches."""
    t, k, n, m, world = synth.Q4_K, 4096, 300, 1, 2
    ws = [synth.make_weights(t, n, k, seed=11 + i) for i in range(2)]
    x = to_dev(synth.make_activations(m, k, 5))
    refs = [_full(lib, x, to_dev(w), t, k, n, m) for w in ws]
    parts = [[to_dev(np.ascontiguousarray(sharded.shard_weight_bytes(w, t, k, n, world, r))) for r in range(world)]
             for w in ws]
    pads = _pads(world)
    epochs = [torch.zeros(1, dtype=torch.int32, device="cuda") for _ in range(world)]
    for rnd in range(1, 3):
        ys = [[torch.full((m, n), float("nan"), device="cuda") for _ in range(world)] for _ in range(2)]
        for r in range(world):
            first = (_lib.SHARD_WAIT_PREV if rnd > 1 else 0) | _lib.SHARD_NO_SIGNAL
            _lib.check(lib.cllm_cuda_matmul_quant_rowshard(dptr(x), dptr(parts[0][r]), t, None, k, n, r, world, m,
                                                           _ptrs(ys[0]), _ptrs(pads), dptr(epochs[r]), first,
                                                           stream()))
            torch.cuda.synchronize()
            assert int(epochs[r].item()) == rnd - 1  # the no-signal call left the round alone
            _lib.check(lib.cllm_cuda_matmul_quant_rowshard(dptr(x), dptr(parts[1][r]), t, None, k, n, r, world, m,
                                                           _ptrs(ys[1]), _ptrs(pads), dptr(epochs[r]), 0, stream()))
        for r in range(world):
            _lib.check(lib.cllm_cuda_shard_wait(dptr(pads[r]), dptr(epochs[r]), world, stream()))
        torch.cuda.synchronize()
        _lib.check(lib.cllm_cuda_check_device_status())
        for r in range(world):
            assert int(epochs[r].item()) == rnd
            assert pads[r][:world].tolist() == [rnd] * world
            assert torch.equal(ys[0][r], refs[0]) and torch.equal(ys[1][r], refs[1])


def test_rowshard_empty_slice_still_signals(lib):
    """More ranks than rows: rank 2 of 3 owns no row of a 2-row matrix, yet its
    call announces the round, so the others' waits do not run out."""
    t, k, n, world = synth.Q8_0, 256, 2, 3
    w = synth.make_weights(t, n, k, seed=4)
    x = to_dev(synth.make_activations(1, k, 6))
    pads, ys = _pads(world), [torch.zeros((1, n), device="cuda") for _ in range(world)]
    epochs = [torch.zeros(1, dtype=torch.int32, device="cuda") for _ in range(world)]
    for r in range(world):
        part = to_dev(np.ascontiguousarray(sharded.shard_weight_bytes(w, t, k, n, world, r)))
        _lib.check(lib.cllm_cuda_matmul_quant_rowshard(dptr(x), dptr(part) if part.numel() else dptr(x), t, None,
                                                       k, n, r, world, 1, _ptrs(ys), _ptrs(pads),
                                                       dptr(epochs[r]), 0, stream()))
    _lib.check(lib.cllm_cuda_shard_wait(dptr(pads[0]), dptr(epochs[0]), world, stream()))
    torch.cuda.synchronize()
    _lib.check(lib.cllm_cuda_check_device_status())
    assert pads[0][:world].tolist() == [1, 1, 1]
    assert torch.equal(ys[0], _full(lib, x, to_dev(w), t, k, n, 1))


@pytest.mark.parametrize("k", [4096, 8192])
def test_rowshard_wait_for_missing_rank_times_out(lib, k):
    """CLLM_SHARD_WAIT_PREV while a peer never finished the previous round:
    the in-kernel wait gives up after its bound, the status reports it, and
    the call still completes (no fault, no hang)."""
    t, n, world = synth.Q4_K, 64, 2
    w = synth.make_weights(t, n, k, seed=8)
    x = to_dev(synth.make_activations(1, k, 1))
    pads, ys = _pads(world), [torch.zeros((1, n), device="cuda") for _ in range(world)]
    epoch = torch.zeros(1, dtype=torch.int32, device="cuda")
    part = to_dev(np.ascontiguousarray(sharded.shard_weight_bytes(w, t, k, n, world, 0)))
    for _ in range(2):  # round 1 completes locally; round 2 waits for rank 1's round 1, which never comes
        _lib.check(lib.cllm_cuda_matmul_quant_rowshard(dptr(x), dptr(part), t, None, k, n, 0, world, 1, _ptrs(ys),
                                                       _ptrs(pads), dptr(epoch), _lib.SHARD_WAIT_PREV, stream()))
    torch.cuda.synchronize()
    assert lib.cllm_cuda_check_device_status() == _lib.ERR_KERNEL_TIMEOUT
    assert int(epoch.item()) == 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_gpu_worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ok = True
    try:
        from oracle.oracle import Oracle

        orc = Oracle()
        lib = _lib.load()
        grp = sharded.RowShardGroup(max_out=16384, max_rows=8)
        for (t, k, n, m) in CASES:
            w = synth.make_weights(t, n, k, seed=k + n)
            x = to_dev(synth.make_activations(m, k, 5))
            bias = to_dev(np.linspace(-1, 1, n).astype(np.float32))
            ref = _full(lib, x, to_dev(w), t, k, n, m, bias)
            sw = grp.shard(torch.from_numpy(w), t, k, n)
            for _ in range(3):  # consecutive calls alternate the two y buffers
                y = grp.matmul(x, sw, m, bias)
                ok &= bool(torch.equal(y, ref))
            # the NCCL baseline runs matmul_quant on the slice alone (its own tile
            # shape), so it is held to the oracle tolerance instead of bitwise
            y_ref, a_ref = orc.matmul(x.cpu().numpy(), w, t, k, n, bias=bias.cpu().numpy(), with_abs=True)
            yn = grp.matmul_nccl(x, sw, m, bias).cpu().numpy()
            ok &= bool(np.all(np.abs(yn.astype(np.float64) - y_ref) <= 1e-5 * a_ref + 1e-30))
        torch.cuda.synchronize()
        ok &= lib.cllm_cuda_check_device_status() == 0
        grp.close()
        dist.barrier()
    finally:
        q.put((rank, ok))
        dist.destroy_process_group()


@pytest.mark.timeout(600)
def test_rowshard_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_two_gpu_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=500) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    assert res == {0: True, 1: True}
    assert all(p.exitcode == 0 for p in procs)
