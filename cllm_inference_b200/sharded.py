"""Row-sharded matmul_quant across the GPUs of one node (one process per GPU).

The 70B decode configuration splits every weight matrix by output rows over
`world` GPUs: rank r keeps rows [begin_r, begin_r + rows_r) in HBM in native
block layout and computes that slice of y = W x.  Row sharding never splits a
quantization block, and every row is summed exactly as on one GPU, so the
gathered y equals the unsharded matmul_quant result bit for bit.

Two ways to gather the slices:

* ``RowShardGroup.matmul`` -- the product path.  The GEMV stores each output
  element straight into the y buffer of every rank (NVLink peer mappings of
  buffers exchanged as CUDA IPC handles, ``cllm_cuda_ipc_*``); its last warp announces the round to every rank with a
  release store, and the next call (or ``sync``) waits for all announcements
  before it reads its input (``cllm_cuda_matmul_quant_rowshard``,
  ``cllm_cuda_shard_wait``).  No separate collective runs.
* ``RowShardGroup.matmul_nccl`` -- the baseline: the local GEMV, then
  ``all_gather_into_tensor`` over NCCL and a reorder (``gather_rows``).

The reference has no multi-GPU code; the single-GPU call it replaces is
``matmul_quant`` (src/core/quant.cpp:1374-1431).
"""
from __future__ import annotations

import ctypes
import os

from . import _lib, synth


def shard_rows(out_dim: int, world: int, rank: int) -> tuple[int, int]:
    """(first row, row count) of `rank`'s slice (cllm_cuda_shard_rows)."""
    lib = _lib.load()
    b, r = ctypes.c_int(0), ctypes.c_int(0)
    _lib.check(lib.cllm_cuda_shard_rows(out_dim, world, rank, ctypes.byref(b), ctypes.byref(r)))
    return b.value, r.value


def shard_weight_bytes(w, type_: int, in_dim: int, out_dim: int, world: int, rank: int):
    """This rank's rows of a [out_dim] x row_bytes weight matrix (any 1-D uint8 tensor
    or array), as a view: rows are contiguous in the GGML row-major layout."""
    rb = synth.row_bytes(type_, in_dim)
    begin, rows = shard_rows(out_dim, world, rank)
    return w[begin * rb:(begin + rows) * rb]


def gather_rows(local, out_dim: int, group=None):
    """All-gather row slices: local is this rank's [n_rows, rows_r] output; returns
    the full [n_rows, out_dim] on every rank.  Slices are padded to the largest
    one for all_gather_into_tensor and put back in row order."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    n_rows = local.shape[0]
    spans = [shard_rows(out_dim, world, q) for q in range(world)]
    width = max(r for _, r in spans)
    assert local.shape[1] == spans[rank][1]
    padded = torch.zeros(n_rows, width, dtype=local.dtype, device=local.device)
    padded[:, :local.shape[1]] = local
    gathered = torch.empty(world * n_rows, width, dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(gathered, padded, group=group)
    gathered = gathered.view(world, n_rows, width)
    out = torch.empty(n_rows, out_dim, dtype=local.dtype, device=local.device)
    for q, (b, r) in enumerate(spans):
        out[:, b:b + r] = gathered[q, :, :r]
    return out


class ShardedWeight:
    """One rank's rows of a quantized weight matrix, resident in HBM."""

    def __init__(self, data, type_: int, in_dim: int, out_dim: int, world: int, rank: int):
        self.data = data  # uint8 CUDA tensor, rows x row_bytes
        self.type = type_
        self.in_dim = in_dim
        self.out_dim = out_dim
        self.begin, self.rows = shard_rows(out_dim, world, rank)


def open_peer_buffers(lib, nbytes: int, rank: int, world: int, allgather):
    """Allocate this rank's peer-mapped buffer and map every other rank's.

    lib: the C ABI (cllm_cuda_ipc_alloc / cllm_cuda_ipc_open); allgather:
    bytes -> list of every rank's bytes in rank order (any host transport).
    Returns (own pointer, [pointer of rank q's buffer in this process],
    [pointers opened here, to close before the owners free theirs])."""
    own = ctypes.c_void_p()
    handle = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES)()
    _lib.check(lib.cllm_cuda_ipc_alloc(nbytes, ctypes.byref(own), handle))
    handles = allgather(bytes(handle))
    if len(handles) != world or bytes(handles[rank]) != bytes(handle):
        raise RuntimeError("peer buffer exchange returned a wrong handle table")
    ptrs, opened = [], []
    for q, hq in enumerate(handles):
        if q == rank:
            ptrs.append(own.value)
            continue
        buf = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES).from_buffer_copy(hq)
        p = ctypes.c_void_p()
        _lib.check(lib.cllm_cuda_ipc_open(buf, ctypes.byref(p)))
        ptrs.append(p.value)
        opened.append(p.value)
    return own.value, ptrs, opened


class _DeviceArray:
    """fp32 / int32 device memory at a raw address, for torch.as_tensor (no copy)."""

    def __init__(self, ptr: int, n: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 3,
                                         "strides": None}


def _torch_allgather(group):
    def allgather(b: bytes):
        import torch.distributed as dist

        out = [None] * dist.get_world_size(group)
        dist.all_gather_object(out, b, group=group)
        return out
    return allgather


class RowShardGroup:
    """The GPUs of one node (one process per GPU) running row-sharded
    matmul_quant calls.

    Every rank's y buffers and signal pad live in one allocation made by the
    C ABI (cllm_cuda_ipc_alloc) and mapped into the other ranks by CUDA IPC
    handles (plain NVLink peer mappings, no multicast objects).  The handles
    travel over `allgather` (bytes -> list of every rank's bytes), by default
    torch.distributed's all_gather_object on `group`.

    max_out / max_rows size the two y buffers (double-buffered: a fast rank
    may write call n+1's slice while a slow rank still reads call n's result)."""

    def __init__(self, max_out: int, max_rows: int = 8, group=None, allgather=None, rank=None, world=None):
        import torch
        import torch.distributed as dist

        self.group = group if group is not None else (dist.group.WORLD if dist.is_initialized() else None)
        self.world = world if world is not None else dist.get_world_size(self.group)
        self.rank = rank if rank is not None else dist.get_rank(self.group)
        if self.world > 8:
            raise ValueError("row sharding is limited to the 8 GPUs of one node")
        self.dev = torch.device("cuda", torch.cuda.current_device())
        self.lib = _lib.load()
        _lib.check(self.lib.cllm_cuda_init(self.dev.index))
        self.max_out, self.max_rows = max_out, max_rows
        ybytes = (max_rows * max_out * 4 + 255) // 256 * 256
        self._off_sig = 2 * ybytes
        self._off_epoch = self._off_sig + 256
        nbytes = self._off_epoch + 256
        self._allgather = allgather or _torch_allgather(self.group)
        self._own, ptrs, self._opened = open_peer_buffers(self.lib, nbytes, self.rank, self.world,
                                                          self._allgather)
        arr = ctypes.c_void_p * self.world
        self._yptrs = [arr(*[p + i * ybytes for p in ptrs]) for i in range(2)]
        self._sigptrs = arr(*[p + self._off_sig for p in ptrs])
        self._y = [torch.as_tensor(_DeviceArray(self._own + i * ybytes, max_rows * max_out, "<f4"), device=self.dev)
                   for i in range(2)]
        self._sig_ptr = self._own + self._off_sig
        self._epoch_ptr = self._own + self._off_epoch
        self._flip = 0
        self._allgather(b"ready")  # every rank has mapped every buffer before any call writes into it

    def shard(self, w_full, type_: int, in_dim: int, out_dim: int) -> ShardedWeight:
        """Copy this rank's rows of a full weight matrix (uint8 tensor, host or
        device) into HBM."""
        part = shard_weight_bytes(w_full, type_, in_dim, out_dim, self.world, self.rank)
        return ShardedWeight(part.to(self.dev).contiguous(), type_, in_dim, out_dim, self.world, self.rank)

    def matmul(self, x, sw: ShardedWeight, n_rows: int = 1, bias=None, out=None):
        """y = W x for the full W (every rank gets all out_dim outputs).  x:
        [n_rows, in_dim] fp32 on this GPU, the same on every rank; bias: full
        out_dim fp32 or None.  Returns [n_rows, out_dim] (a copy, or `out`)."""
        y = self.matmul_unread(x, sw, n_rows, bias)
        if out is None:
            return y.clone()
        out.copy_(y)
        return out

    def matmul_unread(self, x, sw: ShardedWeight, n_rows: int = 1, bias=None, chain: bool = False,
                      wait: bool = True, signal: bool = True):
        """matmul without the copy-out: returns a view of the group's y buffer,
        valid until the call after next overwrites it.  Each call first waits
        (on the GPU) for every rank to have finished the previous call, so x
        may be the previous call's output; wait=False skips that wait for a
        call whose x does not depend on the previous call (k and v after q,
        up after gate).  chain=True skips the wait for this call's own
        completion: its y may then only be read by the next call of this group
        (or after sync()).  signal=False: the call does not announce its
        round (a following signalling call announces both); only for a call
        whose output the next call does not wait on, and never with chain=False."""
        import torch

        if n_rows > self.max_rows or sw.out_dim > self.max_out:
            raise ValueError("call larger than the group's y buffers")
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        buf = self._flip
        self._flip ^= 1
        solo = self.world == 1  # one GPU: stream order alone completes y
        _lib.check(self.lib.cllm_cuda_matmul_quant_rowshard(
            ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(sw.data.data_ptr()), sw.type,
            ctypes.c_void_p(bias.data_ptr()) if bias is not None else None, sw.in_dim, sw.out_dim,
            self.rank, self.world, n_rows, self._yptrs[buf], None if solo else self._sigptrs,
            None if solo else ctypes.c_void_p(self._epoch_ptr),
            (_lib.SHARD_WAIT_PREV if (wait and not solo) else 0) | (0 if signal else _lib.SHARD_NO_SIGNAL), st))
        if not chain:
            if not signal:
                raise ValueError("signal=False needs chain=True")
            self.sync()
        return self._y[buf][:n_rows * sw.out_dim].view(n_rows, sw.out_dim)

    def sync(self):
        """Wait on the GPU until every rank has finished the last call."""
        import torch

        if self.world > 1:
            st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
            _lib.check(self.lib.cllm_cuda_shard_wait(ctypes.c_void_p(self._sig_ptr),
                                                     ctypes.c_void_p(self._epoch_ptr), self.world, st))

    def matmul_nccl(self, x, sw: ShardedWeight, n_rows: int = 1, bias=None):
        """The same result through the local GEMV and an NCCL all-gather."""
        import torch

        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        local = torch.empty(n_rows, sw.rows, dtype=torch.float32, device=self.dev)
        b = bias[sw.begin:sw.begin + sw.rows].contiguous() if bias is not None else None
        _lib.check(self.lib.cllm_cuda_matmul_quant(
            ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(sw.data.data_ptr()), sw.type,
            ctypes.c_void_p(b.data_ptr()) if b is not None else None, sw.in_dim, sw.rows, n_rows,
            ctypes.c_void_p(local.data_ptr()), 0, st))
        return gather_rows(local, sw.out_dim, self.group)

    def close(self):
        """Unmap the peers' buffers, then (after every rank has) free this rank's."""
        import torch

        if self._own is None:
            return
        torch.cuda.synchronize()
        for p in self._opened:
            _lib.check(self.lib.cllm_cuda_ipc_close(ctypes.c_void_p(p)))
        self._opened = []
        self._allgather(b"closed")
        self._y = []
        _lib.check(self.lib.cllm_cuda_ipc_free(ctypes.c_void_p(self._own)))
        self._own = None
