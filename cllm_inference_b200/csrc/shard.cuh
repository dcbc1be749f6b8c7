// Row-sharded GEMV across the GPUs of one node: the completion barrier.
//
// A row-sharded matmul_quant (the 70B decode configuration: every weight
// matrix split by output rows over `world` GPUs) writes each rank's slice of
// y straight into the y buffer of every rank through NVLink peer mappings
// (gemv_put).  shard_barrier_kernel then tells every peer that this rank's
// slice has landed and waits until every peer has said the same, so that on
// return y is complete on this GPU: an all-gather fused into the GEMV's
// stores plus one signal per pair of GPUs.  Plain peer loads and stores only
// (no multicast objects).
#pragma once
#include "common.cuh"
#include "gemv.cuh"

namespace cllm {

struct ShardSignal {
    uint32_t* pads[kMaxPeers];  // pads[q]: rank q's signal words (one per rank), peer-mapped
    uint32_t* epoch;            // this rank's barrier counter (device memory), +1 per barrier
    int world, rank;
};

// One warp.  The epoch lives in device memory so that a CUDA graph that
// replays the barrier advances it on every replay.
// Launched as a programmatic dependent of the GEMV: it may be resident early,
// waits for the GEMV's completion (griddepcontrol.wait), then lets the next
// kernel in the stream launch and prefetch its weights while it signals.  The
// system-scope fence before each release store orders the GEMV's peer stores
// (which happen before this kernel's wait returns) ahead of the signal.
__global__ void __launch_bounds__(32) shard_barrier_kernel(const ShardSignal s) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int q = threadIdx.x;
    const uint32_t ep = *reinterpret_cast<volatile uint32_t*>(s.epoch) + 1u;
    __syncwarp();
    if (q < s.world) {
        __threadfence_system();
        // "rank s.rank has finished epoch ep" into slot s.rank of rank q's pad
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(s.pads[q] + s.rank), "r"(ep) : "memory");
        const uint32_t* mine = s.pads[s.rank] + q;
        const uint64_t t0 = global_timer_ns();
        for (uint32_t it = 0;; ++it) {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
            if ((int32_t)(v - ep) >= 0) break;
            if ((it & 63u) == 63u && global_timer_ns() - t0 > kWaitLimitNs) {
                atomicExch(&g_device_status, kStatusTimeout);
                break;
            }
        }
    }
    __syncwarp();
    if (q == 0) *s.epoch = ep;
}

// Wait (bounded) until every rank has completed the round in *epoch: the
// last warp of each rank's row-sharded GEMV announced it into slot `rank` of
// every pad.  Launched as a programmatic dependent of that GEMV.
__global__ void __launch_bounds__(32) shard_wait_kernel(const uint32_t* pad, const uint32_t* epoch, int world) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int q = threadIdx.x;
    if (q < world) {
        const uint32_t ep = *reinterpret_cast<const volatile uint32_t*>(epoch);
        const uint64_t t0 = global_timer_ns();
        for (uint32_t it = 0;; ++it) {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(pad + q) : "memory");
            if ((int32_t)(v - ep) >= 0) break;
            if ((it & 63u) == 63u && global_timer_ns() - t0 > kWaitLimitNs) {
                atomicExch(&g_device_status, kStatusTimeout);
                break;
            }
        }
    }
}

// A rank that owns no row of a row-sharded call: announce the round like the
// GEMV's last warp would, without launching a GEMV.
__global__ void __launch_bounds__(32) shard_signal_kernel(const ShardSignal s) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int q = threadIdx.x;
    const uint32_t ep = *reinterpret_cast<volatile uint32_t*>(s.epoch) + 1u;
    __syncwarp();
    if (q < s.world) {
        __threadfence_system();
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(s.pads[q] + s.rank), "r"(ep) : "memory");
    }
    __syncwarp();
    if (q == 0) *s.epoch = ep;
}

// Rows of out_dim owned by `rank` of `world`: as even as possible, the first
// out_dim % world ranks one row more.
__host__ __device__ inline void shard_rows(int out_dim, int world, int rank, int* begin, int* rows) {
    const int base = out_dim / world, rem = out_dim % world;
    *rows = base + (rank < rem ? 1 : 0);
    *begin = rank * base + (rank < rem ? rank : rem);
}

}  // namespace cllm
