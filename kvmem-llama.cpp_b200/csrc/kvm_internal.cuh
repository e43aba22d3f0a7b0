// kvm_internal.cuh -- shared device helpers and session layout of libkvm.
//
// sm_100a only.  No fast-math: every float/double operation that must match
// the reference's CPU arithmetic bit for bit uses an explicit _rn intrinsic
// so nvcc cannot contract it into an FMA.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <stdint.h>
#include <utility>

#include "../../include/kvm.h"

namespace kvm {

// ---------------------------------------------------------------- limits --
constexpr uint32_t kMaxBlocks = 65536;      // block-table capacity per session
constexpr uint32_t kMaxLayers = 256;
constexpr uint32_t kMaxHeadDim = 1024;
constexpr uint32_t kMaxHeadsKv = 64;

// Device status word bits (session->d_status).
constexpr uint32_t kErrTimeout = 1u << 0;   // a bounded mbarrier wait gave up
constexpr uint32_t kErrIndex = 1u << 1;     // an index outside the session tables
constexpr uint32_t kErrSlot = 1u << 2;      // a slot outside the window
constexpr uint32_t kErrConfig = 1u << 3;    // a launch saw an impossible configuration

// Bounded waits: give up after this many nanoseconds of %globaltimer.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// ------------------------------------------------------------- plan header --
// Counts written by the select / diff kernels (device), read back by
// kvm_get_plan.  Field order is part of the D2H copy layout.
struct PlanHeader {
    uint32_t n_selected;
    uint32_t n_stage_in;
    uint32_t n_stage_out;
    uint32_t n_remaps;
    uint32_t total_window_tokens;
    uint32_t selection_overlap_blocks;
    uint32_t gpu_reused_blocks;
    uint32_t retained_position_stable;
    uint32_t retained_position_moved;
    uint32_t n_moves;
    uint32_t n_cold;
    uint32_t n_blocks;          // block count the plan was computed for
    uint32_t pad[4];
};
static_assert(sizeof(PlanHeader) == 64, "PlanHeader");

// Device block table (KvMemBlock fields used by the path), SoA.
struct BlockTable {
    uint32_t *n_tokens;
    uint8_t  *tier;
    int32_t  *gpu_slot;
    int64_t  *baked_pos;
    uint32_t *remap_count;
    uint64_t *remap_abs_delta;
    uint8_t  *in_ws;
};

// Device plan arrays (capacity max_blocks each).
struct PlanArrays {
    PlanHeader *hdr;
    uint32_t *selected;
    uint32_t *stage_in;
    uint32_t *stage_out;
    uint32_t *rm_block_id;
    uint32_t *rm_n_tokens;
    int32_t  *rm_from_base;
    int32_t  *rm_to_base;
    uint8_t  *rm_wkr;
    uint8_t  *rm_skip;
    uint8_t  *rm_raw;
    uint32_t *mv_block;
    int32_t  *mv_from;
    int32_t  *mv_to;
    uint32_t *cold_block;
    int32_t  *cold_to;
};

// ------------------------------------------------------- division by d --
// floor(t / d) for a divisor fixed per launch, as a multiply-high by
// m = ceil(2^32 / d).  With m*d = 2^32 + e, 0 <= e < d, t*m / 2^32 = t/d +
// t*e / (d*2^32), and the error term stays below 1/d -- so the floor is exact
// -- whenever t*e < 2^32, in particular whenever t*d <= 2^32.  The task
// decoders below take this path when every dividend times its divisor is
// within that bound and divide otherwise.
struct FastDiv {
    uint32_t d;
    uint64_t m;
};

__device__ __forceinline__ FastDiv make_fastdiv(uint32_t d) {
    return FastDiv{d, ((1ull << 32) + d - 1u) / d};
}

__device__ __forceinline__ uint32_t fast_div(uint32_t t, const FastDiv &f) {
    return static_cast<uint32_t>((static_cast<uint64_t>(t) * f.m) >> 32);
}

// ------------------------------------------------------------ PTX wrappers --
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait that may suspend the thread until the phase completes or
// `hint_ns` nanoseconds pass, so a waiting warp stops taking issue slots.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t *bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase: false after kWaitLimitNs.  Each retry
// suspends for at most kWaitSuspendNs, so the limit is checked at least
// every 64 * kWaitSuspendNs.
constexpr uint32_t kWaitSuspendNs = 1000u;
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 0;; ++i) {
        if (mbar_try_wait_suspend(bar, parity, kWaitSuspendNs)) return true;
        if ((i & 63u) == 63u && global_timer_ns() - t0 > kWaitLimitNs) return false;
    }
}

// Bulk global -> shared copy completing on `bar` (bytes % 16 == 0, both
// addresses 16-byte aligned).  No multicast.
__device__ __forceinline__ void bulk_g2s(void *smem_dst, const void *gmem_src, uint32_t bytes,
                                         uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(smem_dst)), "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Bulk shared -> global copy in the current bulk group.
__device__ __forceinline__ void bulk_s2g(void *gmem_dst, const void *smem_src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gmem_dst),
                 "r"(smem_u32(smem_src)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void bulk_commit() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until at most N bulk groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_all() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// Programmatic dependent launch (sm_90+ PTX).  launch_dependents lets the
// next grid of the stream, launched with programmatic stream serialization,
// start its CTAs now; wait blocks until the grids this one depends on have
// completed and their writes are visible.  Without a programmatic launch
// both are no-ops.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void set_status(uint32_t *status, uint32_t bits) {
    if (status) atomicOr(status, bits);
}

// ------------------------------------------------------------ block scans --
// Exclusive prefix sum over one value per thread of a block of `NT` threads
// (NT multiple of 32, <= 1024).  Returns the exclusive prefix; *total gets the
// block total.  `scratch` holds >= NT/32 + 1 uint32 in shared memory.
template <int NT>
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t *scratch,
                                                         uint32_t *total) {
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    uint32_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) scratch[warp] = x;
    __syncthreads();
    if (warp == 0) {
        constexpr int NW = NT / 32;
        uint32_t w = lane < NW ? scratch[lane] : 0u;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        if (lane < NW) scratch[lane] = w;      // inclusive warp totals
        if (lane == NW - 1) scratch[NW] = w;   // block total
    }
    __syncthreads();
    const uint32_t warp_prefix = warp > 0 ? scratch[warp - 1] : 0u;
    *total = scratch[NT / 32];
    __syncthreads();
    return warp_prefix + x - v;
}

// Four independent exclusive prefix sums in one pass (same contract as
// block_exclusive_scan, component-wise).  `scratch` holds >= NT/32 + 1 uint4.
__device__ __forceinline__ uint4 u4_add(uint4 a, uint4 b) {
    return make_uint4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}

__device__ __forceinline__ uint4 u4_shfl_up(uint4 v, int o) {
    return make_uint4(__shfl_up_sync(0xffffffffu, v.x, o), __shfl_up_sync(0xffffffffu, v.y, o),
                      __shfl_up_sync(0xffffffffu, v.z, o), __shfl_up_sync(0xffffffffu, v.w, o));
}

template <int NT>
__device__ __forceinline__ uint4 block_exclusive_scan4(uint4 v, uint4 *scratch, uint4 *total) {
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    uint4 x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint4 y = u4_shfl_up(x, o);
        if (lane >= o) x = u4_add(x, y);
    }
    if (lane == 31) scratch[warp] = x;
    __syncthreads();
    if (warp == 0) {
        constexpr int NW = NT / 32;
        uint4 w = lane < NW ? scratch[lane] : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint4 y = u4_shfl_up(w, o);
            if (lane >= o) w = u4_add(w, y);
        }
        if (lane < NW) scratch[lane] = w;
        if (lane == NW - 1) scratch[NW] = w;
    }
    __syncthreads();
    const uint4 wp = warp > 0 ? scratch[warp - 1] : make_uint4(0u, 0u, 0u, 0u);
    *total = scratch[NT / 32];
    __syncthreads();
    return make_uint4(wp.x + x.x - v.x, wp.y + x.y - v.y, wp.z + x.z - v.z, wp.w + x.w - v.w);
}

// Eight independent exclusive prefix sums (two uint4) in one pass, same
// contract as block_exclusive_scan4; `scratch` holds >= 2 * (NT/32 + 1) uint4.
template <int NT>
__device__ __forceinline__ void block_exclusive_scan8(uint4 &a, uint4 &b, uint4 *scratch, uint4 *tot_a,
                                                      uint4 *tot_b) {
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    constexpr int NW = NT / 32;
    uint4 xa = a, xb = b;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint4 ya = u4_shfl_up(xa, o);
        const uint4 yb = u4_shfl_up(xb, o);
        if (lane >= o) {
            xa = u4_add(xa, ya);
            xb = u4_add(xb, yb);
        }
    }
    if (lane == 31) {
        scratch[warp] = xa;
        scratch[NW + 1 + warp] = xb;
    }
    __syncthreads();
    if (warp == 0) {
        const uint4 z = make_uint4(0u, 0u, 0u, 0u);
        uint4 wa = lane < NW ? scratch[lane] : z;
        uint4 wb = lane < NW ? scratch[NW + 1 + lane] : z;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint4 ya = u4_shfl_up(wa, o);
            const uint4 yb = u4_shfl_up(wb, o);
            if (lane >= o) {
                wa = u4_add(wa, ya);
                wb = u4_add(wb, yb);
            }
        }
        if (lane < NW) {
            scratch[lane] = wa;
            scratch[NW + 1 + lane] = wb;
        }
        if (lane == NW - 1) {
            scratch[NW] = wa;
            scratch[2 * NW + 1] = wb;
        }
    }
    __syncthreads();
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    const uint4 pa = warp > 0 ? scratch[warp - 1] : z;
    const uint4 pb = warp > 0 ? scratch[NW + warp] : z;
    *tot_a = scratch[NW];
    *tot_b = scratch[2 * NW + 1];
    __syncthreads();
    a = make_uint4(pa.x + xa.x - a.x, pa.y + xa.y - a.y, pa.z + xa.z - a.z, pa.w + xa.w - a.w);
    b = make_uint4(pb.x + xb.x - b.x, pb.y + xb.y - b.y, pb.z + xb.z - b.z, pb.w + xb.w - b.w);
}

// Block-wide sum of one value per thread (all threads get the result).
template <int NT>
__device__ __forceinline__ uint32_t block_sum(uint32_t v, uint32_t *scratch) {
    uint32_t total;
    (void)block_exclusive_scan<NT>(v, scratch, &total);
    return total;
}

// ---------------------------------------------------------- host helpers --

// A launch whose CTAs may start while the previous kernel of the stream is
// still running (programmatic stream serialization); the kernel calls
// pdl_wait() before it reads anything an earlier launch writes.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_after_prev(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                     cudaStream_t stream, Args &&...args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// SM count of the current device (cached per host thread and device).
inline int num_sms() {
    static thread_local int cached[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (cached[dev] <= 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cached[dev] = n > 0 ? n : 148;
    }
    return cached[dev];
}

// Dynamic shared-memory opt-in is a per-device function attribute: set it
// once per device the process launches on.
inline bool attr_once(std::atomic<uint64_t> &done, const void *fn, int bytes) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
    const uint64_t bit = 1ull << dev;
    if (done.load(std::memory_order_acquire) & bit) return true;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
        return false;
    done.fetch_or(bit, std::memory_order_acq_rel);
    return true;
}

}  // namespace kvm
