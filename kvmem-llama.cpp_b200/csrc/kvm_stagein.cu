// kvm_stagein.cu -- fused gather + quantize stage-in and in-place slot moves.
//
// Replaces the reference's stage-in (write_block_to_gpu -> RawKvStore::copy_*
// -> kvmem_stagein_enqueue_v -> kvmem_stagein_flush,
// src/adapter/llama-memory-kvmem.cpp:2726-2791, src/adapter/llama-kvmem-stagein.cu:632-753)
// and the layout gather/scatter of retained blocks (layout_gpu_slots_by_orig_pos,
// llama-memory-kvmem.cpp:931-1254, kvmem_d2d_batched, stagein.cu:965-1000).
//
// stagein_kernel: persistent CTAs walk (cold block, layer, K|V, row tile)
// tasks.  One elected thread streams each F16 tile (rows x n_embd halves,
// contiguous) into shared memory with cp.async.bulk (TMA bulk copy, completed
// on an mbarrier) NSTAGE tiles ahead; all threads quantize the tile into a
// shared-memory output buffer (4 lanes per ggml block), then the elected
// thread writes the tile's quantized rows (contiguous in the window) back with
// one cp.async.bulk shared->global store.  Every wait is bounded.
//
// permute_kernel: moves retained blocks from their old slot to their new slot
// in place.  Each CTA owns a byte column of the slot span for one (layer, K|V)
// and stages that column of every moving block in shared memory before
// writing any of them, so chains and cycles of moves need no scratch buffer
// and each byte crosses HBM once in each direction.
#include "kvm_internal.cuh"
#include "kvm_quant.cuh"
#include "kvm_kernels.h"

#include <atomic>

namespace kvm {

namespace {

struct TaskDesc {
    const uint8_t *src;
    uint8_t *dst;
    uint32_t rows;
    uint32_t kv;
    bool valid;
};

__device__ __forceinline__ TaskDesc decode_task(const StageinArgs &a, uint64_t t,
                                                uint32_t tiles, uint32_t n_items) {
    TaskDesc d{nullptr, nullptr, 0u, 0u, false};
    const uint64_t per_item = static_cast<uint64_t>(a.n_layer) * a.n_kv * tiles;
    const uint32_t item = static_cast<uint32_t>(t / per_item);
    uint32_t r = static_cast<uint32_t>(t % per_item);
    const uint32_t layer = r / (a.n_kv * tiles);
    r %= a.n_kv * tiles;
    const uint32_t kv = r / tiles;
    const uint32_t tile = r % tiles;
    if (item >= n_items) return d;
    const uint32_t idx = a.item0 + item;
    const uint32_t block = a.cold_block[idx];
    const int32_t slot = a.cold_to[idx];
    if (block >= a.max_blocks) {
        set_status(a.status, kErrIndex);
        return d;
    }
    if (slot < 0 || static_cast<uint32_t>(slot) >= a.n_slots) {
        set_status(a.status, kErrSlot);
        return d;
    }
    const uint32_t nt = min(a.n_tokens[block], a.block_tokens);
    const uint32_t row0 = tile * a.rows_per_tile;
    if (row0 >= nt) return d;
    d.rows = min(a.rows_per_tile, nt - row0);
    d.kv = kv;
    const uint64_t src_index = a.src_by_item ? item : block;
    const uint8_t *sbase = kv ? a.src_v : a.src_k;
    d.src = sbase + layer * a.layer_stride + src_index * a.item_stride + row0 * a.row_stride;
    uint8_t *dbase = kv ? a.dst_v[layer] : a.dst_k[layer];
    const uint32_t rb = kv ? a.row_bytes_v : a.row_bytes_k;
    d.dst = dbase + (static_cast<uint64_t>(slot) * a.block_tokens + row0) * rb;
    d.valid = true;
    return d;
}

__device__ __forceinline__ void issue_tile_load(const StageinArgs &a, const TaskDesc &d,
                                                uint8_t *buf, uint64_t *bar) {
    const uint32_t row_in = a.n_embd * 2u;
    const uint32_t bytes = d.rows * row_in;
    mbar_arrive_expect_tx(bar, bytes);
    if (a.row_stride == row_in) {
        bulk_g2s(buf, d.src, bytes, bar);
    } else {
        for (uint32_t r = 0; r < d.rows; ++r) {
            bulk_g2s(buf + r * row_in, d.src + r * a.row_stride, row_in, bar);
        }
    }
}

}  // namespace

// Per-stage tile description, written by the producer before it arms the
// stage's `full` barrier (release) and read by consumers after their wait
// (acquire).  rows == 0 marks the end of this CTA's work.
struct TileSlot {
    uint8_t *dst;
    uint32_t rows;
    int32_t type;
    uint32_t out_bytes;
    uint32_t pad;
};
static_assert(sizeof(TileSlot) == 24, "TileSlot");

// Shared memory: [0,128) barriers (full[NS], done[NS]); [128,384) tile slots;
// then NS input tiles and NS output tiles.
constexpr uint32_t kStageinHeader = 384;

template <int NS>
__global__ void __launch_bounds__(kStageinThreads, 1) stagein_kernel(StageinArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *done = full + NS;
    TileSlot *slot = reinterpret_cast<TileSlot *>(smem + 128);
    uint8_t *in_buf = smem + kStageinHeader;
    uint8_t *out_buf = in_buf + NS * a.tile_in_bytes;

    const uint32_t n_items_raw = a.n_items_dev ? *a.n_items_dev : a.n_items_host;
    const uint32_t n_items = min(n_items_raw, a.max_items);
    const uint32_t tiles = (a.block_tokens + a.rows_per_tile - 1) / a.rows_per_tile;
    const uint64_t total = static_cast<uint64_t>(n_items) * a.n_layer * a.n_kv * tiles;
    if (static_cast<uint64_t>(blockIdx.x) >= total) return;

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&done[s], kStageinConsumerWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();   // the only CTA-wide barrier

    if (warp == kStageinConsumerWarps) {
        // ---------------------------------------------------------- producer
        uint64_t ptask = blockIdx.x;
        uint32_t issued = 0;      // tiles armed with data
        bool ended = false;       // end marker placed
        // Arm the stage of tile index `issued` with the next task, or with
        // the end marker when none is left.  Lane 0 only.
        auto arm_next = [&]() {
            const uint32_t s = issued % NS;
            while (ptask < total) {
                const TaskDesc d = decode_task(a, ptask, tiles, n_items);
                ptask += gridDim.x;
                if (!d.valid) continue;
                TileSlot &ts = slot[s];
                ts.dst = d.dst;
                ts.rows = d.rows;
                ts.type = d.kv ? a.type_v : a.type_k;
                ts.out_bytes = d.rows * (d.kv ? a.row_bytes_v : a.row_bytes_k);
                issue_tile_load(a, d, in_buf + s * a.tile_in_bytes, &full[s]);
                ++issued;
                return;
            }
            slot[s].rows = 0;
            mbar_arrive(&full[s]);
            ended = true;
        };
        if (lane == 0) {
            while (!ended && issued < static_cast<uint32_t>(NS)) arm_next();
        }
        __syncwarp();   // slot[] written by lane 0 is read by every producer lane
        issued = __shfl_sync(0xffffffffu, issued, 0);
        ended = __shfl_sync(0xffffffffu, ended ? 1 : 0, 0) != 0;
        const uint32_t lag = a.bulk_store ? 1u : 0u;
        bool bad = false;
        for (uint32_t j = 0; j < issued; ++j) {
            const uint32_t s = j % NS;
            bool ok = true;
            if (lane == 0) ok = mbar_wait_bounded(&done[s], (j / NS) & 1u);
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (!ok) {
                bad = true;
                break;
            }
            const TileSlot ts = slot[s];
            const uint8_t *ob = out_buf + s * a.tile_out_bytes;
            if (a.bulk_store) {
                if (lane == 0) {
                    fence_proxy_async_smem();
                    bulk_s2g(ts.dst, ob, ts.out_bytes);
                    bulk_commit();
                }
            } else {
                for (uint32_t o = 2u * lane; o < ts.out_bytes; o += 64u)
                    *reinterpret_cast<uint16_t *>(ts.dst + o) =
                        *reinterpret_cast<const uint16_t *>(ob + o);
                __syncwarp();
            }
            if (j >= lag && lane == 0 && !ended) {
                // the stage of tile j - lag is free once its store has read it
                if (a.bulk_store) bulk_wait_read<1>();
                arm_next();
            }
            __syncwarp();
            issued = __shfl_sync(0xffffffffu, issued, 0);
            ended = __shfl_sync(0xffffffffu, ended ? 1 : 0, 0) != 0;
        }
        if (lane == 0) {
            if (bad) {
                set_status(a.status, kErrTimeout);
                // bounded wait for loads still landing in this CTA's smem
                for (int s = 0; s < NS; ++s) {
                    const uint32_t last = issued > static_cast<uint32_t>(s)
                                              ? issued - 1 - ((issued - 1 - s) % NS) : 0u;
                    if (issued > static_cast<uint32_t>(s))
                        (void)mbar_wait_bounded(&full[s], (last / NS) & 1u);
                }
            }
            if (a.bulk_store) bulk_wait_all<0>();
        }
        return;
    }

    // ------------------------------------------------------------- consumers
    const uint32_t qb_per_row = a.n_embd / 32u;
    for (uint32_t j = 0;; ++j) {
        const uint32_t s = j % NS;
        if (!mbar_wait_bounded(&full[s], (j / NS) & 1u)) {
            set_status(a.status, kErrTimeout);
            break;
        }
        const TileSlot ts = slot[s];
        if (ts.rows == 0) break;
        const uint8_t *ib = in_buf + s * a.tile_in_bytes;
        uint8_t *ob = out_buf + s * a.tile_out_bytes;
        const uint32_t nqb = ts.rows * qb_per_row;
        for (uint32_t qb = static_cast<uint32_t>(warp * 32 + lane); qb < nqb;
             qb += kStageinConsumerWarps * 32u) {
            Block32 b;
            load_block(ib, qb, lane, b);
            quant_block(ts.type, b, ob, qb);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&done[s]);
    }
}

// ------------------------------------------------------------- permute --

// Per-move metadata, validated once per CTA and kept in shared memory so the
// copy loops issue one independent global access each.
struct MoveMeta {
    uint32_t from;
    uint32_t to;
    uint32_t n_tok;   // 0 for an invalid move: nothing of it is touched
};

template <typename V>
__device__ __forceinline__ void permute_column(const PermuteArgs &a, const MoveMeta *meta,
                                               uint8_t *col, uint32_t n_moves, uint8_t *base,
                                               uint32_t span, uint32_t rb, uint32_t c0) {
    constexpr uint32_t G = sizeof(V);
    constexpr uint32_t U = 4;                 // accesses in flight per thread
    const uint32_t per_move = a.col_bytes / G;
    const uint32_t n_acc = n_moves * per_move;
    const uint32_t stride = kPermuteThreads * U;
    // gather this column of every moving block into shared memory
    for (uint32_t i0 = threadIdx.x; i0 < n_acc; i0 += stride) {
        V r[U];
        uint32_t off[U];
        bool ok[U];
#pragma unroll
        for (uint32_t j = 0; j < U; ++j) {
            const uint32_t i = i0 + j * kPermuteThreads;
            ok[j] = false;
            if (i < n_acc) {
                const uint32_t m = i / per_move;
                const uint32_t o = (i - m * per_move) * G;
                const MoveMeta mm = meta[m];
                off[j] = m * a.col_bytes + o;
                if (c0 + o < mm.n_tok * rb) {
                    r[j] = *reinterpret_cast<const V *>(base + static_cast<uint64_t>(mm.from) * span + c0 + o);
                    ok[j] = true;
                }
            }
        }
#pragma unroll
        for (uint32_t j = 0; j < U; ++j)
            if (ok[j]) *reinterpret_cast<V *>(col + off[j]) = r[j];
    }
    __syncthreads();
    // scatter it to the new slots
    for (uint32_t i = threadIdx.x; i < n_acc; i += kPermuteThreads) {
        const uint32_t m = i / per_move;
        const uint32_t o = (i - m * per_move) * G;
        const MoveMeta mm = meta[m];
        if (c0 + o < mm.n_tok * rb)
            *reinterpret_cast<V *>(base + static_cast<uint64_t>(mm.to) * span + c0 + o) =
                *reinterpret_cast<const V *>(col + m * a.col_bytes + o);
    }
    __syncthreads();
}

__global__ void __launch_bounds__(kPermuteThreads) permute_kernel(PermuteArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t n_moves = min(*a.n_moves_dev, a.max_moves);
    if (n_moves == 0) return;
    MoveMeta *meta = reinterpret_cast<MoveMeta *>(smem);
    uint8_t *col = smem + permute_meta_bytes(a.max_moves);
    for (uint32_t m = threadIdx.x; m < n_moves; m += kPermuteThreads) {
        const uint32_t blk = a.mv_block[m];
        const int32_t from = a.mv_from[m];
        const int32_t to = a.mv_to[m];
        MoveMeta mm{0u, 0u, 0u};
        if (blk < a.max_blocks && from >= 0 && static_cast<uint32_t>(from) < a.n_slots && to >= 0 &&
            static_cast<uint32_t>(to) < a.n_slots) {
            mm.from = static_cast<uint32_t>(from);
            mm.to = static_cast<uint32_t>(to);
            mm.n_tok = min(a.n_tokens[blk], a.block_tokens);
        } else if (blockIdx.x == 0) {
            set_status(a.status, kErrSlot);
        }
        meta[m] = mm;
    }
    __syncthreads();
    const uint32_t n_cols_k = (a.span_k + a.col_bytes - 1) / a.col_bytes;
    const uint32_t n_cols_v = (a.span_v + a.col_bytes - 1) / a.col_bytes;
    const uint64_t units = static_cast<uint64_t>(a.n_layer) * (n_cols_k + n_cols_v);
    for (uint64_t u = blockIdx.x; u < units; u += gridDim.x) {
        const uint32_t layer = static_cast<uint32_t>(u / (n_cols_k + n_cols_v));
        uint32_t c = static_cast<uint32_t>(u % (n_cols_k + n_cols_v));
        const bool is_v = c >= n_cols_k;
        if (is_v) c -= n_cols_k;
        uint8_t *base = is_v ? a.dst_v[layer] : a.dst_k[layer];
        const uint32_t span = is_v ? a.span_v : a.span_k;
        const uint32_t rb = is_v ? a.row_bytes_v : a.row_bytes_k;
        if (a.vec16)
            permute_column<uint4>(a, meta, col, n_moves, base, span, rb, c * a.col_bytes);
        else
            permute_column<uint16_t>(a, meta, col, n_moves, base, span, rb, c * a.col_bytes);
    }
}

// ------------------------------------------------------------- launchers --

static int g_num_sms = 0;

static int num_sms() {
    if (g_num_sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_num_sms <= 0) g_num_sms = 148;
    }
    return g_num_sms;
}

uint32_t stagein_rows_per_tile(uint32_t n_embd, uint32_t block_tokens) {
    // 16 KiB of F16 per tile (8 rows at n_embd = 1024)
    uint32_t r = 8192u / (n_embd ? n_embd : 1u);
    if (r < 1u) r = 1u;
    if (r > block_tokens) r = block_tokens;
    return r;
}

size_t stagein_smem_bytes(const StageinArgs &a) {
    return kStageinHeader +
           static_cast<size_t>(kStageinStages) * (a.tile_in_bytes + a.tile_out_bytes);
}

// Dynamic shared-memory opt-in is a per-device function attribute: set it
// once per device the process launches on.
static bool attr_once(std::atomic<uint64_t> &done, const void *fn, int bytes) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
    const uint64_t bit = 1ull << dev;
    if (done.load(std::memory_order_acquire) & bit) return true;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
        return false;
    done.fetch_or(bit, std::memory_order_acq_rel);
    return true;
}

static std::atomic<uint64_t> g_stagein_attr{0};
static std::atomic<uint64_t> g_permute_attr{0};

cudaError_t launch_stagein(const StageinArgs &a, cudaStream_t stream, uint32_t grid_cap) {
    const size_t smem = stagein_smem_bytes(a);
    if (smem > 200u * 1024u) return cudaErrorInvalidValue;
    if (!attr_once(g_stagein_attr, reinterpret_cast<const void *>(stagein_kernel<kStageinStages>),
                   200 * 1024))
        return cudaErrorInvalidValue;
    int per_sm = 1;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, stagein_kernel<kStageinStages>,
                                                  kStageinThreads, smem);
    if (per_sm < 1) per_sm = 1;
    uint32_t grid = static_cast<uint32_t>(num_sms() * per_sm);
    if (grid_cap && grid > grid_cap) grid = grid_cap;
    if (grid == 0) grid = 1;
    stagein_kernel<kStageinStages><<<grid, kStageinThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_permute(const PermuteArgs &a, cudaStream_t stream) {
    const size_t smem = permute_meta_bytes(a.max_moves) + static_cast<size_t>(a.max_moves) * a.col_bytes;
    if (smem > 200u * 1024u) return cudaErrorInvalidValue;
    if (!attr_once(g_permute_attr, reinterpret_cast<const void *>(permute_kernel), 200 * 1024))
        return cudaErrorInvalidValue;
    const uint32_t grid = static_cast<uint32_t>(num_sms() * 2);
    permute_kernel<<<grid, kPermuteThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace kvm
