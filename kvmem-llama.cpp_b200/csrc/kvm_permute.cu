// kvm_permute.cu -- in-place slot moves of retained blocks.
//
// Replaces the layout gather/scatter of retained blocks
// (layout_gpu_slots_by_orig_pos, src/adapter/llama-memory-kvmem.cpp:931-1254,
// kvmem_d2d_batched, llama-kvmem-stagein.cu:965-1000).
//
// permute_chain_kernel / permute_kernel move retained blocks from their old
// slot to their new slot in place, each byte crossing HBM once each way.  The
// chronological layout keeps retained blocks in order, so the streaming kernel
// copies the moves of each (layer, K|V, piece of the span) in an order where
// every slot is read before it is overwritten, through a ring of TMA buffers.
// Move lists that are not monotone, and windows that are not 16-byte aligned,
// use column staging instead: a CTA owns a byte column of the slot span for
// one (layer, K|V) and stages that column of every moving block in shared
// memory before writing any of them, so any permutation needs no scratch.
#include "kvm_internal.cuh"
#include "kvm_kernels.h"

#include <atomic>

namespace kvm {

// ------------------------------------------------------------- permute --

// Per-move metadata, validated once per CTA and kept in shared memory so the
// copy loops issue one independent global access each.
struct MoveMeta {
    uint32_t from;
    uint32_t to;
    uint32_t n_tok;   // 0 for an invalid move: nothing of it is touched
};

template <typename V>
__device__ __forceinline__ void permute_column(const MoveMeta *meta, uint8_t *col, uint32_t n_moves,
                                               uint32_t cw, uint8_t *base, uint32_t span, uint32_t rb,
                                               uint32_t c0) {
    constexpr uint32_t G = sizeof(V);
    constexpr uint32_t U = 4;                 // accesses in flight per thread
    const uint32_t per_move = cw / G;
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
                off[j] = m * cw + o;
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
                *reinterpret_cast<const V *>(col + m * cw + o);
    }
    __syncthreads();
}

// The column width follows the actual move count: the widest column (a
// multiple of 16 bytes, at most col_bytes) whose copy for every moving block
// fits the shared-memory region.  Every CTA computes the same width.
__device__ __forceinline__ uint32_t permute_col_width(const PermuteArgs &a, uint32_t region, uint32_t n_moves) {
    uint32_t cw = (region / n_moves) & ~15u;
    if (cw > a.col_bytes) cw = a.col_bytes;
    return cw < 16u ? 16u : cw;
}

// Validates the move list once per CTA into shared memory; an invalid move
// gets n_tok = 0 and is never touched.
__device__ __forceinline__ void permute_load_meta(const PermuteArgs &a, MoveMeta *meta, uint32_t n_moves) {
    for (uint32_t m = threadIdx.x; m < n_moves; m += blockDim.x) {
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
}

// Unit u of a permute launch: (layer, K|V, column index).
struct PermuteUnit {
    uint8_t *base;
    uint32_t span, rb, c0;
};

__device__ __forceinline__ PermuteUnit permute_unit(const PermuteArgs &a, uint64_t u, uint32_t n_cols_k,
                                                    uint32_t n_cols_v, uint32_t cw) {
    const uint32_t layer = static_cast<uint32_t>(u / (n_cols_k + n_cols_v));
    uint32_t c = static_cast<uint32_t>(u % (n_cols_k + n_cols_v));
    const bool is_v = c >= n_cols_k;
    if (is_v) c -= n_cols_k;
    return PermuteUnit{is_v ? a.dst_v[layer] : a.dst_k[layer], is_v ? a.span_v : a.span_k,
                       is_v ? a.row_bytes_v : a.row_bytes_k, c * cw};
}

__global__ void __launch_bounds__(kPermuteThreads) permute_kernel(PermuteArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t n_moves = min(*a.n_moves_dev, a.max_moves);
    if (n_moves == 0) return;
    MoveMeta *meta = reinterpret_cast<MoveMeta *>(smem);
    uint8_t *col = smem + permute_meta_bytes(a.max_moves);
    const uint32_t cw = permute_col_width(a, a.col_region, n_moves);
    permute_load_meta(a, meta, n_moves);
    __syncthreads();
    const uint32_t n_cols_k = (a.span_k + cw - 1) / cw;
    const uint32_t n_cols_v = (a.span_v + cw - 1) / cw;
    const uint64_t units = static_cast<uint64_t>(a.n_layer) * (n_cols_k + n_cols_v);
    for (uint64_t u = blockIdx.x; u < units; u += gridDim.x) {
        const PermuteUnit pu = permute_unit(a, u, n_cols_k, n_cols_v, cw);
        if (a.vec16)
            permute_column<uint4>(meta, col, n_moves, cw, pu.base, pu.span, pu.rb, pu.c0);
        else
            permute_column<uint16_t>(meta, col, n_moves, cw, pu.base, pu.span, pu.rb, pu.c0);
    }
}

// Column permute by TMA for one warp (the streaming kernel's fallback when the
// move list is not monotone): per unit the lanes issue one bulk load per
// moving block -- its piece of the column -- into `col`, all completing on
// one mbarrier, and only then one bulk store per block to its new slot, so
// every move of the column is read before any is written.
__device__ __forceinline__ void permute_columns_bulk(const PermuteArgs &a, const MoveMeta *meta,
                                                     uint32_t n_moves, uint8_t *col, uint32_t region,
                                                     uint64_t *bar) {
    const uint32_t lane = threadIdx.x;
    const uint32_t cw = permute_col_width(a, region, n_moves);
    const uint32_t n_cols_k = (a.span_k + cw - 1) / cw;
    const uint32_t n_cols_v = (a.span_v + cw - 1) / cw;
    const uint64_t units = static_cast<uint64_t>(a.n_layer) * (n_cols_k + n_cols_v);
    uint32_t phase = 0;
    bool ok = true;
    for (uint64_t u = blockIdx.x; u < units; u += gridDim.x) {
        const PermuteUnit pu = permute_unit(a, u, n_cols_k, n_cols_v, cw);
        // bytes of this column for move m: the block's rows end inside it or past it
        auto piece = [&](uint32_t m) -> uint32_t {
            const uint32_t end = meta[m].n_tok * pu.rb;
            return end > pu.c0 ? min(cw, end - pu.c0) : 0u;
        };
        uint32_t mine = 0;
        for (uint32_t m = lane; m < n_moves; m += 32u) mine += piece(m);
        const uint32_t total = __reduce_add_sync(0xffffffffu, mine);
        if (total == 0) continue;
        if (lane == 0) mbar_arrive_expect_tx(bar, total);
        __syncwarp();
        for (uint32_t m = lane; m < n_moves; m += 32u) {
            const uint32_t len = piece(m);
            if (len) bulk_g2s(col + m * cw, pu.base + static_cast<uint64_t>(meta[m].from) * pu.span + pu.c0, len, bar);
        }
        const bool got = mbar_wait_bounded(bar, phase);
        if (!__shfl_sync(0xffffffffu, got ? 1 : 0, 0)) {
            ok = false;
            break;
        }
        phase ^= 1u;
        for (uint32_t m = lane; m < n_moves; m += 32u) {
            const uint32_t len = piece(m);
            if (len) bulk_s2g(pu.base + static_cast<uint64_t>(meta[m].to) * pu.span + pu.c0, col + m * cw, len);
        }
        bulk_commit();
        bulk_wait_read<0>();   // this lane's stores have read the buffer
        __syncwarp();
    }
    if (!ok) {
        if (lane == 0) set_status(a.status, kErrTimeout);
        (void)mbar_wait_bounded(bar, phase);   // bounded wait for loads still landing here
    }
    bulk_wait_all<0>();
}

// One piece of one move in a stream: the bytes at the same span offset of
// the block's old and new slot.
struct ChainItem {
    uint8_t *dst;
    uint32_t bytes;
    uint32_t pad;
};

// Streaming permute (spans, rows and window 16-byte aligned; one warp a CTA).
// The diff lays the window out chronologically, so retained blocks keep their
// order and the old -> new slot map is monotone.  Then a block moving left
// never lands on a slot that a block moving right still has to read (and
// back), and among left moves (ascending new slot) every slot is read before
// the move that overwrites it, as among right moves taken in descending order.
// Each stream -- one (layer, K|V, piece of the span) -- copies the moves in
// that order through a ring of kChainStages TMA buffers: the loads run up to
// kChainStages - 1 moves ahead of the stores, and no load reads a slot that
// an earlier store of the stream wrote.  Streams touch disjoint bytes.  A
// move list that is not monotone (only a block table edited outside the
// diff can give one) takes the column algorithm instead, which needs no
// order.  Shared memory: [0, 64) barriers, [64, 128) the ring's item
// descriptors, [256, ...) the move table and the processing order, then the
// ring buffers.
__global__ void __launch_bounds__(32) permute_chain_kernel(PermuteArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t n_moves = min(*a.n_moves_dev, a.max_moves);
    if (n_moves == 0) return;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *colbar = full + kChainStages;
    ChainItem *items = reinterpret_cast<ChainItem *>(smem + 64);
    MoveMeta *meta = reinterpret_cast<MoveMeta *>(smem + 256);
    uint16_t *ord = reinterpret_cast<uint16_t *>(smem + 256 + permute_meta_bytes(a.max_moves));
    uint8_t *buf = smem + permute_chain_buf_offset(a.max_moves);
    const uint32_t lane = threadIdx.x;
    const uint32_t P = a.piece;
    permute_load_meta(a, meta, n_moves);
    if (lane == 0) {
        for (int s = 0; s < kChainStages; ++s) mbar_init(&full[s], 1);
        mbar_init(colbar, 1);
        fence_mbar_init();
    }
    __syncwarp();
    // monotone: new and old slots both strictly increase along the list, and
    // every move is valid
    bool bad = false;
    for (uint32_t m = lane + 1u; m < n_moves; m += 32u)
        if (!(a.mv_from[m - 1] < a.mv_from[m] && a.mv_to[m - 1] < a.mv_to[m])) bad = true;
    if (__any_sync(0xffffffffu, bad)) {
        permute_columns_bulk(a, meta, n_moves, buf, static_cast<uint32_t>(kChainStages) * P, colbar);
        return;
    }
    // processing order: left moves in list order, then right moves reversed
    uint32_t n_ord = 0;
    for (uint32_t b = 0; b < n_moves; b += 32u) {
        const uint32_t m = b + lane;
        const bool left = m < n_moves && meta[m].to < meta[m].from;
        const uint32_t mask = __ballot_sync(0xffffffffu, left);
        if (left) ord[n_ord + __popc(mask & ((1u << lane) - 1u))] = static_cast<uint16_t>(m);
        n_ord += __popc(mask);
    }
    for (uint32_t b = 0; b < n_moves; b += 32u) {
        const uint32_t m = n_moves - 1u - (b + lane);
        const bool right = b + lane < n_moves && meta[m].to > meta[m].from;
        const uint32_t mask = __ballot_sync(0xffffffffu, right);
        if (right) ord[n_ord + __popc(mask & ((1u << lane) - 1u))] = static_cast<uint16_t>(m);
        n_ord += __popc(mask);
    }
    __syncwarp();
    if (lane != 0) return;
    const uint32_t npk = (a.span_k + P - 1u) / P;
    const uint32_t npv = (a.span_v + P - 1u) / P;
    const uint32_t streams = a.n_layer * (npk + npv);
    // item iterator over this CTA's streams
    uint32_t st = blockIdx.x, k = 0;
    const uint8_t *src = nullptr;
    ChainItem next{nullptr, 0u, 0u};
    auto advance = [&]() -> bool {
        while (st < streams) {
            const uint32_t layer = st / (npk + npv);
            uint32_t p = st - layer * (npk + npv);
            const bool is_v = p >= npk;
            if (is_v) p -= npk;
            uint8_t *base = is_v ? a.dst_v[layer] : a.dst_k[layer];
            const uint32_t span = is_v ? a.span_v : a.span_k;
            const uint32_t rb = is_v ? a.row_bytes_v : a.row_bytes_k;
            const uint32_t off = p * P;
            while (k < n_ord) {
                const MoveMeta mm = meta[ord[k++]];
                const uint32_t end = mm.n_tok * rb;
                if (end > off) {
                    src = base + static_cast<uint64_t>(mm.from) * span + off;
                    next.dst = base + static_cast<uint64_t>(mm.to) * span + off;
                    next.bytes = min(P, end - off);
                    return true;
                }
            }
            st += gridDim.x;
            k = 0;
        }
        return false;
    };
    auto load = [&](uint32_t j) {
        const uint32_t s = j % kChainStages;
        items[s] = next;
        mbar_arrive_expect_tx(&full[s], next.bytes);
        bulk_g2s(buf + s * P, src, next.bytes, &full[s]);
    };
    uint32_t issued = 0;
    while (issued < static_cast<uint32_t>(kChainStages - 1) && advance()) load(issued++);
    for (uint32_t i = 0; i < issued; ++i) {
        const uint32_t s = i % kChainStages;
        if (!mbar_wait_bounded(&full[s], (i / kChainStages) & 1u)) {
            set_status(a.status, kErrTimeout);
            // bounded waits for the loads still landing in this CTA's shared memory
            for (uint32_t j = i; j < issued; ++j)
                (void)mbar_wait_bounded(&full[j % kChainStages], (j / kChainStages) & 1u);
            break;
        }
        bulk_s2g(items[s].dst, buf + s * P, items[s].bytes);
        bulk_commit();
        if (advance()) {
            bulk_wait_read<1>();   // the previous store has read the buffer refilled now
            load(issued++);
        }
    }
    bulk_wait_all<0>();
}

// ------------------------------------------------------------- launchers --

static std::atomic<uint64_t> g_permute_attr{0};
static std::atomic<uint64_t> g_permute_chain_attr{0};

cudaError_t launch_permute(const PermuteArgs &a, cudaStream_t stream) {
    // the streaming kernel when the window is 16-byte aligned and its move
    // table, order and ring (whose columns must also hold 16 bytes of every
    // move for the fallback) fit; the SIMT column kernel otherwise
    const size_t chain_smem = permute_chain_buf_offset(a.max_moves) + static_cast<size_t>(kChainStages) * a.piece;
    if (a.vec16 && a.piece >= 16u && a.piece % 16u == 0 && a.max_moves <= 65535u &&
        static_cast<uint64_t>(kChainStages) * a.piece >= 16ull * a.max_moves && chain_smem <= 200u * 1024u) {
        const size_t smem = chain_smem;
        const void *fn = reinterpret_cast<const void *>(permute_chain_kernel);
        if (!attr_once(g_permute_chain_attr, fn, 200 * 1024)) return cudaErrorInvalidValue;
        int per_sm = 1;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, permute_chain_kernel, 32, smem);
        if (per_sm < 1) per_sm = 1;
        const uint32_t streams = a.n_layer * ((a.span_k + a.piece - 1u) / a.piece + (a.span_v + a.piece - 1u) / a.piece);
        uint32_t grid = static_cast<uint32_t>(num_sms() * per_sm);
        if (grid > streams) grid = streams;
        permute_chain_kernel<<<grid ? grid : 1u, 32, smem, stream>>>(a);
        return cudaGetLastError();
    }
    const size_t smem = permute_meta_bytes(a.max_moves) + a.col_region;
    if (smem > 200u * 1024u || a.col_region < 16u * a.max_moves) return cudaErrorInvalidValue;
    if (!attr_once(g_permute_attr, reinterpret_cast<const void *>(permute_kernel), 200 * 1024))
        return cudaErrorInvalidValue;
    const uint32_t grid = static_cast<uint32_t>(num_sms() * 2);
    permute_kernel<<<grid, kPermuteThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace kvm
