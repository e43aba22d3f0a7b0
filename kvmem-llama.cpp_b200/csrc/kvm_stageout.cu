// kvm_stageout.cu -- stage-out (harvest) of packed window rows, and stage-in
// of packed rows back into the window.
//
// Replaces the reference's harvest gather (harvest_gpu_v ->
// kvmem_stageout_enqueue / kvmem_stageout_submit,
// src/adapter/llama-memory-kvmem.cpp:2318-2410,
// src/adapter/llama-kvmem-stagein.cu:842-963): for a list of blocks, every
// layer's K and V rows (n_tokens rows from the block's window slot, read from
// the device block table so no host round trip is needed) are packed into a
// contiguous destination -- item j at dst + j*item_bytes, layer l at
// + l*T*(row_bytes_k + row_bytes_v), K rows then V rows.
//
// stageout_kernel: a one-warp CTA whose elected lane moves 16 KiB pieces with
// TMA bulk copies -- cp.async.bulk global->shared completing on an mbarrier,
// then cp.async.bulk shared->global -- double-buffered so the store of one
// piece overlaps the load of the next; six or seven such CTAs per SM keep
// ~200 KiB in flight.  A byte-copy path serves destinations or rows that are
// not 16-byte aligned.
//
// packed_stagein_kernel: the reverse copy for kvm_stagein_packed (the
// reference's stage-in as it runs today: write_block_to_gpu ->
// kvmem_stagein_enqueue_v / kvmem_stagein_flush): each cold block's packed
// rows, from a block-indexed source or a staging-ring chunk, into its window
// slot, with the same bulk-copy loop.
#include "kvm_internal.cuh"
#include "kvm_kernels.h"

#include <atomic>

namespace kvm {

namespace {

constexpr uint32_t kPiece = 16u * 1024u;
constexpr int kOutStages = 2;
constexpr uint32_t kOutSmem = 128u + kOutStages * kPiece;

struct Piece {
    const uint8_t *src;
    uint8_t *dst;
    uint32_t bytes;
};

// Unit u = ((j * L + l) * 2 + kv) * pieces + p of a launch of `total` units:
// (j, l, kv, p) by multiply-highs (FastDiv) when total * max(pieces, L) <= 2^32
// (every dividend times its divisor is then within the bound), else by
// division.
struct UnitIndex {
    FastDiv pieces, layers;
    bool magic;
};

__device__ __forceinline__ UnitIndex make_unit_index(uint32_t pieces, uint32_t n_layer, uint64_t total) {
    UnitIndex ui;
    ui.pieces = make_fastdiv(pieces);
    ui.layers = make_fastdiv(n_layer);
    ui.magic = total < (1ull << 32) && total * (pieces > n_layer ? pieces : n_layer) <= (1ull << 32);
    return ui;
}

struct Unit {
    uint32_t j, l, kv, p;
};

__device__ __forceinline__ Unit split_unit(uint64_t u, const UnitIndex &ui) {
    Unit x;
    uint32_t r;
    if (ui.magic) {
        const uint32_t q = fast_div(static_cast<uint32_t>(u), ui.pieces);
        x.p = static_cast<uint32_t>(u) - q * ui.pieces.d;
        x.kv = q & 1u;
        r = q >> 1;
        x.j = fast_div(r, ui.layers);
        x.l = r - x.j * ui.layers.d;
    } else {
        x.p = static_cast<uint32_t>(u % ui.pieces.d);
        const uint64_t q = u / ui.pieces.d;
        x.kv = static_cast<uint32_t>(q & 1u);
        x.l = static_cast<uint32_t>((q >> 1) % ui.layers.d);
        x.j = static_cast<uint32_t>((q >> 1) / ui.layers.d);
    }
    return x;
}

// bytes == 0: nothing to move.
__device__ __forceinline__ Piece decode_piece(const StageoutArgs &a, uint64_t u, const UnitIndex &ui) {
    Piece pc{nullptr, nullptr, 0u};
    const Unit x = split_unit(u, ui);
    const uint32_t p = x.p, kv = x.kv, l = x.l, j = x.j;
    const uint32_t b = a.ids[j];
    const bool ok = b < a.n_blocks;
    const int32_t slot = ok ? a.gpu_slot[b] : -1;
    const bool res = slot >= 0 && static_cast<uint32_t>(slot) < a.n_slots;
    if (p == 0 && l == 0 && kv == 0 && a.resident) a.resident[a.item0 + j] = res ? 1u : 0u;
    if (!res) return pc;
    const uint32_t nt = min(a.n_tokens[b], a.block_tokens);
    const uint32_t rb = kv ? a.row_bytes_v : a.row_bytes_k;
    const uint32_t total = nt * rb;
    const uint32_t off = p * kPiece;
    if (off >= total) return pc;
    pc.bytes = min(kPiece, total - off);
    const uint8_t *base = kv ? a.win_v[l] : a.win_k[l];
    pc.src = base + static_cast<uint64_t>(slot) * a.block_tokens * rb + off;
    pc.dst = a.dst + static_cast<uint64_t>(j) * a.item_bytes +
             static_cast<uint64_t>(l) * a.block_tokens * (a.row_bytes_k + a.row_bytes_v) +
             (kv ? static_cast<uint64_t>(a.block_tokens) * a.row_bytes_k : 0ull) + off;
    return pc;
}

// The copy loop of one CTA over units blockIdx.x, +gridDim.x, ... < total:
// decode(u) names a piece (bytes == 0: nothing to move).  Lane 0 moves pieces
// with bulk copies through two shared-memory buffers; without `bulk` every
// lane copies bytes.
template <typename Decode>
__device__ __forceinline__ void copy_pieces(uint64_t total, bool bulk, uint32_t *status,
                                            const Decode &decode) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint8_t *buf = smem + 128;
    const int lane = threadIdx.x;
    if (!bulk) {
        for (uint64_t u = blockIdx.x; u < total; u += gridDim.x) {
            const Piece pc = decode(u);
            for (uint32_t i = lane; i < pc.bytes; i += 32u) pc.dst[i] = pc.src[i];
        }
        return;
    }
    if (lane != 0) return;
    for (int s = 0; s < kOutStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
    uint64_t u = blockIdx.x;
    // the next piece with bytes to move, or false at the end
    auto next_piece = [&](Piece &pc) {
        for (; u < total; u += gridDim.x) {
            pc = decode(u);
            if (pc.bytes != 0u) {
                u += gridDim.x;
                return true;
            }
        }
        return false;
    };
    Piece cur{nullptr, nullptr, 0u};
    bool have = next_piece(cur);
    uint32_t k = 0;
    bool ok = true;
    while (have) {
        const uint32_t s = k % kOutStages;
        // the store that last read stage s was issued kOutStages pieces ago
        if (k >= static_cast<uint32_t>(kOutStages)) bulk_wait_read<kOutStages - 1>();
        mbar_arrive_expect_tx(&full[s], cur.bytes);
        bulk_g2s(buf + s * kPiece, cur.src, cur.bytes, &full[s]);
        Piece nxt{nullptr, nullptr, 0u};
        have = next_piece(nxt);           // the next decode (global reads) overlaps this load
        if (!mbar_wait_bounded(&full[s], (k / kOutStages) & 1u)) {
            set_status(status, kErrTimeout);
            ok = false;
            break;
        }
        bulk_s2g(cur.dst, buf + s * kPiece, cur.bytes);
        bulk_commit();
        ++k;
        cur = nxt;
    }
    if (!ok) {
        // bounded wait for the load still landing in this CTA's shared memory
        const uint32_t s = k % kOutStages;
        (void)mbar_wait_bounded(&full[s], (k / kOutStages) & 1u);
    }
    bulk_wait_all<0>();
}

__device__ __forceinline__ uint32_t pieces_per_span(uint32_t block_tokens, uint32_t rbk, uint32_t rbv) {
    return (block_tokens * (rbk > rbv ? rbk : rbv) + kPiece - 1u) / kPiece;
}

__global__ void __launch_bounds__(32) stageout_kernel(StageoutArgs a) {
    const uint32_t pieces = pieces_per_span(a.block_tokens, a.row_bytes_k, a.row_bytes_v);
    const uint64_t total = static_cast<uint64_t>(a.n) * a.n_layer * 2u * pieces;
    const UnitIndex ui = make_unit_index(pieces, a.n_layer, total);
    copy_pieces(total, a.bulk != 0u, a.status, [&](uint64_t u) { return decode_piece(a, u, ui); });
}

// Unit u = ((j * L + l) * 2 + kv) * pieces + p over the cold items of this
// launch: block cold_block[item0 + j]'s rows go to window slot cold_to[...].
__device__ __forceinline__ Piece decode_packed_in(const PackedInArgs &a, uint32_t n_items, uint64_t u,
                                                  const UnitIndex &ui) {
    Piece pc{nullptr, nullptr, 0u};
    const Unit x = split_unit(u, ui);
    const uint32_t p = x.p, kv = x.kv, l = x.l, j = x.j;
    if (j >= n_items) return pc;
    const uint32_t idx = a.item0 + j;
    const uint32_t b = a.cold_block[idx];
    const int32_t slot = a.cold_to[idx];
    if (b >= a.max_blocks) {
        if (p == 0 && l == 0 && kv == 0) set_status(a.status, kErrIndex);
        return pc;
    }
    if (slot < 0 || static_cast<uint32_t>(slot) >= a.n_slots) {
        if (p == 0 && l == 0 && kv == 0) set_status(a.status, kErrSlot);
        return pc;
    }
    const uint32_t rb = kv ? a.row_bytes_v : a.row_bytes_k;
    const uint32_t total = min(a.n_tokens[b], a.block_tokens) * rb;
    const uint32_t off = p * kPiece;
    if (off >= total) return pc;
    pc.bytes = min(kPiece, total - off);
    const uint64_t si = a.src_by_item ? j : b;
    pc.src = (kv ? a.src_v : a.src_k) + l * (kv ? a.v_layer_stride : a.k_layer_stride) +
             si * (kv ? a.v_block_stride : a.k_block_stride) + off;
    pc.dst = (kv ? a.win_v[l] : a.win_k[l]) + static_cast<uint64_t>(slot) * a.block_tokens * rb + off;
    return pc;
}

__global__ void __launch_bounds__(32) packed_stagein_kernel(PackedInArgs a) {
    const uint32_t n_items = min(a.n_items_dev ? *a.n_items_dev : a.n_items_host, a.max_items);
    const uint32_t pieces = pieces_per_span(a.block_tokens, a.row_bytes_k, a.row_bytes_v);
    const uint64_t total = static_cast<uint64_t>(n_items) * a.n_layer * 2u * pieces;
    const UnitIndex ui = make_unit_index(pieces, a.n_layer, total);
    copy_pieces(total, a.bulk != 0u, a.status,
                [&](uint64_t u) { return decode_packed_in(a, n_items, u, ui); });
}

}  // namespace

// The copy kernels' shared-memory opt-in, once per device.
static cudaError_t copy_smem_once(const void *kernel, std::atomic<uint64_t> &attr) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!(attr.load(std::memory_order_acquire) & (1ull << dev))) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(kOutSmem));
        if (e != cudaSuccess) return e;
        attr.fetch_or(1ull << dev, std::memory_order_acq_rel);
    }
    return cudaSuccess;
}

static uint32_t copy_grid(const void *kernel, uint64_t total) {
    int dev = 0, per_sm = 1, sms = 148;
    cudaGetDevice(&dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, 32, kOutSmem);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (per_sm < 1) per_sm = 1;
    uint64_t grid = static_cast<uint64_t>(sms) * per_sm;
    if (grid > total) grid = total;
    return grid ? static_cast<uint32_t>(grid) : 1u;
}

cudaError_t launch_stageout(const StageoutArgs &a, cudaStream_t stream) {
    if (a.n == 0) return cudaSuccess;
    static std::atomic<uint64_t> attr{0};
    cudaError_t e = copy_smem_once(reinterpret_cast<const void *>(stageout_kernel), attr);
    if (e != cudaSuccess) return e;
    const uint32_t pieces = (a.block_tokens * (a.row_bytes_k > a.row_bytes_v ? a.row_bytes_k : a.row_bytes_v) +
                             kPiece - 1u) / kPiece;
    const uint64_t total = static_cast<uint64_t>(a.n) * a.n_layer * 2u * pieces;
    stageout_kernel<<<copy_grid(reinterpret_cast<const void *>(stageout_kernel), total), 32, kOutSmem, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_packed_stagein(const PackedInArgs &a, cudaStream_t stream) {
    static std::atomic<uint64_t> attr{0};
    cudaError_t e = copy_smem_once(reinterpret_cast<const void *>(packed_stagein_kernel), attr);
    if (e != cudaSuccess) return e;
    const uint32_t pieces = (a.block_tokens * (a.row_bytes_k > a.row_bytes_v ? a.row_bytes_k : a.row_bytes_v) +
                             kPiece - 1u) / kPiece;
    const uint32_t items = a.n_items_dev ? a.max_items : a.n_items_host;
    const uint64_t total = static_cast<uint64_t>(items) * a.n_layer * 2u * pieces;
    if (total == 0) return cudaSuccess;
    packed_stagein_kernel<<<copy_grid(reinterpret_cast<const void *>(packed_stagein_kernel), total), 32, kOutSmem,
                            stream>>>(a);
    return cudaGetLastError();
}

}  // namespace kvm
