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
// on an mbarrier) NSTAGE tiles ahead; the consumer warps quantize the tile
// into a shared-memory output buffer (one thread per ggml block), then the
// elected thread writes the tile's quantized rows (contiguous in the window)
// back with one cp.async.bulk shared->global store.  An input buffer is
// refilled as soon as its tile is consumed; its output buffer is handed back
// to the consumers separately (ofree barrier) once the store has read it, so
// the loads run NSTAGE-1 tiles ahead of the quantizers.  Every wait is bounded.
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
    uint32_t pos0;     // original position of the tile's first row
    bool valid;
};

__device__ __forceinline__ TaskDesc decode_task(const StageinArgs &a, uint64_t t,
                                                uint32_t tiles, uint32_t n_items) {
    TaskDesc d{nullptr, nullptr, 0u, 0u, 0u, false};
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
    d.pos0 = block * a.block_tokens + row0;
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
    uint32_t meta;     // bit 31: V tile; bits 0-30: original position of row 0
};
static_assert(sizeof(TileSlot) == 24, "TileSlot");

// Shared memory: [0,128) barriers (full[NS], done[NS], ofree[NS]); [128,384)
// tile slots; then NS input tiles and NS output tiles.
constexpr uint32_t kStageinHeader = 384;

// ------------------------------------------------------- transform mode --
//
// A lane owns one ggml block -- 32 consecutive values of one head of one row
// -- and the head_dim/32 lanes of a (row, head) work together: butterflies of
// span < 32 stay in the lane's registers, larger spans pair lanes (xor of the
// lane index), and each lane quantizes its own block in the reference's
// sequential order.  Every float operation is a round-to-nearest intrinsic,
// so the Hadamard and the quantizers match the CPU bit for bit; RoPE calls the
// CUDA sincosf (as the reference's GPU kernel does) and agrees with the host
// cosf / sinf to within their last-bit errors.

// One 32-value block from F32 values, the reference's loops in their order
// (quant_q8_0 / quant_q4_0, llama-kvmem-stagein.cu:180-233; q5_0 as ggml).
__device__ __forceinline__ void quant_f32_block(int type, const float (&v)[32], uint8_t *blk) {
    if (type == KVM_TYPE_F16) {
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
            *reinterpret_cast<uint32_t *>(blk + 2 * j) = f16_bits(v[j]) | (f16_bits(v[j + 1]) << 16);
        }
        return;
    }
    if (type == KVM_TYPE_Q8_0) {
        float amax = 0.0f;
#pragma unroll
        for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(v[j]));
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        st_u16(blk, f16_bits(d));
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
            const uint32_t q0 = static_cast<uint32_t>(round_half_away(__fmul_rn(v[j], id))) & 0xffu;
            const uint32_t q1 = static_cast<uint32_t>(round_half_away(__fmul_rn(v[j + 1], id))) & 0xffu;
            st_u16(blk + 2 + j, q0 | (q1 << 8));
        }
        return;
    }
    const bool q5 = type == KVM_TYPE_Q5_0;
    float amax = 0.0f, vmax = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        const float m = fabsf(v[j]);
        if (amax < m) {
            amax = m;
            vmax = v[j];
        }
    }
    const float d = __fdiv_rn(vmax, q5 ? -16.0f : -8.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    const float off = q5 ? 16.5f : 8.5f;
    const int maxq = q5 ? 31 : 15;
    st_u16(blk, f16_bits(d));
    uint32_t qh = 0;
    uint8_t *qs = blk + (q5 ? 6 : 2);
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
        const uint32_t a0 = code_q(v[j], id, off, maxq), b0 = code_q(v[j + 16], id, off, maxq);
        const uint32_t a1 = code_q(v[j + 1], id, off, maxq), b1 = code_q(v[j + 17], id, off, maxq);
        qh |= ((a0 >> 4) << j) | ((a1 >> 4) << (j + 1)) | ((b0 >> 4) << (j + 16)) | ((b1 >> 4) << (j + 17));
        st_u16(qs + j, ((a0 & 15u) | ((b0 & 15u) << 4)) | (((a1 & 15u) | ((b1 & 15u) << 4)) << 8));
    }
    if (q5) {
        st_u16(blk + 2, qh & 0xffffu);
        st_u16(blk + 4, qh >> 16);
    }
}

// 32 consecutive F16 values of a tile row, widened.
__device__ __forceinline__ void load32(const __half *p, float (&v)[32]) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint4 r = *reinterpret_cast<const uint4 *>(p + 8 * c);
        const __half2 *h = reinterpret_cast<const __half2 *>(&r);
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            const float2 f = __half22float2(h[m]);
            v[8 * c + 2 * m] = f.x;
            v[8 * c + 2 * m + 1] = f.y;
        }
    }
}

__device__ __forceinline__ void transform_tile(const StageinArgs &a, const TileSlot &ts, const uint8_t *ib,
                                               uint8_t *ob, int warp, int lane) {
    const bool is_v = (ts.meta >> 31) != 0u;
    const uint32_t pos0 = ts.meta & 0x7fffffffu;
    const uint32_t nrot = is_v ? a.rot_v : a.rot_k;
    const uint32_t n_rope = is_v ? 0u : a.rope_n_rot;
    const uint32_t half = n_rope / 2u;
    const uint32_t G = a.xform;                    // lanes per (row, head) = head_dim / 32
    const uint32_t D = G * 32u;
    const uint32_t per_warp = 32u / G;
    const uint32_t H = a.n_embd / D;
    const uint32_t rb = is_v ? a.row_bytes_v : a.row_bytes_k;
    const uint32_t bb = static_cast<uint32_t>(block_bytes(ts.type));
    const float scale = nrot ? __fdiv_rn(1.0f, __fsqrt_rn(__uint2float_rn(nrot))) : 1.0f;
    const uint32_t sub = static_cast<uint32_t>(lane) / G;
    const uint32_t j = static_cast<uint32_t>(lane) - sub * G;
    const uint32_t units = ts.rows * H;
    for (uint32_t u0 = static_cast<uint32_t>(warp) * per_warp; u0 < units;
         u0 += kStageinConsumerWarps * per_warp) {
        const uint32_t u = u0 + sub;
        const bool valid = sub < per_warp && u < units;
        const uint32_t row = valid ? u / H : 0u;
        const uint32_t h = valid ? u - row * H : 0u;
        float v[32];
        if (valid) {
            const __half *x = reinterpret_cast<const __half *>(ib + static_cast<size_t>(row) * a.n_embd * 2u) + h * D;
            load32(x + 32u * j, v);
            const uint32_t i0 = 32u * j;
            if (i0 < n_rope) {
                // rope_neox: (x0, x1) = (v[i], v[i + half]) turned by pos * theta[i]
                const bool lo = i0 < half;
                float w[32];
                load32(x + (lo ? i0 + half : i0 - half), w);
                const float pos = __uint2float_rn(pos0 + row);
                const float *th = a.theta + (lo ? i0 : i0 - half);
#pragma unroll
                for (int m = 0; m < 32; ++m) {
                    float sn, cs;
                    sincosf(__fmul_rn(pos, th[m]), &sn, &cs);
                    v[m] = lo ? __fsub_rn(__fmul_rn(v[m], cs), __fmul_rn(w[m], sn))
                              : __fadd_rn(__fmul_rn(w[m], sn), __fmul_rn(v[m], cs));
                }
            }
        } else {
#pragma unroll
            for (int m = 0; m < 32; ++m) v[m] = 0.0f;
        }
        if (nrot) {
#pragma unroll
            for (int m = 0; m < 32; ++m) v[m] = __fmul_rn(v[m], scale);
            // spans 1 .. 16 inside the lane (fwht_kernel's h loop, ascending)
#pragma unroll
            for (int hh = 1; hh < 32; hh <<= 1) {
#pragma unroll
                for (int m = 0; m < 32; ++m) {
                    if ((m & hh) == 0) {
                        const float p = v[m];
                        const float q = v[m | hh];
                        v[m] = __fadd_rn(p, q);
                        v[m | hh] = __fsub_rn(p, q);
                    }
                }
            }
            // spans 32 .. nrot/2: lane j pairs with lane j ^ (span / 32).  The
            // lower lane keeps v + p, the upper p - v: fma(+-1, v, p) forms
            // p +- v exactly before its one rounding, the same value as the
            // add or the subtraction, in one instruction.
            for (uint32_t dl = 1; 32u * dl < nrot; dl <<= 1) {
                const float sgn = (j & dl) != 0u ? -1.0f : 1.0f;
#pragma unroll
                for (int m = 0; m < 32; ++m) {
                    const float p = __shfl_xor_sync(0xffffffffu, v[m], static_cast<int>(dl));
                    v[m] = __fmaf_rn(sgn, v[m], p);
                }
            }
        }
        if (valid)
            quant_f32_block(ts.type, v, ob + static_cast<size_t>(row) * rb + static_cast<size_t>(h * G + j) * bb);
    }
}

// Resident CTAs per SM: three for the plain kernel (its shared memory allows
// three; at most 75 registers a thread), two for the transform variant (16
// consumer warps to hide its ALU latencies).
template <int NS, bool XF>
__global__ void __launch_bounds__(kStageinThreads, XF ? 2 : 3) stagein_kernel(StageinArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *done = full + NS;
    uint64_t *ofree = done + NS;   // phase k of ofree[s]: the store of tile s + k*NS has read out[s]
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
            mbar_init(&ofree[s], 1);
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
                ts.meta = (d.pos0 & 0x7fffffffu) | (d.kv ? 0x80000000u : 0u);
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
                if (lane == 0) mbar_arrive(&ofree[s]);
            }
            if (lane == 0) {
                // the consumers are done with in[s]: refill it right away; the
                // output buffer is released separately through ofree[]
                if (!ended) arm_next();
                if (a.bulk_store && j >= 1) {
                    bulk_wait_read<1>();                  // the store of tile j - 1 has read its buffer
                    mbar_arrive(&ofree[(j - 1) % NS]);
                }
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
        // out[s] was last written for tile j - NS: its store must have read it
        if (j >= static_cast<uint32_t>(NS) && !mbar_wait_bounded(&ofree[s], ((j / NS) - 1u) & 1u)) {
            set_status(a.status, kErrTimeout);
            break;
        }
        const uint8_t *ib = in_buf + s * a.tile_in_bytes;
        uint8_t *ob = out_buf + s * a.tile_out_bytes;
        if (XF) {
            const bool is_v = (ts.meta >> 31) != 0u;
            if (is_v ? a.rot_v != 0u : (a.rot_k != 0u || a.rope_n_rot != 0u)) {
                transform_tile(a, ts, ib, ob, warp, lane);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&done[s]);
                continue;
            }
        }
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

__global__ void __launch_bounds__(kPermuteThreads) permute_kernel(PermuteArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t n_moves = min(*a.n_moves_dev, a.max_moves);
    if (n_moves == 0) return;
    MoveMeta *meta = reinterpret_cast<MoveMeta *>(smem);
    uint8_t *col = smem + permute_meta_bytes(a.max_moves);
    // The column width follows the actual move count: the widest column (a
    // multiple of 16 bytes, at most col_bytes) whose copy for every moving
    // block fits the shared-memory region.  Every CTA computes the same width.
    uint32_t cw = (a.col_region / n_moves) & ~15u;
    if (cw > a.col_bytes) cw = a.col_bytes;
    if (cw < 16u) cw = 16u;
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
    const uint32_t n_cols_k = (a.span_k + cw - 1) / cw;
    const uint32_t n_cols_v = (a.span_v + cw - 1) / cw;
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
            permute_column<uint4>(meta, col, n_moves, cw, base, span, rb, c * cw);
        else
            permute_column<uint16_t>(meta, col, n_moves, cw, base, span, rb, c * cw);
    }
}

// ------------------------------------------------------------- launchers --

// SM count of the current device (cached per host thread and device).
static int num_sms() {
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

template <bool XF>
static cudaError_t launch_stagein_t(const StageinArgs &a, cudaStream_t stream, uint32_t grid_cap,
                                    std::atomic<uint64_t> &attr) {
    const size_t smem = stagein_smem_bytes(a);
    if (smem > 200u * 1024u) return cudaErrorInvalidValue;
    const void *fn = reinterpret_cast<const void *>(stagein_kernel<kStageinStages, XF>);
    if (!attr_once(attr, fn, 200 * 1024)) return cudaErrorInvalidValue;
    int per_sm = 1;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, stagein_kernel<kStageinStages, XF>,
                                                  kStageinThreads, smem);
    if (per_sm < 1) per_sm = 1;
    uint32_t grid = static_cast<uint32_t>(num_sms() * per_sm);
    if (grid_cap && grid > grid_cap) grid = grid_cap;
    if (grid == 0) grid = 1;
    stagein_kernel<kStageinStages, XF><<<grid, kStageinThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

static std::atomic<uint64_t> g_xform_attr{0};

cudaError_t launch_stagein(const StageinArgs &a, cudaStream_t stream, uint32_t grid_cap) {
    if (a.xform == 0) return launch_stagein_t<false>(a, stream, grid_cap, g_stagein_attr);
    // lanes of a (row, head) must tile the warp's xor pairs: head_dim / 32 in
    // 1 .. 32 and, for every Hadamard size, a multiple of size / 32
    if (a.xform > 32u || (a.rot_k && a.xform % (a.rot_k / 32u)) || (a.rot_v && a.xform % (a.rot_v / 32u)))
        return cudaErrorInvalidValue;
    return launch_stagein_t<true>(a, stream, grid_cap, g_xform_attr);
}

cudaError_t launch_permute(const PermuteArgs &a, cudaStream_t stream) {
    const size_t smem = permute_meta_bytes(a.max_moves) + a.col_region;
    if (smem > 200u * 1024u || a.col_region < 16u * a.max_moves) return cudaErrorInvalidValue;
    if (!attr_once(g_permute_attr, reinterpret_cast<const void *>(permute_kernel), 200 * 1024))
        return cudaErrorInvalidValue;
    const uint32_t grid = static_cast<uint32_t>(num_sms() * 2);
    permute_kernel<<<grid, kPermuteThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace kvm
