// kvm_stagein.cu -- fused gather + quantize stage-in.
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
// to the consumers separately (ofree barrier) as soon as the store has read
// it, so the loads run NSTAGE-1 tiles ahead of the quantizers.  The RoPE
// transform kernel has no output buffers: its consumers store the window
// from registers.  Every wait is bounded.

#include "kvm_internal.cuh"
#include "kvm_quant.cuh"
#include "kvm_kernels.h"

#include <atomic>
#include <cmath>

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

// Task t of a launch is (item, layer, K|V, tile), tile fastest.  Its three
// divisions run as multiply-highs (FastDiv) when total * per_item <= 2^32:
// every dividend times its divisor is then within the bound.
struct TaskIndex {
    FastDiv per_item, per_layer, tiles;
    bool magic;
};

__device__ __forceinline__ TaskIndex make_task_index(const StageinArgs &a, uint32_t tiles, uint64_t total) {
    const uint32_t per_layer = a.n_kv * tiles;
    const uint32_t per_item = a.n_layer * per_layer;
    TaskIndex ti;
    ti.per_item = make_fastdiv(per_item);
    ti.per_layer = make_fastdiv(per_layer);
    ti.tiles = make_fastdiv(tiles);
    ti.magic = total < (1ull << 32) && total * per_item <= (1ull << 32);
    return ti;
}

__device__ __forceinline__ TaskDesc decode_task(const StageinArgs &a, uint64_t t, const TaskIndex &ti,
                                                uint32_t n_items) {
    TaskDesc d{nullptr, nullptr, 0u, 0u, 0u, false};
    uint32_t item, layer, kv, tile;
    if (ti.magic) {
        const uint32_t t32 = static_cast<uint32_t>(t);
        item = fast_div(t32, ti.per_item);
        uint32_t r = t32 - item * ti.per_item.d;
        layer = fast_div(r, ti.per_layer);
        r -= layer * ti.per_layer.d;
        kv = fast_div(r, ti.tiles);
        tile = r - kv * ti.tiles.d;
    } else {
        item = static_cast<uint32_t>(t / ti.per_item.d);
        uint32_t r = static_cast<uint32_t>(t % ti.per_item.d);
        layer = r / ti.per_layer.d;
        r %= ti.per_layer.d;
        kv = r / ti.tiles.d;
        tile = r % ti.tiles.d;
    }
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

// Shared memory: [0,192) barriers (full[NS], done[NS], ofree[NO]); [192,512)
// tile slots; then NS input tiles and, except in the RoPE kernel (which
// stores the window from registers), NS output tiles.
constexpr uint32_t kStageinBarBytes = 192;
constexpr uint32_t kStageinHeader = 512;

// Shared-memory copy of the RoPE frequencies (transform mode), between the
// header and the tiles; a multiple of 128 bytes so the tiles stay aligned.
__host__ __device__ inline uint32_t stagein_theta_bytes(const StageinArgs &a) {
    return (a.xform && a.rope_n_rot) ? ((a.rope_n_rot / 2u) * 4u + 127u) & ~127u : 0u;
}

// RoPE angle table of one consumer warp (transform mode with RoPE): the
// (cos, sin) of every (row, frequency) its warp-iteration needs -- the rows
// of its (row, head) units x rope_n_rot / 2 frequencies -- each computed once
// and read by the lanes of every head and of both rotation halves.  Row r,
// frequency i at float2 index r * stride + i + 2 * (i / 32): 16 bytes of
// padding per 32 entries keep the four 256-byte lane segments of one read on
// different banks.
__host__ __device__ inline uint32_t rope_tab_rows(const StageinArgs &a) {
    const uint32_t per_warp = 32u / (a.xform ? a.xform : 1u);
    const uint32_t h = a.xf_heads ? a.xf_heads : 1u;
    const uint32_t r = (per_warp - 1u) / h + 2u;        // rows a warp-iteration can touch
    return r < per_warp ? r : per_warp;
}
__host__ __device__ inline uint32_t rope_tab_stride(const StageinArgs &a) {   // float2 entries a row
    const uint32_t half = a.rope_n_rot / 2u;
    return half + 2u * (half / 32u);
}
__host__ __device__ inline uint32_t rope_tab_warp_bytes(const StageinArgs &a) {
    return (a.xform && a.rope_n_rot) ? ((rope_tab_rows(a) * rope_tab_stride(a) * 8u + 127u) & ~127u) : 0u;
}

// Pipeline depth (measured at config 2): attn_rot at four CTAs an SM fits
// two stages; the RoPE kernel's stages hold no output tile.
__host__ __device__ inline int stagein_stages(const StageinArgs &a) {
    return !a.xform ? kStageinStages : (a.rope_n_rot ? kXfRopeStages : kXfStages);
}

// Output tiles in shared memory: none for the RoPE kernel (it stores from
// registers), kXfOutStages for attn_rot, one per stage otherwise.
__host__ __device__ inline int stagein_out_stages(const StageinArgs &a) {
    return !a.xform ? kStageinStages : (a.rope_n_rot ? 0 : kXfOutStages);
}

// Consumer warps of a launch (see stagein_kernel).
__host__ __device__ inline int stagein_consumer_warps(const StageinArgs &a) {
    return !a.xform ? kStageinConsumerWarps : (a.rope_n_rot ? kXfRopeWarps : kXfConsumerWarps);
}

// ------------------------------------------------------- transform mode --
//
// A lane owns one ggml block -- 32 consecutive values of one head of one row
// -- and the head_dim/32 lanes of a (row, head) work together: butterflies of
// span < 32 stay in the lane's registers, larger spans pair lanes (xor of the
// lane index), and each lane quantizes its own block in the reference's
// order.  The lane keeps its values as 16 float pairs, P[k] = (v[2k],
// v[2k+1]), so that all butterflies of span >= 2, the cross-lane stages and
// the quantizer's adds run on sm_100's packed FP32x2 instructions (f2_add_rn,
// f2_fma_rn: per component the same IEEE operation as the scalar one).  Every
// product that an add consumes is a scalar __fmul_rn, so its rounding stays.
// Every float operation rounds to nearest, so the Hadamard and the
// quantizers match the CPU bit for bit.  RoPE turns each pair by the sin and
// cos of the same float angle as the reference (pos * theta, rounded), from
// rope_sincos, and agrees with the host cosf / sinf to within their last-bit
// errors.
//
// The Hadamard's scale 1/sqrt(n) is a power of two when log2(n) is even (64,
// 256, 1024).  Multiplying by a power of two then commutes exactly with every
// butterfly (F16 inputs keep all sums far above the F32 subnormal range), so
// without RoPE the transform runs unscaled and the quantizer takes the scale
// into amax and id: amax*s and id*s are exact, and x*(id*s) is the same real
// product as (x*s)*id, rounded once.

// The 4 low bytes of q0..q3 as one word (byte i = q_i).
__device__ __forceinline__ uint32_t pack4(int q0, int q1, int q2, int q3) {
    return __byte_perm(__byte_perm(static_cast<uint32_t>(q0), static_cast<uint32_t>(q1), 0x0040u),
                       __byte_perm(static_cast<uint32_t>(q2), static_cast<uint32_t>(q3), 0x0040u), 0x5410u);
}

__device__ __forceinline__ float2 splat2(float x) { return make_float2(x, x); }

// C roundf of both components, as integers (|x| < 2^23).  y must come from
// a rounded product (scalar __fmul_rn), never from a packed multiply.
__device__ __forceinline__ void round_half_away2(float2 y, int &q0, int &q1) {
    const float2 t = f2_add_rn(y, make_float2(copysignf(0x1.fffffep-2f, y.x), copysignf(0x1.fffffep-2f, y.y)));
    q0 = __float2int_rz(t.x);
    q1 = __float2int_rz(t.y);
}

// q8_0 of the lane's 32 values scaled by fs (a power of two; 1 when the scale
// was applied already): quant_q8_0 (llama-kvmem-stagein.cu:180-200).  The
// running fmaxf of the reference is split over four accumulators: max is
// exact and fmaxf ignores NaN in any order, so the result is the same.
__device__ __forceinline__ void quant_q8_pairs(const float2 (&P)[16], float fs, uint8_t *blk) {
    float m0 = 0.0f, m1 = 0.0f, m2 = 0.0f, m3 = 0.0f;
#pragma unroll
    for (int k = 0; k < 16; k += 2) {
        m0 = fmaxf(m0, fabsf(P[k].x));
        m1 = fmaxf(m1, fabsf(P[k].y));
        m2 = fmaxf(m2, fabsf(P[k + 1].x));
        m3 = fmaxf(m3, fabsf(P[k + 1].y));
    }
    const float amax = __fmul_rn(fmaxf(fmaxf(m0, m1), fmaxf(m2, m3)), fs);
    const float d = div127(amax);
    const float id = d != 0.0f ? __fmul_rn(__frcp_rn(d), fs) : 0.0f;
    uint32_t w[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        int q0, q1, q2, q3;
        round_half_away2(make_float2(__fmul_rn(P[2 * k].x, id), __fmul_rn(P[2 * k].y, id)), q0, q1);
        round_half_away2(make_float2(__fmul_rn(P[2 * k + 1].x, id), __fmul_rn(P[2 * k + 1].y, id)), q2, q3);
        w[k] = pack4(q0, q1, q2, q3);
    }
    store_block<8>(blk, f16_bits(d), w);
}

// q4_0 / q5_0 of the lane's 32 values scaled by fs (quant_q4_0,
// llama-kvmem-stagein.cu:202-233; q5_0 as ggml).  vmax -- the first value of
// largest magnitude -- comes from the signed max and min; only a +a / -a tie
// needs the first occurrence.
template <bool Q5>
__device__ __forceinline__ void quant_q4q5_pairs(const float2 (&P)[16], float fs, uint8_t *blk) {
    float hx = P[0].x, hy = P[0].y, lx = P[0].x, ly = P[0].y;
#pragma unroll
    for (int k = 1; k < 16; ++k) {
        hx = fmaxf(hx, P[k].x);
        hy = fmaxf(hy, P[k].y);
        lx = fminf(lx, P[k].x);
        ly = fminf(ly, P[k].y);
    }
    const float hi = fmaxf(hx, hy), lo = fminf(lx, ly);
    const float amax = fmaxf(hi, -lo);
    float vmax = 0.0f;
    if (amax > 0.0f) {
        if (hi != -lo) {
            vmax = hi > -lo ? hi : lo;
        } else {
            // first value (block order) with |v| == amax
            for (int m = 31; m >= 0; --m) {
                const float x = (m & 1) ? P[m >> 1].y : P[m >> 1].x;
                vmax = fabsf(x) == amax ? x : vmax;
            }
        }
    }
    const float d = __fmul_rn(__fmul_rn(vmax, fs), Q5 ? -0.0625f : -0.125f);
    const float id = d != 0.0f ? __fmul_rn(__frcp_rn(d), fs) : 0.0f;
    const float2 off = splat2(Q5 ? 16.5f : 8.5f);
    uint32_t c[8];   // byte codes: word k holds values 4k .. 4k+3
#pragma unroll
    for (int k = 0; k < 8; ++k)
        c[k] = codes4<Q5 ? 31 : 15>(mul_add_off(P[2 * k], id, off), mul_add_off(P[2 * k + 1], id, off));
    // byte j of the nibbles: value j on the low nibble, value j + 16 on the high
    constexpr int NW = Q5 ? 5 : 4;
    uint32_t w[NW];
#pragma unroll
    for (int k = 0; k < 4; ++k) w[NW - 4 + k] = (c[k] & 0x0f0f0f0fu) | ((c[k + 4] << 4) & 0xf0f0f0f0u);
    if (Q5) {
        w[0] = top_bytes4(high_bits8(c[0], c[1]), high_bits8(c[2], c[3]), high_bits8(c[4], c[5]),
                          high_bits8(c[6], c[7]));
    }
    store_block<NW>(blk, f16_bits(d), w);
}

// The lane's block as ggml F16 (no header), scaled by fs.
__device__ __forceinline__ void store_f16_pairs(const float2 (&P)[16], float fs, uint8_t *blk) {
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        const float2 x = f2_mul_rn(P[k], splat2(fs));
        st_u16(blk + 4 * k, f16_bits(x.x));
        st_u16(blk + 4 * k + 2, f16_bits(x.y));
    }
}

// 32 consecutive F16 values of a tile row (64 bytes), widened.  The four
// 16-byte chunks are read in the order k ^ r, r = (lane >> 1) & 1, so that a
// quarter warp reading 8 neighbouring blocks spreads over 4 bank groups (two
// lanes a group instead of four), then put back in order with one
// conditional swap.  Rotating over all four chunks removes the last 2-way
// conflict but costs a second swap, which measured slower.
__device__ __forceinline__ void load32(const __half *p, int lane, float2 (&P)[16]) {
    const uint32_t r = static_cast<uint32_t>(lane >> 1) & 1u;
    uint4 c[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) c[k] = *reinterpret_cast<const uint4 *>(p + 8u * (static_cast<uint32_t>(k) ^ r));
    // c[k] = chunk k ^ r
#pragma unroll
    for (int k = 0; k < 4; k += 2) {
        const uint4 a = c[k], b = c[k + 1];
        c[k] = r ? b : a;
        c[k + 1] = r ? a : b;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const __half2 *h = reinterpret_cast<const __half2 *>(&c[k]);
#pragma unroll
        for (int m = 0; m < 4; ++m) P[4 * k + m] = __half22float2(h[m]);
    }
}

// Butterflies of span 1 .. 16 inside the lane (fwht_kernel's h loop,
// ascending): span 1 inside each pair, spans 2 .. 16 between pairs k and
// k + h/2.  fma(b, -1, a) is a - b with one rounding.
__device__ __forceinline__ void fwht32_in_lane(float2 (&P)[16]) {
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        const float x = P[k].x, y = P[k].y;
        P[k] = make_float2(__fadd_rn(x, y), __fsub_rn(x, y));
    }
    const float2 neg = splat2(-1.0f);
#pragma unroll
    for (int hp = 1; hp < 16; hp <<= 1) {
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            if ((k & hp) == 0) {
                const float2 a = P[k], b = P[k | hp];
                P[k] = f2_add_rn(a, b);
                P[k | hp] = f2_fma_rn(b, neg, a);
            }
        }
    }
}

// Butterflies of span 32 << t: lane j pairs with lane j ^ (1 << t).  The lower
// lane keeps v + p, the upper p - v: fma(+-1, v, p) forms p +- v exactly
// before its one rounding.
__device__ __forceinline__ void fwht_cross_stage(float2 (&P)[16], uint32_t j, uint32_t dl) {
    const float2 sgn = splat2((j & dl) != 0u ? -1.0f : 1.0f);
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        // one 64-bit shuffle keeps the pair in a register pair
        const unsigned long long b = __shfl_xor_sync(
            0xffffffffu,
            (static_cast<unsigned long long>(__float_as_uint(P[k].y)) << 32) | __float_as_uint(P[k].x),
            static_cast<int>(dl));
        const float2 p = make_float2(__uint_as_float(static_cast<uint32_t>(b)),
                                     __uint_as_float(static_cast<uint32_t>(b >> 32)));
        P[k] = f2_fma_rn(sgn, P[k], p);
    }
}

// sin and cos of a RoPE angle x (a float, |x| < 2^31), each within 2 ulp of
// the true value -- the bound CUDA documents for sinf / cosf -- with no slow
// path for large angles, so every lane runs the same instructions.  The
// reduction by pi/2 follows Cody and Waite (W. J. Cody, W. Waite, "Software
// Manual for the Elementary Functions", 1980) in double precision: x is exact
// as a double, k = rint(x * 2/pi), and r = x - k*pi/2 with pi/2 split into
// two doubles P1 + P2 (together within 2^-107 of pi/2) through two FMAs, so r
// is good to about 2^-53 absolute for every such x.  sin r and cos r (|r| at
// most pi/4 and a rounding) are Taylor polynomials of degree 9 and 10 in
// single precision (truncation below 2e-9 and 2e-10), and k mod 4 picks the
// quadrant: x = k*pi/2 + r.
__device__ __forceinline__ void rope_sincos(float x, float *sn, float *cs) {
    const double xd = static_cast<double>(x);
    const double k = rint(xd * 0x1.45f306dc9c883p-1);                              // 2/pi
    const double rd = fma(-k, 0x1.1a62633145c07p-54, fma(-k, 0x1.921fb54442d18p+0, xd));   // P2, P1
    const float r = __double2float_rn(rd);
    const float r2 = __fmul_rn(r, r);
    float ps = fmaf(r2, 1.0f / 362880.0f, -1.0f / 5040.0f);
    ps = fmaf(ps, r2, 1.0f / 120.0f);
    ps = fmaf(ps, r2, -1.0f / 6.0f);
    const float s = fmaf(ps, __fmul_rn(r2, r), r);
    float pc = fmaf(r2, -1.0f / 3628800.0f, 1.0f / 40320.0f);
    pc = fmaf(pc, r2, -1.0f / 720.0f);
    pc = fmaf(pc, r2, 1.0f / 24.0f);
    pc = fmaf(pc, r2, -0.5f);
    const float c = fmaf(pc, r2, 1.0f);
    const int q = static_cast<int>(static_cast<long long>(k)) & 3;
    const float s1 = (q & 1) ? c : s;              // sin(r + pi/2) = cos r, cos(r + pi/2) = -sin r
    const float c1 = (q & 1) ? s : c;
    *sn = (q & 2) ? -s1 : s1;
    *cs = ((q + 1) & 2) ? -c1 : c1;
}

// (sub, j): the lane's unit within the warp and its block within the head;
// per_warp = 32 / xform units a warp-iteration.
template <int CW, bool ROPE>
__device__ __forceinline__ void transform_tile(const StageinArgs &a, const TileSlot &ts, const uint8_t *ib,
                                               uint8_t *ob, int warp, int lane, uint32_t sub, uint32_t j,
                                               uint32_t per_warp, const float *theta_s, float2 *tab) {
    const bool is_v = (ts.meta >> 31) != 0u;
    const uint32_t pos0 = ts.meta & 0x7fffffffu;
    const uint32_t nrot = is_v ? a.rot_v : a.rot_k;
    const uint32_t n_rope = is_v ? 0u : a.rope_n_rot;
    const uint32_t half = n_rope / 2u;
    const uint32_t G = a.xform;                    // lanes per (row, head) = head_dim / 32
    const uint32_t D = G * 32u;
    const uint32_t H = a.xf_heads;
    const uint32_t rb = is_v ? a.row_bytes_v : a.row_bytes_k;
    const uint32_t bb = static_cast<uint32_t>(block_bytes(ts.type));
    const float pre = is_v ? a.xf_pre_v : a.xf_pre_k;
    const float fs = is_v ? a.xf_post_v : a.xf_post_k;
    const uint32_t units = ts.rows * H;
    const uint32_t tstride = rope_tab_stride(a);
    for (uint32_t u0 = static_cast<uint32_t>(warp) * per_warp; u0 < units;
         u0 += CW * per_warp) {
        const uint32_t u = u0 + sub;
        const bool valid = sub < per_warp && u < units;
        const uint32_t row = !valid ? 0u : (H == 1u ? u : __umulhi(u, a.xf_heads_magic));
        const uint32_t h = valid ? u - row * H : 0u;
        // RoPE: the (cos, sin) of this warp-iteration's rows, each angle once
        const uint32_t r0 = H == 1u ? u0 : __umulhi(u0, a.xf_heads_magic);
        if (ROPE && n_rope) {
            const uint32_t ul = min(units, u0 + per_warp) - 1u;
            const uint32_t nr = (H == 1u ? ul : __umulhi(ul, a.xf_heads_magic)) - r0 + 1u;
            __syncwarp();                      // the previous iteration's reads are done
            for (uint32_t rr = 0; rr < nr; ++rr) {
                const float pos = __uint2float_rn(pos0 + r0 + rr);
                for (uint32_t i = static_cast<uint32_t>(lane); i < half; i += 32u) {
                    float sn, cs;
                    rope_sincos(__fmul_rn(pos, theta_s[i]), &sn, &cs);
                    tab[rr * tstride + i + 2u * (i / 32u)] = make_float2(cs, sn);
                }
            }
            __syncwarp();
        }
        float2 P[16];
        const __half *x = reinterpret_cast<const __half *>(ib + static_cast<size_t>(row) * a.n_embd * 2u) + h * D;
        // a lane past the last unit reads row 0 and stores nothing; the lanes
        // of one unit share validity, so its values never reach a valid lane
        load32(x + 32u * j, lane, P);
        const uint32_t i0 = 32u * j;
        if (ROPE && valid && i0 < n_rope) {
            // rope_neox: (x0, x1) = (v[i], v[i + half]) turned by pos * theta[i]
            // (cos, sin from the table); the partner half is read 8 values at a time
            const bool lo = i0 < half;
            const __half *xp = x + (lo ? i0 + half : i0 - half);
            const uint32_t ti = lo ? i0 : i0 - half;            // a multiple of 32
            const float4 *tr = reinterpret_cast<const float4 *>(tab + (row - r0) * tstride + ti + 2u * (ti / 32u));
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint4 raw = *reinterpret_cast<const uint4 *>(xp + 8 * c);
                const __half2 *hw = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
                for (int m2 = 0; m2 < 4; ++m2) {
                    const float4 t2 = tr[4 * c + m2];           // (cos, sin) of values 8c+2m2, +1
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int m = 2 * m2 + e;
                        const float cs = e ? t2.z : t2.x;
                        const float sn = e ? t2.w : t2.y;
                        float &v = e ? P[4 * c + m2].y : P[4 * c + m2].x;
                        const float w = e ? __high2float(hw[m >> 1]) : __low2float(hw[m >> 1]);
                        v = lo ? __fsub_rn(__fmul_rn(v, cs), __fmul_rn(w, sn))
                               : __fadd_rn(__fmul_rn(w, sn), __fmul_rn(v, cs));
                    }
                }
            }
        }
        if (nrot) {
            if (pre != 1.0f) {
#pragma unroll
                for (int k = 0; k < 16; ++k) P[k] = make_float2(__fmul_rn(P[k].x, pre), __fmul_rn(P[k].y, pre));
            }
            fwht32_in_lane(P);
            for (uint32_t dl = 1; 32u * dl < nrot; dl <<= 1) fwht_cross_stage(P, j, dl);
        }
        if (valid) {
            uint8_t *blk = ob + static_cast<size_t>(row) * rb + static_cast<size_t>(h * G + j) * bb;
            switch (ts.type) {
                case KVM_TYPE_Q8_0: quant_q8_pairs(P, fs, blk); break;
                case KVM_TYPE_Q4_0: quant_q4q5_pairs<false>(P, fs, blk); break;
                case KVM_TYPE_Q5_0: quant_q4q5_pairs<true>(P, fs, blk); break;
                default: store_f16_pairs(P, fs, blk); break;
            }
        }
    }
}

// CW consumer warps + the producer.  Resident CTAs per SM: three for the
// plain kernel (its shared memory allows three; at most 72 registers a
// thread), four for attn_rot (7 consumer warps, at most 64 registers a
// thread: 32 warps an SM measured faster than 24 at 80 registers and 16 at
// 128), two with RoPE (8 consumer warps, 96 registers).
template <int NS, bool XF, int CW, bool ROPE = false>
__global__ void __launch_bounds__(CW * 32 + 32, XF ? (ROPE ? kXfRopeMinBlocks : kXfMinBlocks) : 3) stagein_kernel(StageinArgs a) {
    // RoPE tiles are bound by the angle table and the rotation, not by their stores: that kernel's
    // consumers store the window from registers, which leaves its shared
    // memory to a deeper input pipeline.  The others stage each output tile
    // in shared memory and the producer writes it with one bulk copy.
    constexpr bool DS = XF && ROPE;
    // output tiles: NO of them (tile j uses out[j % NO]), fewer than the input
    // stages where shared memory is short
    constexpr int NO = (XF && !ROPE) ? kXfOutStages : NS;
    static_assert(NO >= 1 && NO <= NS, "output tiles");
    static_assert((2 * NS + NO) * 8 <= kStageinBarBytes && kStageinBarBytes + NS * sizeof(TileSlot) <= kStageinHeader,
                  "stage-in header");
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *done = full + NS;
    uint64_t *ofree = done + NS;   // phase k of ofree[o]: the store of tile o + k*NO has read out[o]
    TileSlot *slot = reinterpret_cast<TileSlot *>(smem + kStageinBarBytes);
    float *theta_s = reinterpret_cast<float *>(smem + kStageinHeader);   // RoPE frequencies
    float2 *rope_tab = reinterpret_cast<float2 *>(smem + kStageinHeader + stagein_theta_bytes(a));
    uint8_t *in_buf = smem + kStageinHeader + stagein_theta_bytes(a) + CW * rope_tab_warp_bytes(a);
    uint8_t *out_buf = in_buf + NS * a.tile_in_bytes;

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    // set-up that needs nothing of the previous launch runs before the wait
    if (XF && ROPE) {
        for (uint32_t i = static_cast<uint32_t>(tid); i < a.rope_n_rot / 2u; i += blockDim.x)
            theta_s[i] = a.theta[i];
    }
    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&done[s], CW);
        }
        for (int o = 0; o < NO; ++o) mbar_init(&ofree[o], 1);
        fence_mbar_init();
    }
    __syncthreads();   // the only CTA-wide barrier
    pdl_wait();        // the plan (cold list and its count) is complete

    const uint32_t n_items_raw = a.n_items_dev ? *a.n_items_dev : a.n_items_host;
    const uint32_t n_items = min(n_items_raw, a.max_items);
    const uint32_t tiles = (a.block_tokens + a.rows_per_tile - 1) / a.rows_per_tile;
    const uint64_t total = static_cast<uint64_t>(n_items) * a.n_layer * a.n_kv * tiles;
    if (static_cast<uint64_t>(blockIdx.x) >= total) return;

    if (warp == CW) {
        // ---------------------------------------------------------- producer
        uint64_t ptask = blockIdx.x;
        uint32_t issued = 0;      // tiles armed with data
        bool ended = false;       // end marker placed
        TaskIndex ti;
        // Arm the stage of tile index `issued` with this CTA's next valid
        // task, or with the end marker when none is left.  Lane 0 only.
        // (Decoding one task ahead, so that a freed stage is refilled without
        // the decode's global reads, measured faster for q4_0/q5_0 windows but
        // slower for q8_0, the HBM-bound case.)
        auto arm_next = [&]() {
            const uint32_t s = issued % NS;
            while (ptask < total) {
                const TaskDesc d = decode_task(a, ptask, ti, n_items);
                ptask += gridDim.x;
                if (!d.valid) continue;
                if (a.test_skip && blockIdx.x == 0 && issued == 0) {
                    ++issued;      // test hook: stage 0 is never armed, its waits run out
                    return;
                }
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
            ti = make_task_index(a, tiles, total);
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
            const uint8_t *ob = out_buf + (j % NO) * a.tile_out_bytes;
            if (DS) {
                // the consumers stored this tile from their registers
            } else if (a.bulk_store) {
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
                if (lane == 0) mbar_arrive(&ofree[j % NO]);
            }
            if (lane == 0) {
                // the consumers are done with in[s]: refill it right away; the
                // output buffer is released separately through ofree[]
                if (!ended) arm_next();
                if (!DS && a.bulk_store) {
                    // release out[j % NO] as soon as the store of tile j has
                    // read it (not one tile later, behind the next done wait)
                    bulk_wait_read<0>();
                    mbar_arrive(&ofree[j % NO]);
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
            if (!DS && a.bulk_store) bulk_wait_all<0>();
        }
        return;
    }

    // ------------------------------------------------------------- consumers
    const uint32_t qb_per_row = a.n_embd / 32u;
    // transform mode: the lane's (unit, block-in-head), fixed for the launch
    const uint32_t xg = (XF && a.xform) ? a.xform : 1u;
    const uint32_t xsub = static_cast<uint32_t>(lane) / xg;
    const uint32_t xj = static_cast<uint32_t>(lane) - xsub * xg;
    const uint32_t xper = 32u / xg;
    for (uint32_t j = 0;; ++j) {
        const uint32_t s = j % NS;
        if (!mbar_wait_bounded(&full[s], (j / NS) & 1u)) {
            set_status(a.status, kErrTimeout);
            break;
        }
        const TileSlot ts = slot[s];
        if (ts.rows == 0) break;
        // out[j % NO] was last written for tile j - NO: its store must have read it
        if (!DS && j >= static_cast<uint32_t>(NO) && !mbar_wait_bounded(&ofree[j % NO], ((j / NO) - 1u) & 1u)) {
            set_status(a.status, kErrTimeout);
            break;
        }
        const uint8_t *ib = in_buf + s * a.tile_in_bytes;
        // direct-store kernels write the window itself (2-byte aligned stores)
        uint8_t *ob = DS ? ts.dst : out_buf + (j % NO) * a.tile_out_bytes;
        if (XF) {
            const bool is_v = (ts.meta >> 31) != 0u;
            if (is_v ? a.rot_v != 0u : (a.rot_k != 0u || a.rope_n_rot != 0u)) {
                transform_tile<CW, ROPE>(a, ts, ib, ob, warp, lane, xsub, xj, xper, theta_s,
                                   rope_tab + warp * (rope_tab_warp_bytes(a) / 8u));
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&done[s]);
                continue;
            }
        }
        const uint32_t nqb = ts.rows * qb_per_row;
        for (uint32_t qb = static_cast<uint32_t>(warp * 32 + lane); qb < nqb;
             qb += CW * 32u) {
            quant_block<!DS>(ts.type, ib, qb, lane, ob);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&done[s]);
    }
}

// ------------------------------------------------------------- launchers --


uint32_t stagein_rows_per_tile(uint32_t n_embd, uint32_t block_tokens) {
    // 16 KiB of F16 per tile (8 rows at n_embd = 1024)
    uint32_t r = 8192u / (n_embd ? n_embd : 1u);
    if (r < 1u) r = 1u;
    if (r > block_tokens) r = block_tokens;
    return r;
}

void stagein_set_transform(StageinArgs &a, uint32_t head_dim, uint32_t n_embd, uint32_t rot_k,
                           uint32_t rot_v, uint32_t rope_n_rot, const float *theta) {
    a.xform = 0;
    a.rot_k = a.rot_v = a.rope_n_rot = 0;
    a.theta = nullptr;
    a.xf_pre_k = a.xf_pre_v = a.xf_post_k = a.xf_post_v = 1.0f;
    a.xf_heads = 1;
    a.xf_heads_magic = 0;
    if (!(rot_k || rot_v || rope_n_rot) || head_dim < 32u) return;
    a.xform = head_dim / 32u;
    a.rot_k = rot_k;
    a.rot_v = rot_v;
    a.rope_n_rot = rope_n_rot;
    a.theta = theta;
    a.xf_heads = n_embd / head_dim;
    a.xf_heads_magic = a.xf_heads > 1u
        ? static_cast<uint32_t>(((1ull << 32) + a.xf_heads - 1u) / a.xf_heads) : 0u;
    // rows a tile such that its (row, head) units fill the consumer warps
    // evenly when the shape allows, within 30 KiB of input + output a stage
    const uint32_t per_warp = 32u / a.xform;
    const uint32_t out_row = a.row_bytes_k > a.row_bytes_v ? a.row_bytes_k : a.row_bytes_v;
    uint32_t r = (static_cast<uint32_t>(stagein_consumer_warps(a)) * per_warp) / (a.xf_heads ? a.xf_heads : 1u);
    if (r < 1u) r = 1u;
    while (r > 1u && r * (n_embd * 2u + out_row) > 30u * 1024u) --r;
    if (r > a.block_tokens) r = a.block_tokens;
    a.rows_per_tile = r;
    a.tile_in_bytes = r * n_embd * 2u;
    a.tile_out_bytes = (r * out_row + 15u) & ~15u;
    // fwht_kernel's scale, 1 / sqrtf(n), in IEEE single precision.  A power
    // of two (log2 n even) folds into the quantizer unless RoPE comes first.
    auto scales = [](uint32_t n, bool rope, float &pre, float &post) {
        pre = post = 1.0f;
        if (!n) return;
        const float sc = 1.0f / std::sqrt(static_cast<float>(n));
        uint32_t lg = 0;
        while ((1u << (lg + 1u)) <= n) ++lg;
        if (!rope && (lg & 1u) == 0u) post = sc;
        else pre = sc;
    };
    scales(rot_k, rope_n_rot != 0u, a.xf_pre_k, a.xf_post_k);
    scales(rot_v, false, a.xf_pre_v, a.xf_post_v);
}

size_t stagein_smem_bytes(const StageinArgs &a) {
    return kStageinHeader + stagein_theta_bytes(a) +
           static_cast<size_t>(stagein_consumer_warps(a)) * rope_tab_warp_bytes(a) +
           static_cast<size_t>(stagein_stages(a)) * a.tile_in_bytes +
           static_cast<size_t>(stagein_out_stages(a)) * a.tile_out_bytes;
}


static std::atomic<uint64_t> g_stagein_attr{0};

template <int NS, bool XF, int CW, bool ROPE>
static cudaError_t launch_stagein_t(const StageinArgs &a, cudaStream_t stream, uint32_t grid_cap,
                                    std::atomic<uint64_t> &attr) {
    const size_t smem = stagein_smem_bytes(a);
    if (smem > 200u * 1024u || stagein_stages(a) != NS || stagein_consumer_warps(a) != CW)
        return cudaErrorInvalidValue;
    const void *fn = reinterpret_cast<const void *>(stagein_kernel<NS, XF, CW, ROPE>);
    if (!attr_once(attr, fn, 200 * 1024)) return cudaErrorInvalidValue;
    int per_sm = 1;
    const int threads = CW * 32 + 32;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, stagein_kernel<NS, XF, CW, ROPE>,
                                                  threads, smem);
    if (per_sm < 1) per_sm = 1;
    uint32_t grid = static_cast<uint32_t>(num_sms() * per_sm);
    if (grid_cap && grid > grid_cap) grid = grid_cap;
    if (grid == 0) grid = 1;
    return launch_after_prev(stagein_kernel<NS, XF, CW, ROPE>, dim3(grid), dim3(threads), smem, stream, a);
}

static std::atomic<uint64_t> g_xform_attr{0};
static std::atomic<uint64_t> g_xform_rope_attr{0};

cudaError_t launch_stagein(const StageinArgs &a, cudaStream_t stream, uint32_t grid_cap) {
    if (a.xform == 0)
        return launch_stagein_t<kStageinStages, false, kStageinConsumerWarps, false>(a, stream, grid_cap, g_stagein_attr);
    // lanes of a (row, head) must tile the warp's xor pairs: head_dim / 32 in
    // 1 .. 32 and, for every Hadamard size, a multiple of size / 32
    if (a.xform > 32u || (a.rot_k && a.xform % (a.rot_k / 32u)) || (a.rot_v && a.xform % (a.rot_v / 32u)))
        return cudaErrorInvalidValue;
    if (a.rope_n_rot)
        return launch_stagein_t<kXfRopeStages, true, kXfRopeWarps, true>(a, stream, grid_cap, g_xform_rope_attr);
    return launch_stagein_t<kXfStages, true, kXfConsumerWarps, false>(a, stream, grid_cap, g_xform_attr);
}

}  // namespace kvm
