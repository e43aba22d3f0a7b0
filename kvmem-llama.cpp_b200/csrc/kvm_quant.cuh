// kvm_quant.cuh -- ggml q8_0 / q4_0 / q5_0 block quantizers, one thread per
// 32-value block.
//
// The arithmetic is the reference's (src/adapter/llama-kvmem-stagein.cu:180-233,
// ggml's quantize_row_*_ref):
//   q8_0: d = amax/127, id = d ? 1/d : 0, q = roundf(x*id)
//   q4_0: vmax = first value of largest |x|, d = vmax/-8, q = min(15, (int)(x*id + 8.5))
//   q5_0: d = vmax/-16, q = min(31, (int)(x*id + 16.5)), bit 4 of q_i -> bit i of qh
// Every float operation is an IEEE round-to-nearest intrinsic (no FMA
// contraction, no approximate reciprocal), so the bytes match the CPU bit for
// bit.
//
// Data arrive as four 16-byte chunks (8 halves each).  A lane loads the
// chunks of its block in a lane-dependent order (Block32) so that the
// 128-bit shared-memory loads of a quarter warp spread over the banks; the
// chunk index is then only used as an output offset -- the max is
// order-free and each value is coded independently.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace kvm {

constexpr int kBlockBytesQ8 = 34;
constexpr int kBlockBytesQ4 = 18;
constexpr int kBlockBytesQ5 = 22;

__host__ __device__ constexpr int block_bytes(int type) {
    return type == KVM_TYPE_Q8_0 ? kBlockBytesQ8
         : type == KVM_TYPE_Q4_0 ? kBlockBytesQ4
         : type == KVM_TYPE_Q5_0 ? kBlockBytesQ5
         : type == KVM_TYPE_F16  ? 64 : 0;
}

__device__ __forceinline__ void st_u16(uint8_t *p, uint32_t v) {
    *reinterpret_cast<uint16_t *>(p) = static_cast<uint16_t>(v);
}

__device__ __forceinline__ uint32_t f16_bits(float d) {
    return static_cast<uint32_t>(__half_as_ushort(__float2half_rn(d)));
}

// Packed FP32x2 arithmetic (sm_100) issued as PTX; per component each is the
// IEEE operation with the named rounding.  A packed multiply whose result
// feeds a packed add was observed fused into one FFMA2 -- the product's
// rounding lost -- both through the CUDA __fmul2_rn / __fadd2_rn intrinsics
// and through these .rn wrappers, so every product that an add consumes is a
// scalar __fmul_rn (never merged into a multiply-add); the packed ops below
// only add, or multiply by a power of two (exact).
#define KVM_F2_OP(name, op)                                                               \
    __device__ __forceinline__ float2 name(float2 a, float2 b) {                         \
        float2 d;                                                                         \
        asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t" \
            op " rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"                              \
            : "=f"(d.x), "=f"(d.y)                                                        \
            : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));                                    \
        return d;                                                                         \
    }
KVM_F2_OP(f2_mul_rn, "mul.rn.f32x2")
KVM_F2_OP(f2_add_rn, "add.rn.f32x2")
KVM_F2_OP(f2_add_rz, "add.rz.f32x2")
#undef KVM_F2_OP

// a*b + c per component with one rounding (fused by definition).
__device__ __forceinline__ float2 f2_fma_rn(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "mov.b64 rc, {%6, %7};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

// amax / 127.0f, correctly rounded, for amax >= 0: Markstein's correction
// step (P. Markstein, "IA-64 and Elementary Functions", 2000) with the
// correctly rounded reciprocal r = RN(1/127): q0 = RN(a*r) is within an ulp of
// a/127, the remainder a - q0*127 is exact under one FMA, and RN(q0 + rem*r)
// is RN(a/127).  Checked against IEEE division for every non-negative finite
// float; infinity is passed through as IEEE division does.
__device__ __forceinline__ float div127(float amax) {
    const float r = 0x1.020408p-7f;
    const float q0 = __fmul_rn(amax, r);
    const float rem = __fmaf_rn(-q0, 127.0f, amax);
    const float q1 = __fmaf_rn(rem, r, q0);
    return amax == __int_as_float(0x7f800000) ? amax : q1;
}

// C roundf (round half away from zero) as an integer for |x| < 2^23:
// truncate x + copysign(0.49999997, x).  Adding the largest float below 0.5
// instead of 0.5 keeps the sum exact or correctly rounded on both sides of
// every half-integer; equality with roundf was checked for every float of
// magnitude below 2^23.  q8_0 codes are at most 127.x in magnitude.
__device__ __forceinline__ int round_half_away(float x) {
    return __float2int_rz(__fadd_rn(x, copysignf(0x1.fffffep-2f, x)));
}

// A lane's block as four 16-byte chunks in a lane-dependent order, so that
// the 128-bit shared-memory reads of a quarter warp (8 neighbouring blocks)
// spread over the banks:
//   rotation (q8_0, F16): raw[k] = chunk (c0 + k) & 3, c0 = (lane >> 1) & 3,
//     8 different bank groups;
//   xor (q4_0, q5_0): raw[k] = chunk k ^ c0, c0 = (lane >> 1) & 1, 4 groups
//     (two lanes a group) -- but the nibble partners (chunks c and c ^ 2)
//     stay at registers k and k + 2 with the lower chunk first, so pairing
//     them needs no selects.
struct Block32 {
    uint4 raw[4];      // raw[k] = chunk chunk_of<XOR>(b, k) of the block (8 halves)
    int c0;
};

template <bool XOR>
__device__ __forceinline__ int chunk_of(const Block32 &b, int k) { return XOR ? (k ^ b.c0) : ((b.c0 + k) & 3); }

__device__ __forceinline__ const __half2 *halves(const uint4 &r) {
    return reinterpret_cast<const __half2 *>(&r);
}

__device__ __forceinline__ float absmax32(const Block32 &b) {
    __half2 m = __habs2(halves(b.raw[0])[0]);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
#pragma unroll
        for (int i = (k == 0 ? 1 : 0); i < 4; ++i) m = __hmax2(m, __habs2(halves(b.raw[k])[i]));
    }
    // __hmax2 and fmaxf return the other operand of a NaN, as the reference's
    // fmaxf scan from 0 does; only an all-NaN block leaves NaN, which it reads as 0
    return fmaxf(fmaxf(__low2float(m), __high2float(m)), 0.0f);
}

// Signed value of the first element (in block order) whose magnitude equals
// amax: the reference's strict `amax < |v|` scan.  +0.0 when amax is 0.
template <bool XOR>
__device__ __forceinline__ float first_of_absmax(const Block32 &b, float amax) {
    if (amax == 0.0f) return 0.0f;
    float best = 0.0f;
    int best_c = 4;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        float v = 0.0f;
        bool hit = false;
#pragma unroll
        for (int i = 3; i >= 0; --i) {
            const float2 x = __half22float2(halves(b.raw[k])[i]);
            const bool hy = fabsf(x.y) == amax;
            const bool hx = fabsf(x.x) == amax;
            v = hy ? x.y : v;
            v = hx ? x.x : v;
            hit = hit || hx || hy;
        }
        const int c = chunk_of<XOR>(b, k);
        const bool take = hit && c < best_c;
        best = take ? v : best;
        best_c = take ? c : best_c;
    }
    return best;
}

// q8_0: 34 bytes = f16 d + 32 int8 codes.
__device__ __forceinline__ void quant_q8_0(const Block32 &b, uint8_t *blk) {
    const float amax = absmax32(b);
    const float d = div127(amax);
    const float id = d != 0.0f ? __frcp_rn(d) : 0.0f;
    st_u16(blk, f16_bits(d));
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const __half2 *h = halves(b.raw[k]);
        uint32_t w[2];
#pragma unroll
        for (int p = 0; p < 2; ++p) {
            const float2 a = __half22float2(h[2 * p]);
            const float2 c = __half22float2(h[2 * p + 1]);
            const uint32_t q0 = static_cast<uint32_t>(round_half_away(__fmul_rn(a.x, id))) & 0xffu;
            const uint32_t q1 = static_cast<uint32_t>(round_half_away(__fmul_rn(a.y, id))) & 0xffu;
            const uint32_t q2 = static_cast<uint32_t>(round_half_away(__fmul_rn(c.x, id))) & 0xffu;
            const uint32_t q3 = static_cast<uint32_t>(round_half_away(__fmul_rn(c.y, id))) & 0xffu;
            w[p] = q0 | (q1 << 8) | (q2 << 16) | (q3 << 24);
        }
        uint8_t *qs = blk + 2 + 8 * chunk_of<false>(b, k);
        st_u16(qs, w[0] & 0xffffu);
        st_u16(qs + 2, w[0] >> 16);
        st_u16(qs + 4, w[1] & 0xffffu);
        st_u16(qs + 6, w[1] >> 16);
    }
}

// Byte codes min(MAXQ, (int)t) of four values t >= 0 (the reference's
// `(int)(x*id + off)` and its clamp), MAXQ = 15 or 31.  (int)t for 0 <= t <
// 2^23 is the low byte of RZ(t + 2^23): that sum has an ulp of 1, so rounding
// toward zero drops exactly the fraction.  MAXQ + 1 is the only larger code
// (t is at most MAXQ + 1.5) and is lowered by one.  A NaN t (a NaN or
// infinite input) gives the canonical NaN, low byte 0xff, and code 0, as the
// float-to-int conversion does.
template <int MAXQ>
__device__ __forceinline__ uint32_t codes4(float2 t0, float2 t1) {
    static_assert(MAXQ == 15 || MAXQ == 31, "MAXQ");
    const float2 mg = make_float2(0x1p23f, 0x1p23f);
    const float2 u0 = f2_add_rz(t0, mg);
    const float2 u1 = f2_add_rz(t1, mg);
    uint32_t v = __byte_perm(__byte_perm(__float_as_uint(u0.x), __float_as_uint(u0.y), 0x0040u),
                             __byte_perm(__float_as_uint(u1.x), __float_as_uint(u1.y), 0x0040u), 0x5410u);
    v &= ~(((v >> 7) & 0x01010101u) * 0xffu);
    return v - ((v >> (MAXQ == 15 ? 4 : 5)) & 0x01010101u);
}

// RN(RN(x*id) + off) for a pair: the products scalar and rounded, the add packed.
__device__ __forceinline__ float2 mul_add_off(float2 x, float id, float2 off) {
    return f2_add_rn(make_float2(__fmul_rn(x.x, id), __fmul_rn(x.y, id)), off);
}

// The 8 codes of one chunk as bytes, min(MAXQ, (int)(x*id + off)) each:
// word p holds values 4p .. 4p+3.  The products are scalar and rounded, the
// adds packed (per component the same IEEE add).  x*id lies in [-h, h] for
// vmax = -h*d (h = 8 or 16), so t = x*id + off is in [0.5, MAXQ + 1.5] and
// (int)t is at most MAXQ + 1; the clamp is then one subtraction per 4
// codes of each byte's bit log2(MAXQ + 1).
//   RZ: (int)t as the low byte of RZ(t + 2^23) (see codes4), two packed adds
//     per 4 codes instead of 4 conversions.  Only a NaN t (a NaN or infinite
//     input) gives a byte above MAXQ + 1 (0xff); `nan_bytes` collects the
//     bytes so that the caller can redo such a block without RZ.
//   without RZ: float-to-int conversions, which turn a NaN t into code 0.
template <int MAXQ, bool RZ>
__device__ __forceinline__ void chunk_code_bytes(const uint4 &r, float id, float off, uint32_t (&w)[2],
                                                 uint32_t &nan_bytes) {
    static_assert(MAXQ == 15 || MAXQ == 31, "MAXQ");
    const __half2 *h = halves(r);
    const float2 o2 = make_float2(off, off);
#pragma unroll
    for (int p = 0; p < 2; ++p) {
        const float2 x0 = __half22float2(h[2 * p]);
        const float2 x1 = __half22float2(h[2 * p + 1]);
        const float2 t0 = f2_add_rn(make_float2(__fmul_rn(x0.x, id), __fmul_rn(x0.y, id)), o2);
        const float2 t1 = f2_add_rn(make_float2(__fmul_rn(x1.x, id), __fmul_rn(x1.y, id)), o2);
        uint32_t v;
        if (RZ) {
            const float2 mg = make_float2(0x1p23f, 0x1p23f);
            const float2 u0 = f2_add_rz(t0, mg), u1 = f2_add_rz(t1, mg);
            v = __byte_perm(__byte_perm(__float_as_uint(u0.x), __float_as_uint(u0.y), 0x0040u),
                            __byte_perm(__float_as_uint(u1.x), __float_as_uint(u1.y), 0x0040u), 0x5410u);
            nan_bytes |= v;
        } else {
            const uint32_t c0 = __float2uint_rz(t0.x), c1 = __float2uint_rz(t0.y);
            const uint32_t c2 = __float2uint_rz(t1.x), c3 = __float2uint_rz(t1.y);
            v = __byte_perm(__byte_perm(c0, c1, 0x0040u), __byte_perm(c2, c3, 0x0040u), 0x5410u);
        }
        w[p] = v - ((v >> (MAXQ == 15 ? 4 : 5)) & 0x01010101u);
    }
}

// Bit 4 of each of the 8 byte codes (at most 31) of words a (values 0..3)
// and b (values 4..7), as the top byte of the result: value i's bit on bit
// 24 + i.  One select puts a's bits on bits 8i and b's on bits 8i + 4 (a's
// code bytes shifted down by 4 leave their bit 4 alone in the low nibble,
// b's bits 5..7 are zero); the multiply by 2^24 + 2^17 + 2^10 + 2^3 moves
// byte i's bits to 24 + i and 28 + i, and every other partial product lands
// either above bit 31 or on its own bit below 24, so nothing carries.
__device__ __forceinline__ uint32_t high_bits8(uint32_t a, uint32_t b) {
    const uint32_t x = ((a >> 4) & 0x0f0f0f0fu) | (b & 0xf0f0f0f0u);
    return x * 0x01020408u;
}

// The top bytes of p0..p3 as one word (byte i = top byte of p_i).
__device__ __forceinline__ uint32_t top_bytes4(uint32_t p0, uint32_t p1, uint32_t p2, uint32_t p3) {
    return __byte_perm(__byte_perm(p0, p1, 0x0073u), __byte_perm(p2, p3, 0x0073u), 0x5410u);
}

// vmax of q4_0 / q5_0 -- the first value (block order) of largest magnitude --
// from the block's signed max and min: when max > -min every value of that
// magnitude is the max, when -min > max the min; only a +a / -a tie needs the
// first occurrence.  +0.0 when every value is zero.  *amax_out gets amax.
template <bool XOR>
__device__ __forceinline__ float signed_absmax(const Block32 &b, float *amax_out) {
    __half2 mx = halves(b.raw[0])[0];
    __half2 mn = mx;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
#pragma unroll
        for (int i = (k == 0 ? 1 : 0); i < 4; ++i) {
            mx = __hmax2(mx, halves(b.raw[k])[i]);
            mn = __hmin2(mn, halves(b.raw[k])[i]);
        }
    }
    const float hi = fmaxf(__low2float(mx), __high2float(mx));
    const float lo = fminf(__low2float(mn), __high2float(mn));
    const float amax = fmaxf(hi, -lo);
    *amax_out = amax;
    if (!(amax > 0.0f)) return 0.0f;          // all zero, or all NaN (the reference's scan keeps 0)
    if (hi != -lo) return hi > -lo ? hi : lo;
    return first_of_absmax<XOR>(b, amax);
}

// A ggml block of a 2-byte header (F16 d) followed by NW payload words (4*NW
// bytes), at a 2-byte aligned address: NW word stores and one half-word store.
// At a 4-byte aligned address the words are shifted by two bytes.
template <int NW>
__device__ __forceinline__ void store_block(uint8_t *blk, uint32_t hdr, const uint32_t (&w)[NW]) {
    const bool odd = (reinterpret_cast<uintptr_t>(blk) & 2u) != 0u;
    const uint32_t sel = odd ? 0x7654u : 0x5432u;
    uint32_t *wp = reinterpret_cast<uint32_t *>(blk + (odd ? 2 : 0));
    uint32_t prev = hdr << 16;
#pragma unroll
    for (int k = 0; k < NW; ++k) {
        wp[k] = __byte_perm(prev, w[k], sel);
        prev = w[k];
    }
    st_u16(blk + (odd ? 0 : 4 * NW), odd ? hdr : (w[NW - 1] >> 16));
}

// q4_0 (18 bytes) and q5_0 (22 bytes: d, qh, 16 nibble bytes) of a block
// in the xor chunk order.  d = vmax / -8 (-16) is computed as vmax * -0.125
// (-0.0625): division and multiplication by a power of two return the same
// correctly rounded value.
template <bool Q5>
__device__ __forceinline__ void quant_q4q5(const Block32 &b, uint8_t *blk) {
    float amax;
    const float vmax = signed_absmax<true>(b, &amax);
    const float d = __fmul_rn(vmax, Q5 ? -0.0625f : -0.125f);
    const float id = d != 0.0f ? __frcp_rn(d) : 0.0f;
    const float off = Q5 ? 16.5f : 8.5f;
    uint32_t w[4][2];
    uint32_t nan_bytes = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) chunk_code_bytes<Q5 ? 31 : 15, true>(b.raw[k], id, off, w[k], nan_bytes);
    if (nan_bytes & 0xc0c0c0c0u) {        // a NaN or infinite input: codes by conversion
#pragma unroll
        for (int k = 0; k < 4; ++k) chunk_code_bytes<Q5 ? 31 : 15, false>(b.raw[k], id, off, w[k], nan_bytes);
    }
    // Registers k and k + 2 (k < 2) hold the nibble pair of chunks c0 ^ k and
    // c0 ^ k ^ 2, the lower one first: value j of register k takes the low
    // nibble of byte j, its partner 16 values on the high one.  Pair k = 0 is
    // nibble words 0-1 when c0 = 0, else 2-3.
    uint32_t nib[2][2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
#pragma unroll
        for (int p = 0; p < 2; ++p) nib[k][p] = (w[k][p] & 0x0f0f0f0fu) | ((w[k + 2][p] << 4) & 0xf0f0f0f0u);
    }
    const bool first0 = b.c0 == 0;
    constexpr int NW = Q5 ? 5 : 4;
    uint32_t o[NW];
#pragma unroll
    for (int p = 0; p < 2; ++p) {
        o[NW - 4 + p] = first0 ? nib[0][p] : nib[1][p];
        o[NW - 2 + p] = first0 ? nib[1][p] : nib[0][p];
    }
    if (Q5) {
        // byte k of t is chunk k ^ c0's: swap the bytes of each half when c0 = 1
        const uint32_t t = top_bytes4(high_bits8(w[0][0], w[0][1]), high_bits8(w[1][0], w[1][1]),
                                      high_bits8(w[2][0], w[2][1]), high_bits8(w[3][0], w[3][1]));
        o[0] = __byte_perm(t, 0u, first0 ? 0x3210u : 0x2301u);
    }
    store_block<NW>(blk, f16_bits(d), o);
}

// Block `qb` of a tile (64 bytes per block in shared memory) in the rotation
// (XOR = false) or xor chunk order.
template <bool XOR>
__device__ __forceinline__ void load_block(const uint8_t *tile, uint32_t qb, int lane, Block32 &b) {
    b.c0 = XOR ? (lane >> 1) & 1 : (lane >> 1) & 3;
    const uint8_t *p = tile + static_cast<size_t>(qb) * 64u;
#pragma unroll
    for (int k = 0; k < 4; ++k) b.raw[k] = *reinterpret_cast<const uint4 *>(p + 16 * chunk_of<XOR>(b, k));
}

// One 32-value block of `type`: tile block qb into out_tile block qb.  F16
// blocks are written as 16-byte chunks when out_tile is 16-byte aligned
// (A16), else as 2-byte halves.
template <bool A16 = true>
__device__ __forceinline__ void quant_block(int type, const uint8_t *tile, uint32_t qb, int lane,
                                            uint8_t *out_tile) {
    Block32 b;
    if (type == KVM_TYPE_Q4_0 || type == KVM_TYPE_Q5_0) {
        load_block<true>(tile, qb, lane, b);
        if (type == KVM_TYPE_Q4_0) quant_q4q5<false>(b, out_tile + static_cast<size_t>(qb) * kBlockBytesQ4);
        else quant_q4q5<true>(b, out_tile + static_cast<size_t>(qb) * kBlockBytesQ5);
        return;
    }
    load_block<false>(tile, qb, lane, b);
    if (type == KVM_TYPE_Q8_0) {
        quant_q8_0(b, out_tile + static_cast<size_t>(qb) * kBlockBytesQ8);
    } else {
        uint8_t *o = out_tile + static_cast<size_t>(qb) * 64u;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            if (A16) {
                *reinterpret_cast<uint4 *>(o + 16 * chunk_of<false>(b, k)) = b.raw[k];
            } else {
                const uint32_t w[4] = {b.raw[k].x, b.raw[k].y, b.raw[k].z, b.raw[k].w};
#pragma unroll
                for (int m = 0; m < 4; ++m) {
                    st_u16(o + 16 * chunk_of<false>(b, k) + 4 * m, w[m] & 0xffffu);
                    st_u16(o + 16 * chunk_of<false>(b, k) + 4 * m + 2, w[m] >> 16);
                }
            }
        }
    }
}

}  // namespace kvm
