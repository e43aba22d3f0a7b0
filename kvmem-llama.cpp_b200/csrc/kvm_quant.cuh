// kvm_quant.cuh -- ggml q8_0 / q4_0 / q5_0 block quantizers for a warp.
//
// One 32-value ggml block is handled by 4 consecutive lanes (sub = lane & 3),
// each holding 8 consecutive values.  The arithmetic is the reference's
// (src/adapter/llama-kvmem-stagein.cu:180-233, ggml's quantize_row_*_ref):
//   q8_0: d = amax/127, id = d ? 1/d : 0, q = roundf(x*id)
//   q4_0: vmax = first value of largest |x|, d = vmax/-8, q = min(15, (int)(x*id + 8.5))
//   q5_0: d = vmax/-16, q = min(31, (int)(x*id + 16.5)), bit 4 of q_i -> bit i of qh
// with every operation an IEEE round-to-nearest intrinsic (no FMA
// contraction, no fast reciprocals) so the bytes match the CPU bit for bit.
// All 32 lanes of the warp must call these (they shuffle); `active` masks the
// shared-memory stores of lanes without a block.
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

// 8 halves (one uint4) -> 8 floats, exact.
__device__ __forceinline__ void unpack8(const uint4 raw, float v[8]) {
    const __half2 *h = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(h[k]);
        v[2 * k] = f.x;
        v[2 * k + 1] = f.y;
    }
}

__device__ __forceinline__ uint32_t f16_bits(float d) {
    return static_cast<uint32_t>(__half_as_ushort(__float2half_rn(d)));
}

// q8_0: blk = start of the 34-byte block in shared memory.
__device__ __forceinline__ void quant_q8_0_part(const float v[8], int sub, uint8_t *blk,
                                                bool active) {
    float amax = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) amax = fmaxf(amax, fabsf(v[k]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    if (!active) return;
    if (sub == 0) st_u16(blk, f16_bits(d));
    uint32_t b[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int q = static_cast<int>(roundf(__fmul_rn(v[k], id)));
        b[k] = static_cast<uint32_t>(q) & 0xffu;
    }
    uint8_t *qs = blk + 2 + sub * 8;
#pragma unroll
    for (int k = 0; k < 4; ++k) st_u16(qs + 2 * k, b[2 * k] | (b[2 * k + 1] << 8));
}

// Signed value of the first element of largest magnitude across the 4 lanes
// (strict `amax < |v|` scan in index order; ties resolve to the lower index).
__device__ __forceinline__ float group_first_absmax(const float v[8], int sub) {
    float amax = 0.0f;
    float vmax = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const float a = fabsf(v[k]);
        if (amax < a) {
            amax = a;
            vmax = v[k];
        }
    }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, amax, o);
        const float ov = __shfl_xor_sync(0xffffffffu, vmax, o);
        const bool other_first = (sub ^ o) < sub;
        if (oa > amax || (oa == amax && other_first)) {
            amax = oa;
            vmax = ov;
        }
    }
    return vmax;
}

// q4_0: blk = start of the 18-byte block.
__device__ __forceinline__ void quant_q4_0_part(const float v[8], int sub, uint8_t *blk,
                                                bool active) {
    const float vmax = group_first_absmax(v, sub);
    const float d = __fdiv_rn(vmax, -8.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    uint32_t packed = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        int q = __float2int_rz(__fadd_rn(__fmul_rn(v[k], id), 8.5f));
        q = q > 15 ? 15 : q;
        packed |= (static_cast<uint32_t>(q) & 15u) << (4 * k);
    }
    // element j (j < 16) pairs with element j + 16, held by lane sub ^ 2
    const uint32_t partner = __shfl_xor_sync(0xffffffffu, packed, 2);
    if (!active) return;
    if (sub == 0) st_u16(blk, f16_bits(d));
    if (sub < 2) {
        uint8_t *qs = blk + 2 + sub * 8;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t b0 = ((packed >> (8 * k)) & 15u) | (((partner >> (8 * k)) & 15u) << 4);
            const uint32_t b1 = ((packed >> (8 * k + 4)) & 15u) |
                                (((partner >> (8 * k + 4)) & 15u) << 4);
            st_u16(qs + 2 * k, b0 | (b1 << 8));
        }
    }
}

// q5_0: blk = start of the 22-byte block (d, qh[4], qs[16]).
__device__ __forceinline__ void quant_q5_0_part(const float v[8], int sub, uint8_t *blk,
                                                bool active) {
    const float vmax = group_first_absmax(v, sub);
    const float d = __fdiv_rn(vmax, -16.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    uint32_t packed = 0;
    uint32_t hi = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        int q = __float2int_rz(__fadd_rn(__fmul_rn(v[k], id), 16.5f));
        q = q > 31 ? 31 : q;
        packed |= (static_cast<uint32_t>(q) & 15u) << (4 * k);
        hi |= ((static_cast<uint32_t>(q) >> 4) & 1u) << (sub * 8 + k);
    }
    hi |= __shfl_xor_sync(0xffffffffu, hi, 1);
    hi |= __shfl_xor_sync(0xffffffffu, hi, 2);
    const uint32_t partner = __shfl_xor_sync(0xffffffffu, packed, 2);
    if (!active) return;
    if (sub == 0) {
        st_u16(blk, f16_bits(d));
        st_u16(blk + 2, hi & 0xffffu);
        st_u16(blk + 4, hi >> 16);
    }
    if (sub < 2) {
        uint8_t *qs = blk + 6 + sub * 8;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t b0 = ((packed >> (8 * k)) & 15u) | (((partner >> (8 * k)) & 15u) << 4);
            const uint32_t b1 = ((packed >> (8 * k + 4)) & 15u) |
                                (((partner >> (8 * k + 4)) & 15u) << 4);
            st_u16(qs + 2 * k, b0 | (b1 << 8));
        }
    }
}

// Quantize the 8 values of lane `sub` of ggml block `qb` into `out`
// (type-dispatched; warp-uniform type).  For F16 the 8 halves are copied.
__device__ __forceinline__ void quant_part(int type, const uint4 raw, int sub, uint8_t *out_tile,
                                           uint32_t qb, bool active) {
    float v[8];
    unpack8(raw, v);
    if (type == KVM_TYPE_Q8_0) {
        quant_q8_0_part(v, sub, out_tile + static_cast<size_t>(qb) * kBlockBytesQ8, active);
    } else if (type == KVM_TYPE_Q4_0) {
        quant_q4_0_part(v, sub, out_tile + static_cast<size_t>(qb) * kBlockBytesQ4, active);
    } else if (type == KVM_TYPE_Q5_0) {
        quant_q5_0_part(v, sub, out_tile + static_cast<size_t>(qb) * kBlockBytesQ5, active);
    } else if (active) {
        *reinterpret_cast<uint4 *>(out_tile + static_cast<size_t>(qb) * 64 + sub * 16) = raw;
    }
}

}  // namespace kvm
