// kvm_produce.cu -- device producers of the statistics the scorer reads.
//
// mean_k_kernel: the per-(layer, block) ordered F32 token sum of pre-RoPE K
//   (RawKvStore::add_mean_f32 / write_layer_mean_k, kvmem/src/host/
//   raw_kv_store.cpp:204-223, :674-694), written straight into the tiled
//   summary layout.  Two ways to name the rows:
//     table mode  -- whole blocks of an F16 history source (kvm_summarize):
//                    block b holds min(n_tokens[b], T) rows from offset 0;
//     token mode  -- tokens [pos0, pos0+n) of a captured ggml tensor
//                    (kvm_write_mean_k): row i is position pos0+i, a block
//                    written from offset 0 restarts its sum, a block written
//                    from offset > 0 continues the stored sum.
//   Each warp owns one block and each lane V consecutive channels (V = 8 for
//   16-bit sources, 4 for F32: 16-byte loads, 4 rows in flight), so the rows
//   stream in coalesced 512-byte warp accesses; the 8 blocks of a CTA are
//   transposed through shared memory so every 4 channels' 8 block sums leave
//   as one 128-byte run of the [layer][64-block group][channel/4][64][4] tile.
//   Token-mode calls over few blocks (one ubatch of one layer) instead use
//   mean_k_staged_kernel, which has every row of the block in flight at once.
//
// add_rows_kernel: acc[j] += rows in order (kvmem_meank_add,
//   src/adapter/llama-kvmem-stagein.cu:269-315; harvest 'q',
//   src/adapter/llama-memory-kvmem.cpp:2157-2173), one thread per element.
//
// meank_flush_kernel: RawKvStore::write_layer_mean_sum (raw_kv_store.cpp:
//   696-720) of the decode accumulators into their block, then acc = 0.
#include "kvm_internal.cuh"
#include "kvm_kernels.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <atomic>

namespace kvm {

namespace {

constexpr int kMeanWarps = 8;     // blocks per CTA
constexpr int kStagedThreads = 256;
constexpr uint32_t kStagedSmem = 64u * 1024u;   // row slab of the staged kernel

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b) { return __uint_as_float(b << 16); }

__device__ __forceinline__ float load_elem(const uint8_t *p, int32_t type) {
    if (type == kActF32) return *reinterpret_cast<const float *>(p);
    const uint16_t u = *reinterpret_cast<const uint16_t *>(p);
    if (type == kActF16) return __half2float(__ushort_as_half(u));
    return bf16_bits_to_f32(u);
}

// V consecutive channels of one row, widened to F32 (exact for every type).
template <int V, int TYPE>
struct RowLoad;

template <int TYPE>
struct RowLoad<8, TYPE> {
    static __device__ __forceinline__ void run(const uint8_t *p, float (&x)[8]) {
        const uint4 r = __ldcs(reinterpret_cast<const uint4 *>(p));
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if (TYPE == kActF16) {
                x[2 * i] = __half2float(__ushort_as_half(static_cast<uint16_t>(w[i] & 0xffffu)));
                x[2 * i + 1] = __half2float(__ushort_as_half(static_cast<uint16_t>(w[i] >> 16)));
            } else {
                x[2 * i] = bf16_bits_to_f32(w[i] & 0xffffu);
                x[2 * i + 1] = bf16_bits_to_f32(w[i] >> 16);
            }
        }
    }
};

template <int TYPE>
struct RowLoad<4, TYPE> {
    static __device__ __forceinline__ void run(const uint8_t *p, float (&x)[4]) {
        const float4 r = __ldcs(reinterpret_cast<const float4 *>(p));
        x[0] = r.x;
        x[1] = r.y;
        x[2] = r.z;
        x[3] = r.w;
    }
};

template <int TYPE>
struct RowLoad<1, TYPE> {
    static __device__ __forceinline__ void run(const uint8_t *p, float (&x)[1]) {
        x[0] = load_elem(p, TYPE);
    }
};

template <int V, int TYPE>
__global__ void __launch_bounds__(kMeanWarps * 32) mean_k_kernel(MeanKArgs a) {
    __shared__ float tile[kMeanWarps][32 * V + 1];
    const uint32_t w = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t E = a.sum.n_embd;
    const uint32_t T = a.block_tokens;
    const uint32_t l = a.layer0 + blockIdx.z;
    const uint32_t grp0 = (a.block0 & ~(kMeanWarps - 1u)) + blockIdx.x * kMeanWarps;
    const uint32_t b = grp0 + w;
    const bool in = b >= a.block0 && b < a.block0 + a.n_blk;
    const uint32_t ec = blockIdx.y * 32u * V;            // first channel of this CTA
    const uint32_t e0 = ec + lane * V;                   // first channel of this lane
    uint32_t off = 0, take = 0;
    if (in) {
        if (a.n_tokens) {
            take = min(a.n_tokens[b], T);
        } else {
            const uint32_t p0 = max(b * T, a.pos0);
            const uint32_t p1 = min((b + 1u) * T, a.pos0 + a.n);
            off = p0 - b * T;
            take = p1 - p0;
        }
    }
    float acc[V];
#pragma unroll
    for (int j = 0; j < V; ++j) acc[j] = 0.0f;
    if (in && e0 < E) {
        if (off != 0) {
#pragma unroll
            for (int j = 0; j < V; ++j)
                if (e0 + j < E) acc[j] = a.sum.sum_t[sum_index(a.sum, l, e0 + j, b)];
        }
        const uint32_t head = e0 / a.head_dim;
        const uint32_t d = e0 % a.head_dim;
        const uint8_t *row = a.src + l * a.nb_layer + head * a.nb_head + d * a.nb_dim;
        if (a.n_tokens)
            row += static_cast<uint64_t>(b) * a.nb_block;
        else
            row += static_cast<uint64_t>(b * T + off - a.pos0) * a.nb_row;
        const uint64_t step = a.nb_row;
        uint32_t t = 0;
        for (; t + 4u <= take; t += 4u) {
            float x0[V], x1[V], x2[V], x3[V];
            RowLoad<V, TYPE>::run(row, x0);
            RowLoad<V, TYPE>::run(row + step, x1);
            RowLoad<V, TYPE>::run(row + 2u * step, x2);
            RowLoad<V, TYPE>::run(row + 3u * step, x3);
#pragma unroll
            for (int j = 0; j < V; ++j) {
                acc[j] = __fadd_rn(acc[j], x0[j]);
                acc[j] = __fadd_rn(acc[j], x1[j]);
                acc[j] = __fadd_rn(acc[j], x2[j]);
                acc[j] = __fadd_rn(acc[j], x3[j]);
            }
            row += 4u * step;
        }
        for (; t < take; ++t) {
            float x[V];
            RowLoad<V, TYPE>::run(row, x);
#pragma unroll
            for (int j = 0; j < V; ++j) acc[j] = __fadd_rn(acc[j], x[j]);
            row += step;
        }
    }
#pragma unroll
    for (int j = 0; j < V; ++j) tile[w][lane * V + j] = acc[j];
    if (in && blockIdx.y == 0 && lane == 0) {
        const size_t at = static_cast<size_t>(l) * a.sum.ldb + b;
        uint32_t mt = take;
        if (!a.n_tokens && off != 0) mt = max(a.sum.mean_tok[at], off + take);
        a.sum.mean_tok[at] = mt;
        a.sum.inv_tok[at] = mt ? __fdiv_rn(1.0f, __uint2float_rn(mt)) : 0.0f;
    }
    __syncthreads();
    // 4 channels x 8 blocks of the tiled layout are 32 consecutive floats:
    // thread i writes channel 4*(i/32) + i%4 of block (i%32)/4
    static_assert(kMeanWarps * 4 == 32, "one 128-byte run per channel quad");
    for (uint32_t i = threadIdx.x; i < kMeanWarps * 32u * V; i += kMeanWarps * 32u) {
        const uint32_t el = (i / 32u) * 4u + (i % 4u);
        const uint32_t bw = (i % 32u) / 4u;
        const uint32_t bb = grp0 + bw;
        const uint32_t e = ec + el;
        if (bb >= a.block0 && bb < a.block0 + a.n_blk && e < E)
            a.sum.sum_t[sum_index(a.sum, l, e, bb)] = tile[bw][el];
    }
}

// Token mode for calls that cover few blocks (one ubatch of one layer): one
// CTA per (block, channel chunk) first copies the chunk of every row of its
// block into shared memory -- all loads independent and in flight at once --
// then each thread adds its channel's rows in token order.
template <int TYPE, bool VEC>
__global__ void __launch_bounds__(kStagedThreads) mean_k_staged_kernel(MeanKArgs a, uint32_t C) {
    extern __shared__ __align__(16) uint8_t slab[];   // [take][C] raw elements
    constexpr uint32_t ES = TYPE == kActF32 ? 4u : 2u;
    constexpr uint32_t G = 16u / ES;                 // elements per 16-byte load
    const uint32_t E = a.sum.n_embd;
    const uint32_t T = a.block_tokens;
    const uint32_t l = a.layer0 + blockIdx.z;
    const uint32_t b = a.block0 + blockIdx.x;
    const uint32_t c0 = blockIdx.y * C;
    const uint32_t nc = min(C, E - c0);
    const uint32_t p0 = max(b * T, a.pos0);
    const uint32_t p1 = min((b + 1u) * T, a.pos0 + a.n);
    const uint32_t off = p0 - b * T;
    const uint32_t take = p1 - p0;
    const uint8_t *rows = a.src + l * a.nb_layer + static_cast<uint64_t>(p0 - a.pos0) * a.nb_row;
    if (VEC) {
        // eight independent 16-byte loads in flight per thread, then their stores
        const uint32_t segs = nc / G;
        const uint32_t n_seg = take * segs;
        constexpr uint32_t U = 8;
        for (uint32_t r0 = threadIdx.x; r0 < n_seg; r0 += U * kStagedThreads) {
            uint4 v[U];
            uint32_t at[U];
#pragma unroll
            for (uint32_t k = 0; k < U; ++k) {
                const uint32_t r = r0 + k * kStagedThreads;
                at[k] = 0xffffffffu;
                if (r < n_seg) {
                    const uint32_t t = r / segs;
                    const uint32_t e = c0 + (r - t * segs) * G;
                    const uint8_t *p = rows + t * a.nb_row + (e / a.head_dim) * a.nb_head + (e % a.head_dim) * a.nb_dim;
                    v[k] = __ldcs(reinterpret_cast<const uint4 *>(p));
                    at[k] = t * C + (e - c0);
                }
            }
#pragma unroll
            for (uint32_t k = 0; k < U; ++k)
                if (at[k] != 0xffffffffu) *reinterpret_cast<uint4 *>(slab + static_cast<size_t>(at[k]) * ES) = v[k];
        }
    } else {
        for (uint32_t r = threadIdx.x; r < take * nc; r += kStagedThreads) {
            const uint32_t t = r / nc;
            const uint32_t e = c0 + (r - t * nc);
            const uint8_t *p = rows + t * a.nb_row + (e / a.head_dim) * a.nb_head + (e % a.head_dim) * a.nb_dim;
            uint8_t *q = slab + (static_cast<size_t>(t) * C + (e - c0)) * ES;
            if (ES == 4u)
                *reinterpret_cast<uint32_t *>(q) = *reinterpret_cast<const uint32_t *>(p);
            else
                *reinterpret_cast<uint16_t *>(q) = *reinterpret_cast<const uint16_t *>(p);
        }
    }
    __syncthreads();
    for (uint32_t c = threadIdx.x; c < nc; c += kStagedThreads) {
        const size_t idx = sum_index(a.sum, l, c0 + c, b);
        float acc = off == 0 ? 0.0f : a.sum.sum_t[idx];
        const uint8_t *q = slab + static_cast<size_t>(c) * ES;
#pragma unroll 8
        for (uint32_t t = 0; t < take; ++t) acc = __fadd_rn(acc, load_elem(q + static_cast<size_t>(t) * C * ES, TYPE));
        a.sum.sum_t[idx] = acc;
    }
    if (blockIdx.y == 0 && threadIdx.x == 0) {
        const size_t at = static_cast<size_t>(l) * a.sum.ldb + b;
        const uint32_t mt = off == 0 ? take : max(a.sum.mean_tok[at], off + take);
        a.sum.mean_tok[at] = mt;
        a.sum.inv_tok[at] = mt ? __fdiv_rn(1.0f, __uint2float_rn(mt)) : 0.0f;
    }
}

__global__ void add_rows_kernel(AddRowsArgs a) {
    const uint32_t j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= a.n_elem) return;
    const uint32_t head = j / a.head_dim;
    const uint32_t d = j % a.head_dim;
    const uint8_t *base = a.src + head * a.nb_head + d * a.nb_dim;
    float s = a.acc[j];
    for (uint32_t i = 0; i < a.n; ++i) {
        const uint32_t t = a.tok_list ? a.tok_list[i] : a.tok0 + i;
        s = __fadd_rn(s, load_elem(base + static_cast<uint64_t>(t) * a.nb_tok, a.type));
    }
    a.acc[j] = s;
}

__global__ void meank_flush_kernel(SummaryLayout sum, float *meank, uint32_t layer0, uint32_t pos0,
                                   uint32_t n, uint32_t block_tokens) {
    const uint32_t l = layer0 + blockIdx.y;
    const uint32_t e = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t E = sum.n_embd;
    const uint32_t bid = pos0 / block_tokens;
    const uint32_t off = pos0 % block_tokens;
    const uint32_t take = min(n, block_tokens - off);
    if (e < E) {
        float *acc = meank + static_cast<size_t>(l) * E;
        const size_t idx = sum_index(sum, l, e, bid);
        const float base = off == 0 ? 0.0f : sum.sum_t[idx];
        sum.sum_t[idx] = __fadd_rn(base, acc[e]);
        acc[e] = 0.0f;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        const size_t at = static_cast<size_t>(l) * sum.ldb + bid;
        const uint32_t mt = off == 0 ? take : max(sum.mean_tok[at], off + take);
        sum.mean_tok[at] = mt;
        sum.inv_tok[at] = mt ? __fdiv_rn(1.0f, __uint2float_rn(mt)) : 0.0f;
    }
}

template <int V, int TYPE>
cudaError_t launch_mean_k_t(const MeanKArgs &a, uint32_t n_layers, cudaStream_t stream) {
    const uint32_t g0 = a.block0 / kMeanWarps;
    const uint32_t g1 = (a.block0 + a.n_blk + kMeanWarps - 1u) / kMeanWarps;
    dim3 grid(g1 - g0, (a.sum.n_embd + 32u * V - 1u) / (32u * V), n_layers);
    mean_k_kernel<V, TYPE><<<grid, kMeanWarps * 32, 0, stream>>>(a);
    return cudaGetLastError();
}

template <int TYPE, bool VEC>
cudaError_t launch_staged_t(const MeanKArgs &a, uint32_t n_layers, uint32_t C, cudaStream_t stream) {
    static std::atomic<uint64_t> attr{0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!(attr.load(std::memory_order_acquire) & (1ull << dev))) {
        cudaError_t e = cudaFuncSetAttribute(mean_k_staged_kernel<TYPE, VEC>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, kStagedSmem);
        if (e != cudaSuccess) return e;
        attr.fetch_or(1ull << dev, std::memory_order_acq_rel);
    }
    const size_t es = TYPE == kActF32 ? 4u : 2u;
    const size_t smem = static_cast<size_t>(a.block_tokens) * C * es;
    dim3 grid(a.n_blk, (a.sum.n_embd + C - 1u) / C, n_layers);
    mean_k_staged_kernel<TYPE, VEC><<<grid, kStagedThreads, smem, stream>>>(a, C);
    return cudaGetLastError();
}

}  // namespace

uint32_t mean_k_vec(int32_t type, uint32_t head_dim, uint64_t nb_dim, uint64_t align_mask) {
    if ((type == kActF16 || type == kActBF16) && nb_dim == 2u && head_dim % 8u == 0u &&
        (align_mask & 15u) == 0u)
        return 8u;
    if (type == kActF32 && nb_dim == 4u && head_dim % 4u == 0u && (align_mask & 15u) == 0u)
        return 4u;
    return 1u;
}

cudaError_t launch_mean_k(const MeanKArgs &a, uint32_t n_layers, cudaStream_t stream) {
    if (a.n_blk == 0 || n_layers == 0) return cudaSuccess;
    // Token-mode calls that would give the warp kernel less than two CTAs per
    // SM use the staged kernel when a 32-channel slab of the block fits.
    const uint32_t es = a.type == kActF32 ? 4u : 2u;
    const uint32_t warp_ctas = ((a.n_blk + kMeanWarps - 1u) / kMeanWarps + 1u) *
                               ((a.sum.n_embd + 32u * a.vec - 1u) / (32u * a.vec)) * n_layers;
    uint32_t C = (kStagedSmem / (a.block_tokens * es)) & ~31u;
    if (C > 256u) C = 256u;
    if (!a.n_tokens && C >= 32u && warp_ctas < 2u * 148u) {
        const bool vec = a.vec > 1u;
        switch (a.type * 2 + (vec ? 1 : 0)) {
            case kActF32 * 2 + 1: return launch_staged_t<kActF32, true>(a, n_layers, C, stream);
            case kActF32 * 2: return launch_staged_t<kActF32, false>(a, n_layers, C, stream);
            case kActF16 * 2 + 1: return launch_staged_t<kActF16, true>(a, n_layers, C, stream);
            case kActF16 * 2: return launch_staged_t<kActF16, false>(a, n_layers, C, stream);
            case kActBF16 * 2 + 1: return launch_staged_t<kActBF16, true>(a, n_layers, C, stream);
            case kActBF16 * 2: return launch_staged_t<kActBF16, false>(a, n_layers, C, stream);
            default: return cudaErrorInvalidValue;
        }
    }
    switch (a.vec * 100 + a.type) {
        case 800 + kActF16: return launch_mean_k_t<8, kActF16>(a, n_layers, stream);
        case 800 + kActBF16: return launch_mean_k_t<8, kActBF16>(a, n_layers, stream);
        case 400 + kActF32: return launch_mean_k_t<4, kActF32>(a, n_layers, stream);
        case 100 + kActF16: return launch_mean_k_t<1, kActF16>(a, n_layers, stream);
        case 100 + kActBF16: return launch_mean_k_t<1, kActBF16>(a, n_layers, stream);
        case 100 + kActF32: return launch_mean_k_t<1, kActF32>(a, n_layers, stream);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_add_rows(const AddRowsArgs &a, cudaStream_t stream) {
    if (a.n_elem == 0 || a.n == 0) return cudaSuccess;
    add_rows_kernel<<<(a.n_elem + 255u) / 256u, 256, 0, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_meank_flush(const SummaryLayout &s, float *meank, uint32_t layer0, uint32_t n_layers,
                               uint32_t pos0, uint32_t n, uint32_t block_tokens, cudaStream_t stream) {
    if (n_layers == 0 || n == 0) return cudaSuccess;
    dim3 grid((s.n_embd + 255u) / 256u, n_layers);
    meank_flush_kernel<<<grid, 256, 0, stream>>>(s, meank, layer0, pos0, n, block_tokens);
    return cudaGetLastError();
}

}  // namespace kvm
