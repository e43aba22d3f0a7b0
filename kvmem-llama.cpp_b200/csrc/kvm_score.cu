// kvm_score.cu -- mean-K summaries, query preparation and the block scorer.
//
// Scorer: llama_memory_kvmem::score_retrieval (src/adapter/llama-memory-kvmem.cpp:2869-2916),
// restated for the device without changing its arithmetic:
//   per (block, layer, kv head): dot/nk accumulate in float over d in order,
//     r = dot / (sqrt(nq) * sqrt(nk) + 1e-6f)
//   per (block, layer): layer = sum of r over heads in order (double), term = layer / H_kv
//   per block: score = (sum of terms over layers with a query, in layer order) / n_active
// The summaries are stored channel-major in 64-block tiles
// ([layer][64-block group][channel][64]) so that a warp of threads, one per
// block, reads 128 contiguous bytes per channel while each thread keeps the
// reference's sequential channel order -- coalesced streaming without
// changing the float rounding of a single block's score.  A tree
// (warp-shuffle) reduction over channels would round differently, and a
// near-tie at the top-k boundary could then flip the selection.
//
// The head/layer combine is a second, per-block kernel.  Doing it in the last
// CTA of each block group (threadfence + atomic counter) put a serial tail of
// L2 round trips after the last unit: 17 us of a 53 us scorer.
#include "kvm_internal.cuh"
#include "kvm_kernels.h"

#include <atomic>

namespace kvm {

// ------------------------------------------------------------ summaries --

// [n][n_embd] F32 sums + counts -> channel-major layout (transpose through smem).
__global__ void upload_summaries_kernel(SummaryLayout s, uint32_t layer, uint32_t block0,
                                        uint32_t n, const float *__restrict__ sums,
                                        const uint32_t *__restrict__ counts) {
    __shared__ float tile[32][33];
    const uint32_t E = s.n_embd;
    const uint32_t i0 = blockIdx.x * 32u;
    const uint32_t e0 = blockIdx.y * 32u;
    for (uint32_t r = threadIdx.y; r < 32u; r += blockDim.y) {
        const uint32_t i = i0 + r;
        const uint32_t e = e0 + threadIdx.x;
        tile[r][threadIdx.x] = (i < n && e < E) ? sums[static_cast<size_t>(i) * E + e] : 0.0f;
    }
    __syncthreads();
    for (uint32_t r = threadIdx.y; r < 32u; r += blockDim.y) {
        const uint32_t e = e0 + r;
        const uint32_t i = i0 + threadIdx.x;
        if (i < n && e < E) {
            s.sum_t[sum_index(s, layer, e, block0 + i)] = tile[threadIdx.x][r];
        }
    }
    if (blockIdx.y == 0 && threadIdx.y == 0) {
        const uint32_t i = i0 + threadIdx.x;
        if (i < n) {
            const uint32_t c = counts[i];
            const size_t at = static_cast<size_t>(layer) * s.ldb + block0 + i;
            s.mean_tok[at] = c;
            // RawKvStore::mean_k: inv = 1.0f / (float)mean_tokens
            s.inv_tok[at] = c ? __fdiv_rn(1.0f, __uint2float_rn(c)) : 0.0f;
        }
    }
}

// Tiled layout -> [n][n_embd] rows (transpose through smem).
__global__ void download_summaries_kernel(SummaryLayout s, uint32_t layer, uint32_t block0,
                                          uint32_t n, float *__restrict__ sums) {
    __shared__ float tile[32][33];
    const uint32_t E = s.n_embd;
    const uint32_t i0 = blockIdx.x * 32u;
    const uint32_t e0 = blockIdx.y * 32u;
    for (uint32_t r = threadIdx.y; r < 32u; r += blockDim.y) {
        const uint32_t e = e0 + r;
        const uint32_t i = i0 + threadIdx.x;
        tile[r][threadIdx.x] = (i < n && e < E) ? s.sum_t[sum_index(s, layer, e, block0 + i)] : 0.0f;
    }
    __syncthreads();
    for (uint32_t r = threadIdx.y; r < 32u; r += blockDim.y) {
        const uint32_t i = i0 + r;
        const uint32_t e = e0 + threadIdx.x;
        if (i < n && e < E) sums[static_cast<size_t>(i) * E + e] = tile[threadIdx.x][r];
    }
}

// ----------------------------------------------------------------- query --

// qv[l][h][d] = (sum over the GQA group of q_sum, in group order) * invq and
// nq[l][h] = sum over d of qv*qv, both exactly as the reference loop computes
// them; invq = 1.0f / (q_count * g).
__global__ void query_prep_kernel(QueryState q, uint32_t n_head_kv, uint32_t n_head_q,
                                  uint32_t head_dim) {
    extern __shared__ float qv_s[];
    const uint32_t l = blockIdx.x;
    const uint32_t cnt = q.q_count[l];
    if (cnt == 0) return;
    const uint32_t g = n_head_kv == 0 ? 1u : n_head_q / n_head_kv;
    const uint32_t gg = g > 1u ? g : 1u;
    const float invq = __fdiv_rn(1.0f, __uint2float_rn(cnt * gg));
    const uint32_t E = n_head_kv * head_dim;
    const float *qs = q.q_sum + static_cast<size_t>(l) * n_head_q * head_dim;
    float *qv = q.qv + static_cast<size_t>(l) * E;
    for (uint32_t i = threadIdx.x; i < E; i += blockDim.x) {
        const uint32_t h = i / head_dim;
        const uint32_t d = i % head_dim;
        // the group members' values are loaded together, then added in order
        const uint32_t n_in = min(g, n_head_q > h * g ? n_head_q - h * g : 0u);
        float qh = 0.0f;
        for (uint32_t g0 = 0; g0 < n_in; g0 += 8u) {
            float x[8];
#pragma unroll
            for (uint32_t k = 0; k < 8u; ++k)
                x[k] = g0 + k < n_in ? qs[static_cast<size_t>(h * g + g0 + k) * head_dim + d] : 0.0f;
#pragma unroll
            for (uint32_t k = 0; k < 8u; ++k)
                if (g0 + k < n_in) qh = __fadd_rn(qh, x[k]);
        }
        const float v = __fmul_rn(qh, invq);
        qv[i] = v;
        qv_s[i] = v;
    }
    __syncthreads();
    // nq per head: the reference's sequential sum over d, one thread per head,
    // reading the prepared vector from shared memory
    for (uint32_t h = threadIdx.x; h < n_head_kv; h += blockDim.x) {
        float nq = 0.0f;
        const float *v = qv_s + static_cast<size_t>(h) * head_dim;
#pragma unroll 16
        for (uint32_t d = 0; d < head_dim; ++d) nq = __fadd_rn(nq, __fmul_rn(v[d], v[d]));
        q.nq[static_cast<size_t>(l) * n_head_kv + h] = nq;
    }
}

// ---------------------------------------------------------------- scorer --

// One CTA = (group of kScoreBlocks blocks, one KV head, one layer): D*256
// contiguous bytes of the tiled summary tensor.  Each thread owns one block
// and keeps kScoreBatch coalesced channel loads in flight, then walks the
// channels in the reference's order.  Small units (2048 at config 2) and
// small CTAs (~14 per SM) make one balanced wave.  Per-head results go to rbuf; the last CTA of a
// block range (over heads x layers) forms the per-layer terms in head order
// and, when combining, the final scores in layer order.
__global__ void __launch_bounds__(kScoreThreads) score_kernel(ScoreArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    float *q_s = reinterpret_cast<float *>(smem);
    const uint32_t H = a.n_head_kv;
    const uint32_t D = a.head_dim;
    const uint32_t ldb = a.sum.ldb;
    const uint32_t g = blockIdx.x;
    const uint32_t h = blockIdx.y;
    const uint32_t l = a.layer0 + blockIdx.z;
    const uint32_t b0 = g * kScoreBlocks;
    const uint32_t nb = min(static_cast<uint32_t>(kScoreBlocks), a.n_blocks - b0);
    const bool active = a.q_count[l] > 0;
    const int tid = threadIdx.x;
    for (uint32_t i = tid; i < D; i += blockDim.x)
        q_s[i] = active ? a.qv[(static_cast<size_t>(l) * H + h) * D + i] : 0.0f;
    __syncthreads();
    {
        // One thread per block.  Channel c of the unit is the 256-byte row
        // h*D + c of tile (l, g): a warp's 32 loads of one channel are one
        // 128-byte line.  kScoreBatch channels are loaded at once, then added
        // in the reference's channel order.
        const uint32_t b = b0 + tid;
        const bool mine = active && static_cast<uint32_t>(tid) < nb;
        const float inv = mine ? a.sum.inv_tok[static_cast<size_t>(l) * ldb + b] : 0.0f;
        float dot = 0.0f;
        float nk = 0.0f;
        if (inv != 0.0f) {
            const float *col = a.sum.sum_t + sum_index(a.sum, l, h * D, b0) + tid;
            for (uint32_t c0 = 0; c0 < D; c0 += kScoreBatch) {
                float x[kScoreBatch];
#pragma unroll
                for (uint32_t r = 0; r < static_cast<uint32_t>(kScoreBatch); ++r)
                    x[r] = c0 + r < D ? __ldcs(col + static_cast<size_t>(c0 + r) * kSumGroup) : 0.0f;
#pragma unroll
                for (uint32_t r = 0; r < static_cast<uint32_t>(kScoreBatch); ++r) {
                    if (c0 + r < D) {
                        const float mk = __fmul_rn(x[r], inv);
                        dot = __fadd_rn(dot, __fmul_rn(q_s[c0 + r], mk));
                        nk = __fadd_rn(nk, __fmul_rn(mk, mk));
                    }
                }
            }
        }
        if (static_cast<uint32_t>(tid) < nb) {
            float rr = 0.0f;
            if (active) {
                const float den = __fadd_rn(__fmul_rn(__fsqrt_rn(a.nq[static_cast<size_t>(l) * H + h]),
                                                      __fsqrt_rn(nk)), 1e-6f);
                rr = __fdiv_rn(dot, den);
            }
            a.rbuf[(static_cast<size_t>(l) * H + h) * ldb + b] = rr;
        }
    }
}

// x / d in double; a power-of-two d divides exactly by scaling, so the
// product with its reciprocal is the same value as the quotient.
__device__ __forceinline__ double div_exact_pow2(double x, uint32_t d) {
    if ((d & (d - 1u)) == 0u) return __dmul_rn(x, 1.0 / static_cast<double>(d));
    return __ddiv_rn(x, static_cast<double>(d));
}

// Combine of the scorer's per-head results (llama-memory-kvmem.cpp:2881-2912):
// the layer term is the sum over heads in head order (double) divided by
// n_head_kv; the score is the sum of the active layers' terms in layer order
// divided by their number, 0 for a block without statistics.  A CTA covers
// kCombineBlocks blocks x kCombineLanes layer lanes: each thread forms the
// terms of its layers (their head values loaded together, coalesced across
// the blocks), parks them in shared memory, and one thread per block then
// adds them in layer order.
constexpr uint32_t kCombineBlocks = 32;
constexpr uint32_t kCombineLanes = 8;

__global__ void __launch_bounds__(kCombineBlocks * kCombineLanes) combine_kernel(ScoreArgs a) {
    extern __shared__ double term_s[];                 // [n_layers][kCombineBlocks]
    const uint32_t tb = threadIdx.x % kCombineBlocks;
    const uint32_t ly = threadIdx.x / kCombineBlocks;
    const uint32_t bb = blockIdx.x * kCombineBlocks + tb;
    const uint32_t H = a.n_head_kv;
    const uint32_t ldb = a.sum.ldb;
    const bool mine = bb < a.n_blocks;
    if (mine) {
        for (uint32_t li = ly; li < a.n_layers; li += kCombineLanes) {
            const uint32_t ll = a.layer0 + li;
            const float *rb = a.rbuf + static_cast<size_t>(ll) * H * ldb + bb;
            double term = 0.0;
            if (a.q_count[ll] > 0) {
                double layer = 0.0;
                for (uint32_t h0 = 0; h0 < H; h0 += 8u) {
                    float x[8];
#pragma unroll
                    for (uint32_t k = 0; k < 8u; ++k)
                        x[k] = h0 + k < H ? rb[static_cast<size_t>(h0 + k) * ldb] : 0.0f;
#pragma unroll
                    for (uint32_t k = 0; k < 8u; ++k)
                        if (h0 + k < H) layer = __dadd_rn(layer, static_cast<double>(x[k]));
                }
                term = div_exact_pow2(layer, H > 1u ? H : 1u);
            }
            a.terms[static_cast<size_t>(ll) * a.ldt + bb] = term;
            term_s[li * kCombineBlocks + tb] = term;
        }
    }
    if (!a.combine) return;
    __syncthreads();
    if (ly != 0 || !mine) return;
    double acc = 0.0;
    uint32_t nlay = 0;
    for (uint32_t li = 0; li < a.n_layers; ++li) {
        if (a.q_count[a.layer0 + li] > 0) {
            acc = __dadd_rn(acc, term_s[li * kCombineBlocks + tb]);
            ++nlay;
        }
    }
    bool has = false;
    for (uint32_t ll = 0; ll < a.sum.n_layer; ++ll)
        has |= a.sum.mean_tok[static_cast<size_t>(ll) * ldb + bb] > 0u;
    a.scores[bb] = (has && nlay) ? div_exact_pow2(acc, nlay) : 0.0;
}

__global__ void reduce_terms_kernel(const double *__restrict__ terms, uint32_t n_layers,
                                    uint32_t ldt, uint32_t n_blocks, double *__restrict__ acc) {
    const uint32_t b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n_blocks) return;
    double a = 0.0;
    for (uint32_t l = 0; l < n_layers; ++l) a = __dadd_rn(a, terms[static_cast<size_t>(l) * ldt + b]);
    acc[b] = a;
}

__global__ void scores_from_sum_kernel(SummaryLayout s, uint32_t n_blocks,
                                       const double *__restrict__ acc, uint32_t n_active,
                                       double *__restrict__ scores) {
    const uint32_t b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n_blocks) return;
    bool has = false;
    for (uint32_t l = 0; l < s.n_layer; ++l) has |= s.mean_tok[static_cast<size_t>(l) * s.ldb + b] > 0u;
    scores[b] = (has && n_active) ? __ddiv_rn(acc[b], static_cast<double>(n_active)) : 0.0;
}

// ------------------------------------------------------------- launchers --

cudaError_t launch_upload_summaries(const SummaryLayout &s, uint32_t layer, uint32_t block0,
                                    uint32_t n, const float *d_sums, const uint32_t *d_counts,
                                    cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    dim3 grid((n + 31u) / 32u, (s.n_embd + 31u) / 32u);
    dim3 block(32, 8);
    upload_summaries_kernel<<<grid, block, 0, stream>>>(s, layer, block0, n, d_sums, d_counts);
    return cudaGetLastError();
}

cudaError_t launch_download_summaries(const SummaryLayout &s, uint32_t layer, uint32_t block0,
                                      uint32_t n, float *d_sums, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    dim3 grid((n + 31u) / 32u, (s.n_embd + 31u) / 32u);
    download_summaries_kernel<<<grid, dim3(32, 8), 0, stream>>>(s, layer, block0, n, d_sums);
    return cudaGetLastError();
}

cudaError_t launch_query_prep(const QueryState &q, uint32_t n_layer, uint32_t n_head_kv,
                              uint32_t n_head_q, uint32_t head_dim, cudaStream_t stream) {
    const size_t smem = static_cast<size_t>(n_head_kv) * head_dim * sizeof(float);
    if (smem > 48u * 1024u)
        cudaFuncSetAttribute(query_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    query_prep_kernel<<<n_layer, 1024, smem, stream>>>(q, n_head_kv, n_head_q, head_dim);
    return cudaGetLastError();
}

// The hardware fills an SM with as many resident CTAs as its shared memory
// allows before it uses the next one, so a one-wave grid smaller than the
// GPU's capacity lands unevenly (measured: busiest SM active 83K cycles, the
// least busy 42K, of 89K).  Padding each CTA's shared memory caps residency at
// ceil(units / SMs) and so spreads the wave over every SM.
static size_t score_smem_for(uint32_t units, size_t smem_min) {
    // per host thread: sessions on different threads must not race on it
    static thread_local size_t cache_smem[64] = {};
    static thread_local uint32_t cache_units[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return smem_min;
    if (cache_units[dev] == units && cache_smem[dev] >= smem_min) return cache_smem[dev];
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int want = static_cast<int>((units + static_cast<uint32_t>(sms) - 1u) / static_cast<uint32_t>(sms));
    size_t smem = smem_min;
    int occ = 0;
    for (int it = 0; it < 512; ++it) {
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, score_kernel, kScoreThreads, smem) != cudaSuccess)
            return smem_min;
        if (occ <= want || smem >= 200u * 1024u) break;
        smem += 256u;
    }
    if (occ < want) smem = smem_min;       // never cap below one wave
    cache_units[dev] = units;
    cache_smem[dev] = smem;
    return smem;
}

cudaError_t launch_score(const ScoreArgs &a, cudaStream_t stream) {
    if (a.n_blocks == 0 || a.n_layers == 0) return cudaSuccess;
    const size_t smem_min = (a.head_dim * sizeof(float) + 127u) & ~static_cast<size_t>(127u);
    cudaError_t e = cudaFuncSetAttribute(score_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    dim3 grid((a.n_blocks + kScoreBlocks - 1u) / kScoreBlocks, a.n_head_kv, a.n_layers);
    const size_t smem = score_smem_for(grid.x * grid.y * grid.z, smem_min);
    score_kernel<<<grid, kScoreThreads, smem, stream>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const size_t csmem = static_cast<size_t>(a.n_layers) * kCombineBlocks * sizeof(double);
    if (csmem > 48u * 1024u) {
        e = cudaFuncSetAttribute(combine_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(csmem));
        if (e != cudaSuccess) return e;
    }
    combine_kernel<<<(a.n_blocks + kCombineBlocks - 1u) / kCombineBlocks, kCombineBlocks * kCombineLanes,
                     csmem, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_reduce_terms(const double *terms, uint32_t n_layers, uint32_t ldt,
                                uint32_t n_blocks, double *acc, cudaStream_t stream) {
    if (n_blocks == 0) return cudaSuccess;
    reduce_terms_kernel<<<(n_blocks + 255u) / 256u, 256, 0, stream>>>(terms, n_layers, ldt, n_blocks, acc);
    return cudaGetLastError();
}

cudaError_t launch_scores_from_sum(const SummaryLayout &s, uint32_t n_blocks, const double *acc,
                                   uint32_t n_active, double *scores, cudaStream_t stream) {
    if (n_blocks == 0) return cudaSuccess;
    scores_from_sum_kernel<<<(n_blocks + 255u) / 256u, 256, 0, stream>>>(s, n_blocks, acc, n_active,
                                                                        scores);
    return cudaGetLastError();
}

}  // namespace kvm
