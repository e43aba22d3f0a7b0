// kvm_score.cu -- mean-K summary upload/download and the block scorer.
//
// Scorer: llama_memory_kvmem::score_retrieval (src/adapter/llama-memory-kvmem.cpp:2869-2916),
// restated for the device without changing its arithmetic:
//   per (block, layer, kv head): dot/nk accumulate in float over d in order,
//     r = dot / (sqrt(nq) * sqrt(nk) + 1e-6f)
//   per (block, layer): layer = sum of r over heads in order (double), term = layer / H_kv
//   per block: score = (sum of terms over layers with a query, in layer order) / n_active
// The summaries are tiled ([layer][64-block group][channel/4][64][4]) so that
// a warp of threads, one per block, reads 512 contiguous bytes per four
// channels while each thread keeps the reference's sequential channel order
// -- coalesced 16-byte streaming without changing the float rounding of a
// single block's score.  A tree (warp-shuffle) reduction over channels would
// round differently, and a near-tie at the top-k boundary could then flip the
// selection.
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

// x / d in double; a power-of-two d divides exactly by scaling, so the
// product with its reciprocal is the same value as the quotient.
__device__ __forceinline__ double div_exact_pow2(double x, uint32_t d) {
    if ((d & (d - 1u)) == 0u) return __dmul_rn(x, 1.0 / static_cast<double>(d));
    return __ddiv_rn(x, static_cast<double>(d));
}

// ----------------------------------------------------------------- query --

// One CTA = (layer, KV head), one thread per channel:
//   qv[l][h][d] = (sum over the GQA group of q_sum, in group order) * invq,
//   invq = 1.0f / (q_count * g); nq[l][h] = sum over d of qv*qv in order.
// With ld.src (kvm_set_query of a device query) the CTA also copies its
// group's rows -- the last KV head's CTA also any heads past H * g -- into
// q.q_sum, each value as it is summed, and q_count comes from the launch
// parameters.
__global__ void query_prep_kernel(QueryState q, QueryLoad ld, uint32_t n_head_kv, uint32_t n_head_q,
                                  uint32_t head_dim) {
    extern __shared__ float qv_s[];
    const uint32_t l = blockIdx.x;
    const uint32_t h = blockIdx.y;
    const uint32_t D = head_dim;
    const uint32_t g = n_head_kv == 0 ? 1u : n_head_q / n_head_kv;
    const size_t row0 = static_cast<size_t>(l) * n_head_q * D;
    uint32_t cnt;
    if (ld.src) {
        // the source was written by earlier work on the stream, and a scorer
        // launched after this prep reads nothing of it before it waits
        pdl_wait();
        pdl_launch_dependents();
        cnt = ld.count[l];
        if (h == 0 && threadIdx.x == 0) q.q_count[l] = cnt;
    } else {
        pdl_launch_dependents();     // the scorer may start its summary loads now
        cnt = q.q_count[l];
    }
    const uint32_t n_in = min(g, n_head_q > h * g ? n_head_q - h * g : 0u);
    if (ld.src) {
        // rows this CTA does not sum below: all of them for a layer without
        // query, and the last KV head's heads past H * g
        const uint32_t c0 = h * g + (cnt == 0 ? 0u : n_in);
        const uint32_t c1 = h + 1u == n_head_kv ? n_head_q : min(n_head_q, h * g + g);
        for (size_t i = static_cast<size_t>(c0) * D + threadIdx.x; i < static_cast<size_t>(c1) * D; i += blockDim.x)
            q.q_sum[row0 + i] = ld.src[row0 + i];
    }
    if (cnt == 0) return;        // the scorer skips a layer without query
    const uint32_t gg = g > 1u ? g : 1u;
    const float invq = __fdiv_rn(1.0f, __uint2float_rn(cnt * gg));
    const size_t grp = row0 + static_cast<size_t>(h) * g * D;
    const float *qs = (ld.src ? ld.src : q.q_sum) + grp;
    for (uint32_t d = threadIdx.x; d < D; d += blockDim.x) {
        float qh = 0.0f;
        for (uint32_t g0 = 0; g0 < n_in; g0 += 8u) {
            float x[8];
#pragma unroll
            for (uint32_t k = 0; k < 8u; ++k)
                x[k] = g0 + k < n_in ? qs[static_cast<size_t>(g0 + k) * D + d] : 0.0f;
#pragma unroll
            for (uint32_t k = 0; k < 8u; ++k) {
                if (g0 + k < n_in) {
                    qh = __fadd_rn(qh, x[k]);
                    if (ld.src) q.q_sum[grp + static_cast<size_t>(g0 + k) * D + d] = x[k];   // the kept copy
                }
            }
        }
        const float v = __fmul_rn(qh, invq);
        q.qv[(static_cast<size_t>(l) * n_head_kv + h) * D + d] = v;
        qv_s[d] = v;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float nq = 0.0f;
#pragma unroll 16
        for (uint32_t d = 0; d < D; ++d) nq = __fadd_rn(nq, __fmul_rn(qv_s[d], qv_s[d]));
        q.nq[static_cast<size_t>(l) * n_head_kv + h] = nq;
    }
}

// ---------------------------------------------------------------- scorer --

// 16-byte global -> shared copy by this thread (L2 only), completing in the
// thread's current cp.async group.
__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gmem_src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// One CTA = (range of kScoreRange blocks = one summary tile, one layer);
// warp h scores KV head h of the range, one lane per block.  Per (block,
// head) the thread walks the head's channels in the reference's order; its
// next four channels are one 16-byte vector of the tiled summary tensor, so
// the warp's loads are consecutive 512-byte pieces of one contiguous
// head_dim*128-byte run.  Each lane streams its vectors through a ring of S
// shared-memory stages with cp.async (S vectors in flight, no registers
// held); the ring is filled before the CTA waits for the query prep (a
// programmatic dependent launch).  The per-layer term (heads in order,
// double, / H_kv) is formed in shared memory; with `combine`, the last CTA
// of a range to finish adds the layers' terms in layer order into the block
// scores.

template <bool VEC, int S>
__global__ void __launch_bounds__(1024) score_kernel(ScoreArgs a) {
    extern __shared__ __align__(16) float sm[];
    __shared__ uint32_t s_last;
    const uint32_t H = a.n_head_kv;
    const uint32_t D = a.head_dim;
    const uint32_t ldb = a.sum.ldb;
    const uint32_t h = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t l = a.layer0 + blockIdx.y;
    const uint32_t b = blockIdx.x * kScoreRange + lane;
    const bool mine = b < a.n_blocks;
    float4 *ring = reinterpret_cast<float4 *>(sm);                 // [H][S][32]
    float *qv_s = sm + static_cast<size_t>(H) * S * 128u;          // [H][D]
    float *r_s = qv_s + static_cast<size_t>(H) * D;                // [H][32]
    float *nq_s = r_s + H * 32u;                                   // [H]
    // before the wait only the summaries are read (q_count may still be
    // written by the prep): loads start for every block with statistics
    const float inv0 = mine ? a.sum.inv_tok[static_cast<size_t>(l) * ldb + b] : 0.0f;
    const bool load = inv0 != 0.0f;

    // summary vectors of (block b, head h): channel quad c of the head is at
    // vec[c * kSumGroup]; ring stage c % S of this lane at slot[(c % S) * 32]
    const uint32_t n4 = D / 4u;
    const float4 *vec = reinterpret_cast<const float4 *>(a.sum.sum_t) +
                        ((static_cast<size_t>(l) * (ldb / kSumGroup) + b / kSumGroup) * (a.sum.n_embd / 4u) +
                         (VEC ? h * n4 : 0u)) * kSumGroup + (b % kSumGroup);
    float4 *slot = ring + static_cast<size_t>(h) * S * 32u + lane;
    if (VEC && load) {
#pragma unroll
        for (int c = 0; c < S; ++c) {
            if (static_cast<uint32_t>(c) < n4) cp_async16(slot + c * 32, vec + static_cast<size_t>(c) * kSumGroup);
            cp_async_commit();
        }
    }
    pdl_wait();                  // the query prep's qv / nq / q_count are complete
    const bool active = a.q_count[l] > 0;
    const float inv = active ? inv0 : 0.0f;
    const bool go = load && active;
    if (VEC && load && !active) cp_async_wait<0>();   // a layer without query: drain the ring
    if (active) {
        const float *qg = a.qv + (static_cast<size_t>(l) * H + h) * D;
        for (uint32_t d = lane; d < D; d += 32u) qv_s[h * D + d] = qg[d];
        if (lane == 0) nq_s[h] = a.nq[static_cast<size_t>(l) * H + h];
    }
    __syncwarp();

    float dot = 0.0f;
    float nk = 0.0f;
    const float *q = qv_s + h * D;
    if (go) {
        if (VEC) {
            // group c is complete once at most S-1 later groups are pending;
            // its stage is refilled with vector c+S after its values are used
            uint32_t st = 0;
            for (uint32_t c = 0; c < n4; ++c) {
                cp_async_wait<S - 1>();
                const float4 x = slot[st * 32u];
                const float4 qq = *reinterpret_cast<const float4 *>(q + 4u * c);
                float mk = __fmul_rn(x.x, inv);
                dot = __fadd_rn(dot, __fmul_rn(qq.x, mk));
                nk = __fadd_rn(nk, __fmul_rn(mk, mk));
                mk = __fmul_rn(x.y, inv);
                dot = __fadd_rn(dot, __fmul_rn(qq.y, mk));
                nk = __fadd_rn(nk, __fmul_rn(mk, mk));
                mk = __fmul_rn(x.z, inv);
                dot = __fadd_rn(dot, __fmul_rn(qq.z, mk));
                nk = __fadd_rn(nk, __fmul_rn(mk, mk));
                mk = __fmul_rn(x.w, inv);
                dot = __fadd_rn(dot, __fmul_rn(qq.w, mk));
                nk = __fadd_rn(nk, __fmul_rn(mk, mk));
                if (c + S < n4) cp_async16(slot + st * 32u, vec + static_cast<size_t>(c + S) * kSumGroup);
                cp_async_commit();
                st = st + 1u == static_cast<uint32_t>(S) ? 0u : st + 1u;
            }
        } else {
            // head_dim not a multiple of 4: one channel at a time
            const uint32_t e0 = h * D;
            for (uint32_t d0 = 0; d0 < D; d0 += 8u) {
                float x[8];
#pragma unroll
                for (uint32_t k = 0; k < 8u; ++k)
                    x[k] = d0 + k < D ? __ldcs(a.sum.sum_t + sum_index(a.sum, l, e0 + d0 + k, b)) : 0.0f;
#pragma unroll
                for (uint32_t k = 0; k < 8u; ++k) {
                    if (d0 + k < D) {
                        const float mk = __fmul_rn(x[k], inv);
                        dot = __fadd_rn(dot, __fmul_rn(q[d0 + k], mk));
                        nk = __fadd_rn(nk, __fmul_rn(mk, mk));
                    }
                }
            }
        }
    }
    // r = dot / (sqrt(nq) * sqrt(nk) + 1e-6f) of (block, head)
    float rr = 0.0f;
    if (active)
        rr = __fdiv_rn(dot, __fadd_rn(__fmul_rn(__fsqrt_rn(nq_s[h]), __fsqrt_rn(nk)), 1e-6f));
    r_s[h * 32u + lane] = rr;
    __syncthreads();
    // only now may the dependent selection launch: every CTA of this grid
    // is resident by the time the last one gets here, so the dependent can
    // never hold an SM a CTA of this grid still waits for
    pdl_launch_dependents();
    if (h == 0 && mine) {
        // layer term: the heads' results summed in head order (double) / H
        double term = 0.0;
        if (active) {
            double layer = 0.0;
            for (uint32_t hh = 0; hh < H; ++hh) layer = __dadd_rn(layer, static_cast<double>(r_s[hh * 32u + lane]));
            term = div_exact_pow2(layer, H > 1u ? H : 1u);
        }
        a.terms[static_cast<size_t>(l) * a.ldt + b] = term;
    }
    if (!a.combine) return;
    // publish the terms, then count the range's arrivals; the last CTA of the
    // range adds the layers' terms in layer order
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&a.range_done[blockIdx.x], 1u) == gridDim.y - 1u ? 1u : 0u;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (h == 0 && mine) {
        double acc = 0.0;
        uint32_t nlay = 0;
        for (uint32_t l0 = 0; l0 < a.n_layers; l0 += 8u) {
            double t[8];
            uint32_t c[8];
#pragma unroll
            for (uint32_t k = 0; k < 8u; ++k) {
                const uint32_t ll = a.layer0 + l0 + k;
                const bool in = l0 + k < a.n_layers;
                c[k] = in ? a.q_count[ll] : 0u;
                t[k] = in ? __ldcg(a.terms + static_cast<size_t>(ll) * a.ldt + b) : 0.0;
            }
#pragma unroll
            for (uint32_t k = 0; k < 8u; ++k) {
                if (c[k] > 0u) {
                    acc = __dadd_rn(acc, t[k]);
                    ++nlay;
                }
            }
        }
        bool has = false;
        for (uint32_t ll = 0; ll < a.sum.n_layer; ++ll)
            has |= __ldcg(a.sum.mean_tok + static_cast<size_t>(ll) * ldb + b) > 0u;
        a.scores[b] = (has && nlay) ? div_exact_pow2(acc, nlay) : 0.0;
    }
    if (threadIdx.x == 0) a.range_done[blockIdx.x] = 0u;    // ready for the next launch
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

// The hardware fills an SM with as many resident CTAs as its resources allow
// before it uses the next one, so a one-wave grid smaller than the GPU's
// capacity lands unevenly (measured: busiest SM active 83K cycles, the least
// busy 42K, of 89K).  Padding each CTA's shared memory caps residency at
// ceil(units / SMs) and so spreads the wave over every SM.
// The hardware fills an SM with as many resident CTAs as its resources allow
// before it uses the next one, so a one-wave grid smaller than the GPU's
// capacity lands unevenly (measured: busiest SM active 83K cycles, the least
// busy 42K, of 89K).  Padding each CTA's shared memory caps residency at
// ceil(units / SMs) and so spreads the wave over every SM.
template <bool VEC, int S>
static size_t score_smem_for(uint32_t units, uint32_t threads, size_t smem_min) {
    // per host thread: sessions on different threads must not race on it
    static thread_local size_t cache_smem[64] = {};
    static thread_local uint32_t cache_units[64] = {};
    static thread_local uint32_t cache_threads[64] = {};
    static thread_local size_t cache_min[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return smem_min;
    if (cache_units[dev] == units && cache_threads[dev] == threads && cache_min[dev] == smem_min)
        return cache_smem[dev];
    const int sms = num_sms();
    const int want = static_cast<int>((units + static_cast<uint32_t>(sms) - 1u) / static_cast<uint32_t>(sms));
    size_t smem = smem_min;
    int occ = 0;
    for (int it = 0; it < 1024; ++it) {
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, score_kernel<VEC, S>, static_cast<int>(threads),
                                                          smem) != cudaSuccess)
            return smem_min;
        if (occ <= want || smem >= 200u * 1024u) break;
        smem += 256u;
    }
    if (occ < want) smem = smem_min;       // never cap below one wave
    cache_units[dev] = units;
    cache_threads[dev] = threads;
    cache_min[dev] = smem_min;
    cache_smem[dev] = smem;
    return smem;
}

template <bool VEC, int S>
static cudaError_t launch_score_t(const ScoreArgs &a, bool after_prep, cudaStream_t stream) {
    static std::atomic<uint64_t> attr{0};
    if (!attr_once(attr, reinterpret_cast<const void *>(score_kernel<VEC, S>), 200 * 1024))
        return cudaErrorInvalidValue;
    const uint32_t threads = 32u * a.n_head_kv;
    const size_t smem_min = (static_cast<size_t>(a.n_head_kv) * (S * 128u + a.head_dim + 33u) * sizeof(float) +
                             127u) & ~static_cast<size_t>(127u);
    dim3 grid((a.n_blocks + kScoreRange - 1u) / kScoreRange, a.n_layers);
    const size_t smem = score_smem_for<VEC, S>(grid.x * grid.y, threads, smem_min);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = after_prep ? 1u : 0u;
    return cudaLaunchKernelEx(&cfg, score_kernel<VEC, S>, a);
}

cudaError_t launch_query_load(const QueryState &q, const QueryLoad &ld, uint32_t n_layer, uint32_t n_head_kv,
                              uint32_t n_head_q, uint32_t head_dim, cudaStream_t stream) {
    if (n_layer == 0 || n_layer > kQueryInlineLayers || n_head_kv == 0 || head_dim == 0 || head_dim > 1024u ||
        ld.src == nullptr)
        return cudaErrorInvalidValue;
    return launch_after_prev(query_prep_kernel, dim3(n_layer, n_head_kv), dim3(head_dim),
                             static_cast<size_t>(head_dim) * sizeof(float), stream, q, ld, n_head_kv, n_head_q,
                             head_dim);
}

cudaError_t launch_score(const ScoreArgs &a, const QueryState *prep, uint32_t n_layer_all, cudaStream_t stream,
                         bool after_prep_load) {
    if (a.n_blocks == 0 || a.n_layers == 0) return cudaSuccess;
    if (a.n_head_kv == 0 || a.n_head_kv > 32u || a.head_dim == 0 || a.head_dim > 1024u)
        return cudaErrorInvalidValue;
    if (prep) {
        const size_t smem = static_cast<size_t>(a.head_dim) * sizeof(float);
        const QueryLoad none{};
        query_prep_kernel<<<dim3(n_layer_all, a.n_head_kv), a.head_dim, smem, stream>>>(*prep, none, a.n_head_kv,
                                                                                          a.n_head_q, a.head_dim);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    // ring depth: kScoreStages vectors a lane while the ring stays within
    // 48 KiB a CTA (up to 8 KV heads), 3 beyond
    const bool after = prep != nullptr || after_prep_load;
    if (a.head_dim % 4u != 0u) return launch_score_t<false, 1>(a, after, stream);
    if (a.n_head_kv <= 8u) return launch_score_t<true, kScoreStages>(a, after, stream);
    return launch_score_t<true, 3>(a, after, stream);
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
