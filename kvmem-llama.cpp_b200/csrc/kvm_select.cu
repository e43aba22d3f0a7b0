// kvm_select.cu -- top-k block selection on the device.
//
// KvMemStore::pick_topk_blocks(mandatory) -> pick_topk_ungrouped, TopK policy
// (kvmem/src/host/kvmem_store.cpp:357-359, :482-623):
//   n <= budget (or budget 0): every block, ascending.
//   else keep sinks 0..min(sink,n)-1, then the mandatory list walked from its
//   end (newest first), then the `recent` newest blocks, each only while
//   fewer than `budget` are kept; fill the remaining `need` slots with the
//   best other blocks ordered by score descending, then block id descending.
//
// One CTA of 1024 threads per session.  The sink/mandatory/recent pins are a
// short sequential walk (thread 0, exactly the reference's order).  The fill
// is a radix select over an order-preserving 64-bit key of the f64 score: a
// one-bit first digit (the key's sign half, counted with the bits the half's
// keys share), then 8-bit digits below those bits, find the need-th best
// score T; every candidate above T is taken, and among candidates equal to T
// the ones with the highest block ids are taken -- the reference's strict
// total order (score, id), so the selected set is identical to its
// nth_element.  -0.0 and +0.0 compare equal as in the reference; NaN scores
// (undefined behaviour in the reference's comparator) rank below every
// number.
#include "kvm_diff.cuh"
#include "kvm_internal.cuh"
#include "kvm_kernels.h"

#include <atomic>

namespace kvm {

__device__ __forceinline__ uint64_t score_key(double s) {
    if (s != s) return 0ull;
    if (s == 0.0) s = 0.0;
    const uint64_t u = static_cast<uint64_t>(__double_as_longlong(s));
    return (u & 0x8000000000000000ull) ? ~u : (u | 0x8000000000000000ull);
}

// Ascending compaction of flags[i] != 0 (i < n) into out; returns the count.
__device__ uint32_t compact_flags(const uint8_t *flags, uint32_t n, uint32_t *out,
                                  uint32_t *scratch) {
    const uint32_t per = (n + kSelectThreads - 1u) / kSelectThreads;
    const uint32_t lo = min(n, threadIdx.x * per);
    const uint32_t hi = min(n, lo + per);
    uint32_t c = 0;
    for (uint32_t i = lo; i < hi; ++i) c += flags[i] != 0;
    uint32_t total;
    uint32_t off = block_exclusive_scan<kSelectThreads>(c, scratch, &total);
    for (uint32_t i = lo; i < hi; ++i)
        if (flags[i]) out[off++] = i;
    return total;
}

// The selection into kept[] (n bytes of shared memory: nonzero = selected)
// and a.selected (ascending); returns the selected count to every thread.
// Called by every thread of a kSelectThreads CTA.
//
// The radix select first picks the key half (top bit) that holds the
// threshold, then starts at the highest bit in which two keys of that half
// differ (the bits above it are common to all of them) and resolves 8 bits a
// pass.  Histogram counts are aggregated per warp (__match_any_sync: early
// passes put most keys in one bin), and
// the histogram is double-buffered so a pass needs two barriers.  The taken
// candidates and the ascending compaction come out of one block scan: the
// candidates equal to the threshold key that are taken are the `rem` with the
// highest ids, i.e. the equal ones after the first (equal total - rem).
static __device__ uint32_t select_core(const SelectArgs &a, uint8_t *kept) {
    __shared__ uint4 scratch4[kSelectThreads / 32 + 1];
    __shared__ uint32_t hist[2][256];
    __shared__ uint32_t s_red[9][kSelectThreads / 32];
    __shared__ uint32_t s_kc;
    __shared__ uint32_t s_remaining;
    __shared__ uint64_t s_prefix;
    __shared__ uint64_t s_mask;
    __shared__ int32_t s_hi;           // highest unresolved key bit, -1 when none
    const uint32_t n = a.n_blocks;
    const uint32_t budget = a.budget;
    const uint32_t tid = threadIdx.x;
    const uint32_t lane = tid & 31u;
    if (n == 0) {
        if (tid == 0) a.hdr->n_selected = 0;
        return 0u;
    }
    if (budget == 0 || n <= budget) {
        for (uint32_t i = tid; i < n; i += kSelectThreads) {
            a.selected[i] = i;
            kept[i] = 1;
        }
        if (tid == 0) a.hdr->n_selected = n;
        __syncthreads();
        return n;
    }
    for (uint32_t i = tid; i < n; i += kSelectThreads) kept[i] = 0;
    for (uint32_t i = tid; i < 512u; i += kSelectThreads) (&hist[0][0])[i] = 0u;
    __syncthreads();
    if (tid == 0) {
        uint32_t kc = 0;
        const uint32_t sink = min(a.sink, n);
        for (uint32_t i = 0; i < sink && kc < budget; ++i)
            if (!kept[i]) { kept[i] = 1; ++kc; }
        for (uint32_t i = a.n_mandatory; i > 0 && kc < budget; --i) {
            const uint32_t id = a.mandatory[i - 1];
            if (id < n && !kept[id]) { kept[id] = 1; ++kc; }
        }
        const uint32_t recent = min(a.recent, n);
        for (uint32_t i = 0; i < recent && kc < budget; ++i) {
            const uint32_t id = n - 1 - i;
            if (!kept[id]) { kept[id] = 1; ++kc; }
        }
        s_kc = kc;
    }
    __syncthreads();
    const uint32_t kc = s_kc;
    const uint32_t need = budget - kc;
    const uint32_t n_cand = n - kc;
    const bool take_all = need > 0 && need >= n_cand;
    const bool radix = need > 0 && !take_all;
    // Each thread owns the contiguous ids [lo, hi); up to kKeysCached keys
    // stay in registers across the passes.
    constexpr uint32_t kKeysCached = 8;
    const uint32_t per = (n + kSelectThreads - 1u) / kSelectThreads;
    const uint32_t lo = min(n, tid * per);
    const uint32_t hi = min(n, lo + per);
    const bool cached = per <= kKeysCached;
    uint64_t kcache[kKeysCached];
    uint32_t live = 0;                        // bit j: id lo + j is a candidate
#pragma unroll
    for (uint32_t j = 0; j < kKeysCached; ++j) {
        kcache[j] = 0ull;
        if (radix && cached && lo + j < hi && !kept[lo + j]) {
            kcache[j] = score_key(a.scores[lo + j]);
            live |= 1u << j;
        }
    }
    // f(j, live, key) for every owned slot j < per: a count uniform over the
    // CTA (warp-wide intrinsics in f see every lane); live is false past hi.
    // Cached keys are indexed with compile-time j (registers, no select chain).
    auto for_keys = [&](auto &&f) {
        if (cached) {
#pragma unroll
            for (uint32_t j = 0; j < kKeysCached; ++j)
                if (j < per) f(j, ((live >> j) & 1u) != 0u, kcache[j]);
        } else {
            for (uint32_t j = 0; j < per; ++j) {
                const bool lv = radix && lo + j < hi && !kept[lo + j];
                f(j, lv, lv ? score_key(a.scores[lo + j]) : 0ull);
            }
        }
    };
    uint64_t thr = 0ull, msk = 0ull;
    uint32_t rem = 0;
    if (radix) {
        // The candidates split by the key's top bit (scores >= 0 above the
        // negative ones and NaN): the count of the upper half says which half
        // holds the threshold -- a one-bit first digit -- and the AND and OR
        // of that half's keys give the leading bits all of its keys share, so
        // the passes start at the highest bit in which two of them differ.
        // Word r of a thread: AND / OR (low, high) of the upper half, the same
        // of the lower half, the upper count.
        uint64_t and1 = ~0ull, or1 = 0ull, and0 = ~0ull, or0 = 0ull;
        uint32_t c1 = 0;
        for_keys([&](uint32_t, bool lv, uint64_t k) {
            if (!lv) return;
            if (k >> 63) {
                and1 &= k;
                or1 |= k;
                ++c1;
            } else {
                and0 &= k;
                or0 |= k;
            }
        });
        uint32_t r[9] = {static_cast<uint32_t>(and1), static_cast<uint32_t>(and1 >> 32),
                         static_cast<uint32_t>(or1),  static_cast<uint32_t>(or1 >> 32),
                         static_cast<uint32_t>(and0), static_cast<uint32_t>(and0 >> 32),
                         static_cast<uint32_t>(or0),  static_cast<uint32_t>(or0 >> 32), c1};
        auto warp_reduce = [&]() {
#pragma unroll
            for (int w = 0; w < 8; w += 4) {
                r[w] = __reduce_and_sync(0xffffffffu, r[w]);
                r[w + 1] = __reduce_and_sync(0xffffffffu, r[w + 1]);
                r[w + 2] = __reduce_or_sync(0xffffffffu, r[w + 2]);
                r[w + 3] = __reduce_or_sync(0xffffffffu, r[w + 3]);
            }
            r[8] = __reduce_add_sync(0xffffffffu, r[8]);
        };
        warp_reduce();
        if (lane == 0) {
#pragma unroll
            for (int w = 0; w < 9; ++w) s_red[w][tid >> 5] = r[w];
        }
        __syncthreads();
        if (tid < 32) {
            const bool in = lane < kSelectThreads / 32;
#pragma unroll
            for (int w = 0; w < 9; ++w) {
                const uint32_t neutral = (w < 8 && (w & 2) == 0) ? ~0u : 0u;   // AND words: all ones
                r[w] = in ? s_red[w][lane] : neutral;
            }
            warp_reduce();
            if (lane == 0) {
                const bool upper = r[8] >= need;
                const int w0 = upper ? 0 : 4;
                const uint64_t A = (static_cast<uint64_t>(r[w0 + 1]) << 32) | r[w0];
                const uint64_t O = (static_cast<uint64_t>(r[w0 + 3]) << 32) | r[w0 + 2];
                const uint64_t x = A ^ O;   // never bit 63: it is the half's own
                const int hb = x ? 63 - __clzll(static_cast<long long>(x)) : -1;
                const uint64_t common = hb < 0 ? ~0ull : ~((2ull << hb) - 1ull);
                s_prefix = A & common;
                s_mask = common;
                s_hi = hb;
                // the lower half: every upper candidate is above the threshold
                s_remaining = upper ? need : need - r[8];
            }
        }
        __syncthreads();
        for (uint32_t pass = 0; s_hi >= 0; ++pass) {
            const int hib = s_hi;
            const int lob = hib >= 7 ? hib - 7 : 0;
            const uint32_t dmask = (1u << (hib - lob + 1)) - 1u;
            const uint64_t prefix = s_prefix;
            const uint64_t mask = s_mask;
            uint32_t *H = hist[pass & 1u];
            for_keys([&](uint32_t, bool lv, uint64_t k) {
                const uint32_t d = (lv && (k & mask) == prefix) ? static_cast<uint32_t>(k >> lob) & dmask
                                                                : 0xffffffffu;
                const uint32_t peers = __match_any_sync(0xffffffffu, d);
                if (d != 0xffffffffu && lane == static_cast<uint32_t>(__ffs(peers) - 1))
                    atomicAdd(&H[d], static_cast<uint32_t>(__popc(peers)));
            });
            uint32_t *Hn = hist[(pass + 1u) & 1u];
            for (uint32_t i = tid; i < 256u; i += kSelectThreads) Hn[i] = 0u;
            __syncthreads();
            if (tid < 32) {
                // lane l owns bins 255-8l .. 248-8l (highest digits first)
                const uint32_t r0 = s_remaining;   // read before any lane writes it
                uint32_t local = 0;
                for (int q = 0; q < 8; ++q) local += H[255u - 8u * lane - q];
                uint32_t cum = local;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const uint32_t y = __shfl_up_sync(0xffffffffu, cum, o);
                    if (lane >= static_cast<uint32_t>(o)) cum += y;
                }
                const uint32_t ex = cum - local;
                if (ex < r0 && r0 <= cum) {
                    uint32_t acc = ex;
                    for (int q = 0; q < 8; ++q) {
                        const uint32_t bin = 255u - 8u * lane - q;
                        const uint32_t hc = H[bin];
                        if (acc + hc >= r0) {
                            s_remaining = r0 - acc;
                            s_prefix = prefix | (static_cast<uint64_t>(bin) << lob);
                            s_mask = mask | (static_cast<uint64_t>(dmask) << lob);
                            // the whole bin is needed: every candidate with this
                            // prefix is taken, no further digit matters
                            s_hi = (acc + hc == r0) ? -1 : lob - 1;
                            break;
                        }
                        acc += hc;
                    }
                }
            }
            __syncthreads();
        }
        thr = s_prefix;
        msk = s_mask;
        rem = s_remaining;
    }
    // pins, candidates above the threshold, and the `rem` highest-id
    // candidates equal to it; one scan gives every offset of the ascending list
    uint32_t above = 0, eq = 0;
    for_keys([&](uint32_t j, bool lv, uint64_t k) {
        if (lo + j >= hi) return;
        if (kept[lo + j] || take_all) {
            ++above;
        } else if (lv) {
            k &= msk;
            if (k > thr) ++above;
            else if (k == thr) ++eq;
        }
    });
    uint4 tot;
    const uint4 off = block_exclusive_scan4<kSelectThreads>(make_uint4(above, eq, 0u, 0u), scratch4, &tot);
    const uint32_t e0 = tot.y > rem ? tot.y - rem : 0u;    // equal candidates not taken (lowest ids)
    uint32_t seen = off.y;
    uint32_t o = off.x + (off.y > e0 ? off.y - e0 : 0u);
    for_keys([&](uint32_t j, bool lv, uint64_t k) {
        const uint32_t i = lo + j;
        if (i >= hi) return;
        bool take = kept[i] != 0 || take_all;
        if (!take && lv) {
            k &= msk;
            if (k > thr) take = true;
            else if (k == thr) take = seen++ >= e0;
        }
        if (take) {
            if (!kept[i]) kept[i] = 2;
            a.selected[o++] = i;
        }
    });
    const uint32_t m = tot.x + (tot.y > e0 ? tot.y - e0 : 0u);
    if (tid == 0) a.hdr->n_selected = m;
    __syncthreads();
    return m;
}

__global__ void __launch_bounds__(kSelectThreads) select_kernel(SelectArgs a) {
    extern __shared__ uint8_t kept[];
    (void)select_core(a, kept);
}

// kvm_select followed by kvm_diff in one launch: the selection stays in
// shared memory as the diff's block flags, and the selected list is read
// back from the plan (written by this CTA, visible after the barrier).
static_assert(kSelectThreads == kDiffThreads, "one CTA runs both");

// L2 prefetch of [p, p + bytes), one 128-byte line a thread a round.
__device__ __forceinline__ void prefetch_l2(const void *p, size_t bytes) {
    const uintptr_t b0 = reinterpret_cast<uintptr_t>(p) & ~static_cast<uintptr_t>(127);
    const uintptr_t b1 = reinterpret_cast<uintptr_t>(p) + bytes;
    for (uintptr_t a = b0 + 128u * threadIdx.x; a < b1; a += 128u * blockDim.x)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(a));
}

__global__ void __launch_bounds__(kSelectThreads) select_diff_kernel(SelectArgs sa, DiffArgs da) {
    extern __shared__ uint8_t fl[];
    const uint32_t n = sa.n_blocks;
    // the scores and the block table were usually evicted from L2 by the
    // previous stage-in: start fetching all of them now, so the dependent
    // reads of the selection and the diff phases hit L2
    prefetch_l2(sa.scores, sizeof(double) * n);
    prefetch_l2(da.bt.in_ws, n);
    prefetch_l2(da.bt.tier, n);
    prefetch_l2(da.bt.gpu_slot, sizeof(int32_t) * n);
    prefetch_l2(da.bt.n_tokens, sizeof(uint32_t) * n);
    prefetch_l2(da.bt.baked_pos, sizeof(int64_t) * n);
    prefetch_l2(da.bt.remap_count, sizeof(uint32_t) * n);
    prefetch_l2(da.bt.remap_abs_delta, sizeof(uint64_t) * n);
    pdl_wait();                  // the scores (and any earlier write) are complete
    uint8_t *kept = fl;
    uint8_t *was = fl + (n ? n : 1u);
    const uint32_t m = select_core(sa, kept);
    // the stage-in's CTAs may now take SMs for their set-up (this grid's one
    // CTA is running); they wait for this kernel to finish before reading the plan
    pdl_launch_dependents();
    diff_core(da, min(m, n), kept, was, true);
}

// set_selection's canonicalisation: sort ascending, drop duplicates and ids
// >= n (kvmem_store.cpp:761-768), via a flag per block.
__global__ void __launch_bounds__(kSelectThreads) canon_ids_kernel(const uint32_t *ids,
                                                                   uint32_t n_ids, uint32_t n,
                                                                   uint32_t *selected,
                                                                   PlanHeader *hdr) {
    extern __shared__ uint8_t flag[];
    __shared__ uint32_t scratch[40];
    for (uint32_t i = threadIdx.x; i < n; i += kSelectThreads) flag[i] = 0;
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < n_ids; i += kSelectThreads) {
        const uint32_t id = ids[i];
        if (id < n) flag[id] = 1;
    }
    __syncthreads();
    const uint32_t m = compact_flags(flag, n, selected, scratch);
    if (threadIdx.x == 0) hdr->n_selected = m;
}

cudaError_t launch_select(const SelectArgs &a, cudaStream_t stream) {
    const size_t smem = a.n_blocks ? a.n_blocks : 1u;
    if (smem > 48u * 1024u)
        cudaFuncSetAttribute(select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    select_kernel<<<1, kSelectThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_select_diff(const SelectArgs &sa, const DiffArgs &da, cudaStream_t stream) {
    const size_t smem = 2u * (sa.n_blocks ? sa.n_blocks : 1u);
    if (smem > 48u * 1024u) {
        const cudaError_t e = cudaFuncSetAttribute(select_diff_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    return launch_after_prev(select_diff_kernel, dim3(1), dim3(kSelectThreads), smem, stream, sa, da);
}

cudaError_t launch_canon_ids(const uint32_t *ids, uint32_t n_ids, uint32_t n_blocks,
                             uint32_t *selected, PlanHeader *hdr, cudaStream_t stream) {
    const size_t smem = n_blocks ? n_blocks : 1u;
    if (smem > 48u * 1024u)
        cudaFuncSetAttribute(canon_ids_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    canon_ids_kernel<<<1, kSelectThreads, smem, stream>>>(ids, n_ids, n_blocks, selected, hdr);
    return cudaGetLastError();
}

// ------------------------------------------------------ semantic groups --
//
// KvMemStore::pick_semantic_groups (kvmem/src/host/kvmem_store.cpp:625-756):
// the same sink / mandatory / recent pins as pick_topk_blocks, then whole
// groups (half-open token spans, each covering every block it overlaps) in
// the order score desc, group id desc; a group whose not-yet-kept blocks do
// not fit in the remaining budget is skipped, never admitted in part; stop
// once the budget is full.  Blocks a group shares with kept ones are charged
// once.  The remaining budget is left unused, as in the reference.
//
// One CTA: candidates are built in parallel and sorted (bitonic, shared
// memory) on (score key + 1, group id) descending -- invalid spans get key 0
// and sink to the end; NaN scores rank below every number (the reference's
// comparator is undefined on NaN).  Warp 0 then walks the sorted groups in
// order; each group's new-block count and marking use the whole warp.
__global__ void __launch_bounds__(kSelectThreads) group_select_kernel(GroupSelectArgs a) {
    extern __shared__ __align__(16) uint8_t gsm[];
    __shared__ uint32_t scratch[40];
    __shared__ uint32_t s_kc;
    __shared__ uint32_t s_valid;
    const uint32_t n = a.n_blocks;
    const uint32_t budget = a.budget;
    const uint32_t tid = threadIdx.x;
    if (n == 0) {
        if (tid == 0) a.hdr->n_selected = 0;
        return;
    }
    if (budget == 0 || n <= budget) {
        for (uint32_t i = tid; i < n; i += kSelectThreads) a.selected[i] = i;
        if (tid == 0) a.hdr->n_selected = n;
        return;
    }
    uint32_t P = 1;
    while (P < a.n_groups) P <<= 1;
    uint64_t *key = reinterpret_cast<uint64_t *>(gsm);
    uint32_t *grp = reinterpret_cast<uint32_t *>(gsm + 8u * P);
    uint8_t *kept = gsm + 12u * P;
    for (uint32_t i = tid; i < n; i += kSelectThreads) kept[i] = 0;
    if (tid == 0) s_valid = 0;
    __syncthreads();
    if (tid == 0) {
        uint32_t kc = 0;
        const uint32_t sink = min(a.sink, n);
        for (uint32_t i = 0; i < sink && kc < budget; ++i)
            if (!kept[i]) { kept[i] = 1; ++kc; }
        for (uint32_t i = a.n_mandatory; i > 0 && kc < budget; --i) {
            const uint32_t id = a.mandatory[i - 1];
            if (id < n && !kept[id]) { kept[id] = 1; ++kc; }
        }
        const uint32_t recent = min(a.recent, n);
        for (uint32_t i = 0; i < recent && kc < budget; ++i) {
            const uint32_t id = n - 1 - i;
            if (!kept[id]) { kept[id] = 1; ++kc; }
        }
        s_kc = kc;
    }
    const uint32_t bt = max(1u, a.block_tokens);
    for (uint32_t g = tid; g < P; g += kSelectThreads) {
        uint64_t k = 0ull;
        if (g < a.n_groups) {
            const uint32_t begin = a.spans[2u * g];
            const uint32_t end = a.spans[2u * g + 1u];
            if (end > begin && begin < a.covered_tokens && begin / bt < n) {
                k = score_key(a.scores[g]) + 1ull;
                atomicAdd(&s_valid, 1u);
            }
        }
        key[g] = k;
        grp[g] = g;
    }
    __syncthreads();
    // bitonic sort, descending on (key, group)
    for (uint32_t size = 2; size <= P; size <<= 1) {
        for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
            for (uint32_t i = tid; i < P / 2u; i += kSelectThreads) {
                const uint32_t lo = 2u * stride * (i / stride) + (i % stride);
                const uint32_t hi = lo + stride;
                const bool desc = (lo & size) == 0u;
                const uint64_t kl = key[lo], kh = key[hi];
                const uint32_t gl = grp[lo], gh = grp[hi];
                const bool lo_first = kl > kh || (kl == kh && gl > gh);   // lo ranks ahead
                if (lo_first != desc) {
                    key[lo] = kh;
                    key[hi] = kl;
                    grp[lo] = gh;
                    grp[hi] = gl;
                }
            }
            __syncthreads();
        }
    }
    // the sorted groups' block ranges, packed into the key slots
    const uint32_t nv = s_valid;
    uint32_t *range = reinterpret_cast<uint32_t *>(key);
    for (uint32_t c = tid; c < nv; c += kSelectThreads) {
        const uint32_t g = grp[c];
        const uint32_t begin = a.spans[2u * g];
        const uint32_t end = min(a.spans[2u * g + 1u], a.covered_tokens);
        range[2u * c] = begin / bt;
        range[2u * c + 1u] = min((end - 1u) / bt, n - 1u);
    }
    __syncthreads();
    if (tid < 32) {
        const uint32_t lane = tid;
        uint32_t kc = s_kc;
        for (uint32_t c = 0; c < nv && kc < budget; ++c) {
            const uint32_t first = range[2u * c];
            const uint32_t last = range[2u * c + 1u];
            if (last - first >= budget - kc) {
                // more blocks than the remaining budget: fits only if enough are kept
                uint32_t fresh = 0;
                for (uint32_t id0 = first; id0 <= last; id0 += 32u) {
                    const uint32_t id = id0 + lane;
                    fresh += __popc(__ballot_sync(0xffffffffu, id <= last && !kept[id]));
                }
                if (fresh > budget - kc) continue;
            }
            uint32_t fresh = 0;
            for (uint32_t id0 = first; id0 <= last; id0 += 32u) {
                const uint32_t id = id0 + lane;
                const bool add = id <= last && !kept[id];
                fresh += __popc(__ballot_sync(0xffffffffu, add));
                if (add) kept[id] = 1;
            }
            __syncwarp();
            kc += fresh;
        }
    }
    __syncthreads();
    const uint32_t total = compact_flags(kept, n, a.selected, scratch);
    if (tid == 0) a.hdr->n_selected = total;
}

size_t group_select_smem(uint32_t n_groups, uint32_t n_blocks) {
    uint32_t P = 1;
    while (P < n_groups) P <<= 1;
    return 12u * static_cast<size_t>(P) + ((n_blocks + 15u) & ~15u);
}

cudaError_t launch_group_select(const GroupSelectArgs &a, cudaStream_t stream) {
    const size_t smem = group_select_smem(a.n_groups, a.n_blocks);
    if (smem > 200u * 1024u) return cudaErrorInvalidValue;
    static std::atomic<uint64_t> attr{0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!(attr.load(std::memory_order_acquire) & (1ull << dev))) {
        cudaError_t e = cudaFuncSetAttribute(group_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             200 * 1024);
        if (e != cudaSuccess) return e;
        attr.fetch_or(1ull << dev, std::memory_order_acq_rel);
    }
    group_select_kernel<<<1, kSelectThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace kvm
