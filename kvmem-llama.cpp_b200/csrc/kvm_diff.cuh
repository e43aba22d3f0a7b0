// kvm_diff.cuh -- the body of the selection diff, shared by diff_kernel
// (kvm_diff.cu) and the fused select + diff kernel (kvm_select.cu).
//
// KvMemStore::set_selection (kvmem/src/host/kvmem_store.cpp:758-882) on the
// device, for an already canonical (ascending, unique, in-range) selection:
//   stage_out = GPU-tier blocks not selected (or every GPU block when
//               optimize_stage_in is off), ascending; they leave the working set
//   stage_in  = selected blocks not in the working set, ascending
//   remaps    = one per selected block in window order: from_base = current
//               bake position, to_base = running window position, skip /
//               raw_refresh per the immutable-source rules; counters
//               selection_overlap / gpu_reused / retained_position_{stable,moved}
// plus the adapter's chronological layout (layout_gpu_slots_by_orig_pos,
// src/adapter/llama-memory-kvmem.cpp:931-1254, with reset_slots/alloc_slot):
// the i-th selected block ends in window slot i; a selected block already
// resident in another slot is moved (move list), a selected block not
// resident is gathered + quantized from the stored history (cold list);
// unselected GPU blocks lose their slot and drop to the CPU tier
// (KvMemRuntime::stage_out with no lower tier, kvmem_runtime.cpp:238-292).
//
// One CTA of kDiffThreads threads; per-block work is split into contiguous
// id chunks per thread so every output list comes out in ascending order
// from one block-wide exclusive scan.
#pragma once

#include "kvm_internal.cuh"
#include "kvm_kernels.h"

namespace kvm {

// KvMemStore::set_selection + the chronological layout for the `k` selected
// blocks in a.plan.selected.  Called by every thread of a kDiffThreads CTA.
// now / was: n bytes of shared memory each; with now_ready the caller has
// already set now[i] != 0 exactly for the selected blocks.  With
// a.reset_window the block table is first reset as kvm_reset_window does
// (nothing in the working set, GPU-tier blocks drop to the CPU tier, no
// slots): the reset is applied to the values as they are read and written
// back with the new layout.
//
// Three phases.  A: every thread reads its block chunk and its selection
// chunk and counts (stage_out, overlap | tokens, stage_in, moves, cold); one
// block-wide scan of the six counts gives every list offset.  B: the lists,
// the remaps and the working-set / bake updates, with the remaining four
// counters summed in shared memory.  C: the new layout (tier and slot of
// every block) and the plan header.
struct DiffView {                  // a block's table entry as the diff sees it
    uint8_t in_ws;
    uint8_t tier;
    int32_t slot;
};

__device__ __forceinline__ DiffView diff_view(const BlockTable &bt, uint32_t id, bool reset) {
    DiffView v{bt.in_ws[id], bt.tier[id], bt.gpu_slot[id]};
    if (reset) {
        v.in_ws = 0;
        if (v.tier == KVM_TIER_GPU) v.tier = KVM_TIER_CPU;
        v.slot = -1;
    }
    return v;
}

static __device__ void diff_core(const DiffArgs &a, uint32_t k, uint8_t *now, uint8_t *was,
                                 bool now_ready) {
    __shared__ uint4 scratch8[2 * (kDiffThreads / 32 + 1)];
    __shared__ uint32_t s_cnt[4];      // stable, moved, reused, errors
    const uint32_t n = a.n_blocks;
    PlanHeader *hdr = a.plan.hdr;
    const uint32_t tid = threadIdx.x;
    const bool reset = a.reset_window != 0;
    const uint32_t *sel = a.plan.selected;
    const bool ffr = a.optimize_stage_in == 0;
    const bool imm = a.immutable_source_k != 0;
    BlockTable bt = a.bt;

    if (!now_ready) {
        for (uint32_t i = tid; i < n; i += kDiffThreads) now[i] = 0;
        __syncthreads();
        for (uint32_t s = tid; s < k; s += kDiffThreads) {
            const uint32_t id = sel[s];
            if (id < n) now[id] = 1;
            else set_status(a.status, kErrIndex);
        }
        __syncthreads();
    }
    if (tid < 4) s_cnt[tid] = 0u;

    // ---- A: counts over this thread's block chunk and selection chunk
    const uint32_t per = (n + kDiffThreads - 1u) / kDiffThreads;
    const uint32_t lo = min(n, tid * per);
    const uint32_t hi = min(n, lo + per);
    const uint32_t sper = (k + kDiffThreads - 1u) / kDiffThreads;
    const uint32_t slo = min(k, tid * sper);
    const uint32_t shi = min(k, slo + sper);
    uint32_t overlap = 0, n_out = 0;
    for (uint32_t i = lo; i < hi; ++i) {
        const DiffView v = diff_view(bt, i, reset);
        was[i] = v.in_ws;
        overlap += (v.in_ws && now[i]) ? 1u : 0u;
        n_out += (v.tier == KVM_TIER_GPU && (!now[i] || ffr)) ? 1u : 0u;
    }
    uint32_t tok = 0, n_in = 0, n_mv = 0, n_cold = 0;
    for (uint32_t s = slo; s < shi; ++s) {
        const uint32_t id = sel[s];
        const DiffView v = diff_view(bt, id, reset);
        // a selected GPU block also leaves the working set when every GPU
        // block is staged out (optimize_stage_in off)
        const bool ws = v.in_ws && !(ffr && v.tier == KVM_TIER_GPU);
        tok += bt.n_tokens[id];
        n_in += ws ? 0u : 1u;
        const bool resident = !ffr && v.tier == KVM_TIER_GPU && v.slot >= 0;
        if (resident) n_mv += v.slot != static_cast<int32_t>(s) ? 1u : 0u;
        else ++n_cold;
    }
    uint4 c1 = make_uint4(n_out, overlap, tok, n_in), c2 = make_uint4(n_mv, n_cold, 0u, 0u);
    uint4 t1, t2;
    block_exclusive_scan8<kDiffThreads>(c1, c2, scratch8, &t1, &t2);   // was[] visible after it

    // ---- B: lists, remaps, working-set and bake updates
    uint32_t off_out = c1.x;
    for (uint32_t i = lo; i < hi; ++i) {
        const uint8_t t = bt.tier[i];
        if (t == KVM_TIER_GPU && !reset && (!now[i] || ffr)) a.plan.stage_out[off_out++] = i;
    }
    uint32_t wpos = c1.z, off_in = c1.w, off_mv = c2.x, off_cold = c2.y;
    uint32_t stable = 0, moved = 0, reused = 0, err = 0;
    for (uint32_t s = slo; s < shi; ++s) {
        const uint32_t id = sel[s];
        const DiffView v = diff_view(bt, id, reset);
        const int64_t baked = bt.baked_pos[id];
        const uint32_t ntok = bt.n_tokens[id];
        const bool reusable = was[id] && v.tier == KVM_TIER_GPU;
        if (reusable) {
            if (baked == static_cast<int64_t>(wpos)) ++stable;
            else ++moved;
            if (!ffr) ++reused;
        }
        const bool cold = v.tier != KVM_TIER_GPU || ffr;
        const bool ws = v.in_ws && !(ffr && v.tier == KVM_TIER_GPU);
        if (!ws) a.plan.stage_in[off_in++] = id;
        const bool wkr = !cold;
        const bool same = baked == static_cast<int64_t>(wpos);
        const bool skip = same && (!imm || wkr) && !a.force_raw_refresh;
        const uint64_t delta = static_cast<uint64_t>(baked > static_cast<int64_t>(wpos)
                                                         ? baked - static_cast<int64_t>(wpos)
                                                         : static_cast<int64_t>(wpos) - baked);
        bool raw = false;
        if (imm && (cold || !same)) {
            const uint64_t lim = a.immutable_refresh_abs_delta_tokens;
            const uint64_t have = bt.remap_abs_delta[id];
            const bool remap_limit = a.immutable_refresh_remaps > 0 &&
                                     bt.remap_count[id] >= a.immutable_refresh_remaps;
            const bool delta_limit = lim > 0 && (have >= lim || delta >= lim - (have < lim ? have : lim));
            const uint64_t maxp = a.immutable_max_baked_position;
            const bool out_of_range = maxp > 0 && (baked < 0 || static_cast<uint64_t>(baked) + ntok > maxp);
            raw = cold || remap_limit || delta_limit || out_of_range;
        }
        if (imm && a.force_raw_refresh) raw = true;
        if (skip && raw) ++err;   // std::logic_error in the reference (unreachable)
        a.plan.rm_block_id[s] = id;
        a.plan.rm_n_tokens[s] = ntok;
        a.plan.rm_from_base[s] = static_cast<int32_t>(baked);
        a.plan.rm_to_base[s] = static_cast<int32_t>(wpos);
        a.plan.rm_wkr[s] = wkr ? 1 : 0;
        a.plan.rm_skip[s] = skip ? 1 : 0;
        a.plan.rm_raw[s] = raw ? 1 : 0;
        // layout
        const bool resident = !ffr && v.tier == KVM_TIER_GPU && v.slot >= 0;
        if (resident) {
            if (v.slot != static_cast<int32_t>(s)) {
                a.plan.mv_block[off_mv] = id;
                a.plan.mv_from[off_mv] = v.slot;
                a.plan.mv_to[off_mv] = static_cast<int32_t>(s);
                ++off_mv;
            }
        } else {
            a.plan.cold_block[off_cold] = id;
            a.plan.cold_to[off_cold] = static_cast<int32_t>(s);
            ++off_cold;
        }
        if (s >= a.n_slots) err += 1u << 16;
        // working-set and bake updates
        bt.in_ws[id] = 1;
        if (!skip) {
            if (raw) {
                bt.remap_count[id] = 0;
                bt.remap_abs_delta[id] = 0;
            } else {
                bt.remap_count[id] += 1u;
                bt.remap_abs_delta[id] += delta;
            }
        }
        bt.baked_pos[id] = static_cast<int64_t>(wpos);
        wpos += ntok;
    }
    // the four counters: warp sums, one shared atomic each per warp
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        stable += __shfl_xor_sync(0xffffffffu, stable, o);
        moved += __shfl_xor_sync(0xffffffffu, moved, o);
        reused += __shfl_xor_sync(0xffffffffu, reused, o);
        err += __shfl_xor_sync(0xffffffffu, err, o);
    }
    if ((tid & 31u) == 0u && (stable | moved | reused | err)) {
        atomicAdd(&s_cnt[0], stable);
        atomicAdd(&s_cnt[1], moved);
        atomicAdd(&s_cnt[2], reused);
        atomicAdd(&s_cnt[3], err);
    }
    __syncthreads();   // every entry was read above; now install the layout

    // ---- C: the layout and the header.  Nothing here depends on order, and
    // the two loops write disjoint entries (unselected, then selected blocks),
    // so the threads take them strided: consecutive threads, consecutive
    // entries, coalesced stores.
    for (uint32_t i = tid; i < n; i += kDiffThreads) {
        if (now[i]) continue;
        // unselected GPU blocks are staged out (or dropped by the reset)
        const bool gpu = bt.tier[i] == KVM_TIER_GPU;
        if (reset || gpu) bt.in_ws[i] = 0;
        if (gpu) bt.tier[i] = KVM_TIER_CPU;
        bt.gpu_slot[i] = -1;
    }
    for (uint32_t s = tid; s < k; s += kDiffThreads) {
        const uint32_t id = sel[s];
        bt.tier[id] = KVM_TIER_GPU;
        bt.gpu_slot[id] = static_cast<int32_t>(s);
    }
    if (tid == 0) {
        hdr->n_stage_in = t1.w;
        hdr->n_stage_out = t1.x;
        hdr->n_remaps = k;
        hdr->total_window_tokens = t1.z;
        hdr->selection_overlap_blocks = t1.y;
        hdr->gpu_reused_blocks = s_cnt[2];
        hdr->retained_position_stable = s_cnt[0];
        hdr->retained_position_moved = s_cnt[1];
        hdr->n_moves = t2.x;
        hdr->n_cold = t2.y;
        hdr->n_blocks = n;
        if (s_cnt[3] & 0xffffu) set_status(a.status, kErrConfig);
        if (s_cnt[3] >> 16) set_status(a.status, kErrSlot);
    }
}

}  // namespace kvm
