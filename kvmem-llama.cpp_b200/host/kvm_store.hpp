// kvm_store.hpp -- C++ host mirror of the reference's block store, backed by
// libkvm on a B200.
//
// Same names, argument meanings and error behaviour as kvmem::KvMemStore
// (kvmem/include/kvmem/kvmem_store.hpp:329-487) for the members on the
// reselection path, so an adapter written against kvmem::KvMemStore (such as
// llama_memory_kvmem, src/adapter/llama-memory-kvmem.cpp) can swap the type:
//   register_append, block_count, total_tokens, budget_blocks,
//   set_retrieval_scores, pick_topk_blocks(mandatory), pick_semantic_groups,
//   set_selection(ids),
//   set_block_tier, set_block_gpu_slot, clear_working_set.
// The block table lives on the device: pick_topk_blocks and set_selection run
// the selector / diff kernels and read their results back (one bounded wait
// each).  Errors throw like the reference: std::invalid_argument for a bad
// configuration, std::runtime_error for device failures.
//
// The GPU-native extensions (scoring, stage-in) are reachable through
// session() and the C ABI in kvm.h.
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "kvm.h"

namespace kvm {

enum class KvTier : uint8_t { GPU = 0, CPU = 1, SSD = 2 };

struct KvMemRemap {
    uint32_t block_id = 0;
    uint32_t n_tokens = 0;
    int32_t from_base = 0;
    int32_t to_base = 0;
    bool working_k_resident = false;
    bool skip = false;
    bool raw_refresh = false;
};

struct KvMemPlan {
    std::vector<uint32_t> stage_in;
    std::vector<uint32_t> stage_out;
    std::vector<KvMemRemap> remaps;
    uint32_t total_window_tokens = 0;
    uint32_t selection_overlap_blocks = 0;
    uint32_t gpu_reused_blocks = 0;
    uint32_t retained_position_stable = 0;
    uint32_t retained_position_moved = 0;
    // chronological layout (layout_gpu_slots_by_orig_pos): slot i = selected[i]
    std::vector<uint32_t> selected;
    struct Move { uint32_t block_id; int32_t from; int32_t to; };
    std::vector<Move> moves;
    struct Cold { uint32_t block_id; int32_t to; };
    std::vector<Cold> cold;
};

struct KvMemStoreConfig {
    // KvMemStoreConfig fields used by the reselection path
    uint32_t block_tokens = 128;
    uint32_t select_budget = 131072;
    uint32_t gen_budget = 32768;         // window slots beyond the budget (gen-reserve)
    uint32_t sink_blocks = 1;
    uint32_t recent_blocks = 0;
    bool optimize_stage_in = true;
    bool immutable_source_k = false;
    uint32_t immutable_refresh_remaps = 8;
    uint64_t immutable_refresh_abs_delta_tokens = 262144;
    uint64_t immutable_max_baked_position = 262144;
    // device-side shape of the session
    uint32_t n_layer = 1;
    uint32_t n_head_kv = 4;
    uint32_t head_dim = 256;
    uint32_t n_head_q = 24;
    uint32_t max_blocks = 8192;
    int32_t type_k = KVM_TYPE_Q8_0;
    int32_t type_v = KVM_TYPE_Q8_0;
};

class KvMemStore {
public:
    explicit KvMemStore(KvMemStoreConfig cfg, int device = 0, kvm_stream stream = nullptr,
                        uint32_t timeout_ms = 30000)
        : cfg_(cfg), stream_(stream), timeout_ms_(timeout_ms) {
        kvm_config c;
        kvm_config_default(&c);
        c.block_tokens = cfg.block_tokens;
        c.select_budget = cfg.select_budget;
        c.gen_reserve = cfg.gen_budget;
        c.sink_blocks = cfg.sink_blocks;
        c.recent_blocks = cfg.recent_blocks;
        c.optimize_stage_in = cfg.optimize_stage_in ? 1u : 0u;
        c.immutable_source_k = cfg.immutable_source_k ? 1u : 0u;
        c.immutable_refresh_remaps = cfg.immutable_refresh_remaps;
        c.immutable_refresh_abs_delta_tokens = cfg.immutable_refresh_abs_delta_tokens;
        c.immutable_max_baked_position = cfg.immutable_max_baked_position;
        c.n_layer = cfg.n_layer;
        c.n_head_kv = cfg.n_head_kv;
        c.head_dim = cfg.head_dim;
        c.n_head_q = cfg.n_head_q;
        c.max_blocks = cfg.max_blocks;
        c.type_k = cfg.type_k;
        c.type_v = cfg.type_v;
        const kvm_status st = kvm_session_create(&c, device, &s_);
        if (st == KVM_EINVAL) throw std::invalid_argument(kvm_last_error(nullptr));
        if (st != KVM_OK) throw std::runtime_error(kvm_last_error(nullptr));
    }
    ~KvMemStore() { kvm_session_destroy(s_); }
    KvMemStore(const KvMemStore &) = delete;
    KvMemStore &operator=(const KvMemStore &) = delete;

    const KvMemStoreConfig &config() const { return cfg_; }
    uint32_t block_count() const { return kvm_block_count(s_); }
    uint32_t total_tokens() const { return total_tokens_; }
    uint32_t budget_blocks() const { return cfg_.select_budget / cfg_.block_tokens; }
    kvm_session *session() const { return s_; }

    // New blocks are GPU-tier without a window slot, as the reference store
    // leaves them (KvMemBlock::tier defaults to GPU, gpu_slot to -1).
    void register_append(uint32_t n_new_tokens) {
        if (n_new_tokens == 0) return;
        const uint32_t before = block_count();
        check(kvm_register_append(s_, stream_, n_new_tokens, 0));
        for (uint32_t id = before; id < block_count(); ++id)
            check(kvm_set_block_tier(s_, stream_, id, KVM_TIER_GPU));
        total_tokens_ += n_new_tokens;
    }

    void set_retrieval_scores(const std::vector<double> &scores) {
        check(kvm_set_scores(s_, stream_, scores.data(), static_cast<uint32_t>(scores.size())));
    }

    std::vector<uint32_t> pick_topk_blocks(const std::vector<uint32_t> &mandatory = {}) {
        check(kvm_select(s_, stream_, mandatory.data(), static_cast<uint32_t>(mandatory.size())));
        std::vector<uint32_t> sel(std::max<uint32_t>(1u, block_count()));
        kvm_plan p{};
        p.capacity = static_cast<uint32_t>(sel.size());
        p.selected = sel.data();
        check(kvm_get_plan(s_, stream_, &p, timeout_ms_));
        sel.resize(p.n_selected);
        return sel;
    }

    // KvMemStore::pick_semantic_groups (kvmem_store.cpp:625-756): whole
    // variable-length groups of half-open token spans under the block budget.
    std::vector<uint32_t> pick_semantic_groups(const std::vector<std::pair<uint32_t, uint32_t>> &groups,
                                               const std::vector<double> &group_scores,
                                               const std::vector<uint32_t> &mandatory_blocks = {}) {
        if (groups.size() != group_scores.size())
            throw std::runtime_error("KVMem semantic group spans/scores size mismatch");
        std::vector<uint32_t> spans(2 * groups.size());
        for (size_t i = 0; i < groups.size(); ++i) {
            spans[2 * i] = groups[i].first;
            spans[2 * i + 1] = groups[i].second;
        }
        check(kvm_select_groups(s_, stream_, spans.data(), group_scores.data(),
                                static_cast<uint32_t>(groups.size()), mandatory_blocks.data(),
                                static_cast<uint32_t>(mandatory_blocks.size())));
        std::vector<uint32_t> sel(std::max<uint32_t>(1u, block_count()));
        kvm_plan p{};
        p.capacity = static_cast<uint32_t>(sel.size());
        p.selected = sel.data();
        check(kvm_get_plan(s_, stream_, &p, timeout_ms_));
        sel.resize(p.n_selected);
        return sel;
    }

    KvMemPlan set_selection(std::vector<uint32_t> selected_ids, bool force_raw_refresh = false) {
        check(kvm_set_selection_ids(s_, stream_, selected_ids.data(),
                                    static_cast<uint32_t>(selected_ids.size())));
        check(kvm_diff(s_, stream_, force_raw_refresh ? 1 : 0));
        const uint32_t cap = std::max<uint32_t>(1u, block_count());
        KvMemPlan out;
        std::vector<uint32_t> sel(cap), si(cap), so(cap), rb(cap), rn(cap), mb(cap), cb(cap);
        std::vector<int32_t> rf(cap), rt(cap), mf(cap), mt(cap), ct(cap);
        std::vector<uint8_t> rw(cap), rs(cap), rr(cap);
        kvm_plan p{};
        p.capacity = cap;
        p.selected = sel.data();
        p.stage_in = si.data();
        p.stage_out = so.data();
        p.rm_block_id = rb.data();
        p.rm_n_tokens = rn.data();
        p.rm_from_base = rf.data();
        p.rm_to_base = rt.data();
        p.rm_working_k_resident = rw.data();
        p.rm_skip = rs.data();
        p.rm_raw_refresh = rr.data();
        p.mv_block = mb.data();
        p.mv_from = mf.data();
        p.mv_to = mt.data();
        p.cold_block = cb.data();
        p.cold_to = ct.data();
        check(kvm_get_plan(s_, stream_, &p, timeout_ms_));
        out.stage_in.assign(si.begin(), si.begin() + p.n_stage_in);
        out.stage_out.assign(so.begin(), so.begin() + p.n_stage_out);
        out.selected.assign(sel.begin(), sel.begin() + p.n_selected);
        out.remaps.resize(p.n_remaps);
        for (uint32_t i = 0; i < p.n_remaps; ++i) {
            out.remaps[i] = KvMemRemap{rb[i], rn[i], rf[i], rt[i], rw[i] != 0, rs[i] != 0, rr[i] != 0};
        }
        for (uint32_t i = 0; i < p.n_moves; ++i) out.moves.push_back({mb[i], mf[i], mt[i]});
        for (uint32_t i = 0; i < p.n_cold; ++i) out.cold.push_back({cb[i], ct[i]});
        out.total_window_tokens = p.total_window_tokens;
        out.selection_overlap_blocks = p.selection_overlap_blocks;
        out.gpu_reused_blocks = p.gpu_reused_blocks;
        out.retained_position_stable = p.retained_position_stable;
        out.retained_position_moved = p.retained_position_moved;
        return out;
    }

    void set_block_tier(uint32_t block_id, KvTier tier, int32_t /*cpu_slot*/ = -1,
                        int32_t /*nvme_slot*/ = -1) {
        check(kvm_set_block_tier(s_, stream_, block_id, static_cast<int32_t>(tier)));
    }
    void set_block_gpu_slot(uint32_t block_id, int32_t gpu_slot) {
        check(kvm_set_block_gpu_slot(s_, stream_, block_id, gpu_slot));
    }
    // Reset working-set membership and window residency (a new session).
    void clear_working_set() { check(kvm_reset_window(s_, stream_)); }

private:
    void check(kvm_status st) const {
        if (st == KVM_OK) return;
        const std::string m = kvm_last_error(s_);
        if (st == KVM_EINVAL) throw std::invalid_argument(m);
        throw std::runtime_error(m);
    }

    KvMemStoreConfig cfg_;
    kvm_stream stream_ = nullptr;
    uint32_t timeout_ms_ = 30000;
    kvm_session *s_ = nullptr;
    uint32_t total_tokens_ = 0;
};

}  // namespace kvm
