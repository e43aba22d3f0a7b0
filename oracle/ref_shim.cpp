// ref_shim.cpp -- TEST INFRASTRUCTURE ONLY.
//
// extern "C" wrappers around the reference's own libkvmem (KvMemStore,
// RawKvStore), compiled from the reference sources where they lie by
// oracle/Makefile into oracle/_ref/libkvmem_ref.so.  Used to pin the C
// restatement (kvm_oracle.c) and to generate tests/golden fixtures.  Nothing
// in the product links this.
#include "kvmem/kvmem_store.hpp"
#include "kvmem/raw_kv_store.hpp"
#include "kvmem/rope.hpp"

#include <cstdint>
#include <cstring>
#include <exception>
#include <vector>

extern "C" {

struct ref_cfg {
    uint32_t block_tokens;
    uint32_t select_budget;     // tokens
    uint32_t sink_blocks;
    uint32_t recent_blocks;
    uint32_t optimize_stage_in;
    uint32_t immutable_source_k;
    uint32_t immutable_refresh_remaps;
    uint32_t pad0;
    uint64_t immutable_refresh_abs_delta_tokens;
    uint64_t immutable_max_baked_position;
};

void *ref_store_new(const ref_cfg *c) {
    kvmem::KvMemStoreConfig cfg;
    cfg.block_tokens = c->block_tokens;
    cfg.select_budget = c->select_budget;
    cfg.sink_blocks = c->sink_blocks;
    cfg.recent_blocks = c->recent_blocks;
    cfg.optimize_stage_in = c->optimize_stage_in != 0;
    cfg.immutable_source_k = c->immutable_source_k != 0;
    cfg.immutable_refresh_remaps = c->immutable_refresh_remaps;
    cfg.immutable_refresh_abs_delta_tokens = c->immutable_refresh_abs_delta_tokens;
    cfg.immutable_max_baked_position = c->immutable_max_baked_position;
    return new kvmem::KvMemStore(cfg);
}

void ref_store_free(void *s) { delete static_cast<kvmem::KvMemStore *>(s); }

void ref_register_append(void *s, uint32_t n) {
    static_cast<kvmem::KvMemStore *>(s)->register_append(n);
}

uint32_t ref_block_count(void *s) {
    return static_cast<kvmem::KvMemStore *>(s)->block_count();
}

void ref_set_retrieval_scores(void *s, const double *scores, uint32_t n) {
    std::vector<double> v(scores, scores + n);
    static_cast<kvmem::KvMemStore *>(s)->set_retrieval_scores(v);
}

uint32_t ref_pick_topk(void *s, const uint32_t *mand, uint32_t n_mand, uint32_t *out) {
    std::vector<uint32_t> m(mand, mand + n_mand);
    auto sel = static_cast<kvmem::KvMemStore *>(s)->pick_topk_blocks(m);
    std::memcpy(out, sel.data(), sel.size() * sizeof(uint32_t));
    return static_cast<uint32_t>(sel.size());
}

uint32_t ref_pick_semantic_groups(void *s, const uint32_t *spans, const double *scores, uint32_t n_groups,
                                  const uint32_t *mand, uint32_t n_mand, uint32_t *out) {
    std::vector<std::pair<uint32_t, uint32_t>> g(n_groups);
    for (uint32_t i = 0; i < n_groups; ++i) g[i] = {spans[2 * i], spans[2 * i + 1]};
    std::vector<double> sc(scores, scores + n_groups);
    std::vector<uint32_t> m(mand, mand + n_mand);
    auto sel = static_cast<kvmem::KvMemStore *>(s)->pick_semantic_groups(g, sc, m);
    std::memcpy(out, sel.data(), sel.size() * sizeof(uint32_t));
    return static_cast<uint32_t>(sel.size());
}

// Plan arrays must hold block_count() entries.  Returns 0, or -1 on a throw.
int ref_set_selection(void *s, const uint32_t *ids, uint32_t n_ids, int force_raw,
                      uint32_t *stage_in, uint32_t *n_stage_in,
                      uint32_t *stage_out, uint32_t *n_stage_out,
                      uint32_t *rm_block, uint32_t *rm_ntok, int32_t *rm_from,
                      int32_t *rm_to, uint8_t *rm_wkr, uint8_t *rm_skip,
                      uint8_t *rm_raw, uint32_t *n_remaps, uint32_t *counters) {
    try {
        std::vector<uint32_t> v(ids, ids + n_ids);
        auto p = static_cast<kvmem::KvMemStore *>(s)->set_selection(v, force_raw != 0);
        *n_stage_in = static_cast<uint32_t>(p.stage_in.size());
        std::memcpy(stage_in, p.stage_in.data(), p.stage_in.size() * 4);
        *n_stage_out = static_cast<uint32_t>(p.stage_out.size());
        std::memcpy(stage_out, p.stage_out.data(), p.stage_out.size() * 4);
        *n_remaps = static_cast<uint32_t>(p.remaps.size());
        for (size_t i = 0; i < p.remaps.size(); ++i) {
            rm_block[i] = p.remaps[i].block_id;
            rm_ntok[i] = p.remaps[i].n_tokens;
            rm_from[i] = p.remaps[i].from_base;
            rm_to[i] = p.remaps[i].to_base;
            rm_wkr[i] = p.remaps[i].working_k_resident;
            rm_skip[i] = p.remaps[i].skip;
            rm_raw[i] = p.remaps[i].raw_refresh;
        }
        counters[0] = p.total_window_tokens;
        counters[1] = p.selection_overlap_blocks;
        counters[2] = p.gpu_reused_blocks;
        counters[3] = p.retained_position_stable;
        counters[4] = p.retained_position_moved;
        return 0;
    } catch (const std::exception &) {
        return -1;
    }
}

void ref_set_block_tier(void *s, uint32_t id, int tier, int32_t cpu_slot, int32_t nvme_slot) {
    static_cast<kvmem::KvMemStore *>(s)->set_block_tier(
        id, static_cast<kvmem::KvTier>(tier), cpu_slot, nvme_slot);
}

void ref_set_block_gpu_slot(void *s, uint32_t id, int32_t slot) {
    static_cast<kvmem::KvMemStore *>(s)->set_block_gpu_slot(id, slot);
}

void ref_clear_working_set(void *s) {
    static_cast<kvmem::KvMemStore *>(s)->clear_working_set();
}

// Block table snapshot (structure of arrays, block_count() entries each).
void ref_get_blocks(void *s, uint32_t *n_tokens, uint8_t *tier, int32_t *gpu_slot,
                    int64_t *baked_pos, uint32_t *remap_count,
                    uint64_t *remap_abs_delta, uint8_t *in_ws) {
    const auto &bl = static_cast<kvmem::KvMemStore *>(s)->blocks();
    for (size_t i = 0; i < bl.size(); ++i) {
        n_tokens[i] = bl[i].n_tokens;
        tier[i] = static_cast<uint8_t>(bl[i].tier);
        gpu_slot[i] = bl[i].gpu_slot;
        baked_pos[i] = bl[i].baked_pos;
        remap_count[i] = bl[i].remap_count;
        remap_abs_delta[i] = bl[i].remap_abs_delta;
        in_ws[i] = bl[i].in_working_set;
    }
}

void *ref_raw_new(uint32_t n_layer, uint32_t n_embd, uint32_t block_tokens) {
    kvmem::RawKvStoreConfig cfg;
    cfg.n_layer = n_layer;
    cfg.n_embd_k = n_embd;
    cfg.n_embd_v = n_embd;
    cfg.block_tokens = block_tokens;
    cfg.k_row_bytes = static_cast<uint64_t>(n_embd) + 64;  // opaque: no F16 fallback
    return new kvmem::RawKvStore(cfg);
}

void ref_raw_free(void *r) { delete static_cast<kvmem::RawKvStore *>(r); }

void ref_raw_write_mean_k(void *r, uint32_t pos0, uint32_t n, uint32_t il, const float *k) {
    static_cast<kvmem::RawKvStore *>(r)->write_layer_mean_k(pos0, n, il, k);
}

void ref_raw_write_mean_sum(void *r, uint32_t pos0, uint32_t n, uint32_t il, const float *sum) {
    static_cast<kvmem::RawKvStore *>(r)->write_layer_mean_sum(pos0, n, il, sum);
}

void ref_raw_mean_k(void *r, uint32_t block_id, uint32_t il, float *out) {
    static_cast<kvmem::RawKvStore *>(r)->mean_k(block_id, il, out);
}

void ref_rope_neox(uint32_t n_rot, uint32_t head_dim, uint32_t n_head, float freq_base, float freq_scale,
                   const float *k, uint32_t n_tokens, int32_t pos0, float *out) {
    kvmem::RopeConfig cfg;
    cfg.n_rot = n_rot;
    cfg.n_embd_head = head_dim;
    cfg.n_head_kv = n_head;
    cfg.freq_base = freq_base;
    cfg.freq_scale = freq_scale;
    kvmem::rope_neox_apply(cfg, k, n_tokens, pos0, out);
}

int ref_raw_has_block(void *r, uint32_t block_id) {
    return static_cast<kvmem::RawKvStore *>(r)->has_block(block_id) ? 1 : 0;
}

}  // extern "C"
