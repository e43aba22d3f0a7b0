// ref_score.cpp -- TEST INFRASTRUCTURE ONLY.
//
// Runs the reference adapter's own scorer, llama_memory_kvmem::score_retrieval
// (src/adapter/llama-memory-kvmem.cpp:2869-2916), on given summaries and
// query sums.  The adapter as a whole cannot be compiled without llama.cpp,
// but that one member function reads only kvmem types (RawKvStore::has_block
// and mean_k, KvMemStore::block_count and set_retrieval_scores) and nine data
// members.  oracle/Makefile extracts the function's text unchanged from the
// reference file where it lies into _ref/score_retrieval.inc, a temporary
// that make deletes after the link; it is compiled here inside a stand-in
// class that declares just those members, against the reference's own
// libkvmem, with the reference's default x86-64 floating point (no FMA
// contraction).  The result pins the C restatement in kvm_oracle.c (and
// through it the device scorer) to the reference's code rather than to a
// second restatement.
#include "kvmem/kvmem_runtime.hpp"
#include "kvmem/raw_kv_store.hpp"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <exception>
#include <memory>
#include <vector>

// The members score_retrieval reads, with the reference header's types
// (src/adapter/llama-memory-kvmem.h:347-363, :423-424).
class llama_memory_kvmem {
public:
    void score_retrieval();

    std::unique_ptr<kvmem::KvMemRuntime> runtime_;
    std::unique_ptr<kvmem::RawKvStore> raw_;
    uint32_t n_layer_ = 0;
    uint32_t n_embd_k_ = 0;
    uint32_t n_head_ = 0;
    uint32_t n_head_kv_ = 0;
    uint32_t n_embd_head_ = 0;
    std::vector<std::vector<float>> q_sum_;
    std::vector<uint32_t> q_count_;
};

#include "score_retrieval.inc"

extern "C" {

struct ref_score_shape {
    uint32_t n_blocks;
    uint32_t block_tokens;
    uint32_t n_layer;
    uint32_t n_head_kv;
    uint32_t n_head;       // query heads
    uint32_t head_dim;
};

// A scorer over fixed summaries: sums [n_layer][n_blocks][n_head_kv*head_dim]
// F32 block sums of K, counts [n_layer][n_blocks] tokens summed (0 = no
// statistics; at most block_tokens).  Each sum is installed with
// RawKvStore::write_layer_mean_sum, as the decode harvest does.  Returns
// null when the reference threw.
void *ref_scorer_new(const ref_score_shape *s, const float *sums, const uint32_t *counts) {
    try {
        const uint32_t E = s->n_head_kv * s->head_dim;
        auto m = std::make_unique<llama_memory_kvmem>();
        kvmem::KvMemRuntimeConfig rc;
        rc.store.block_tokens = s->block_tokens;
        m->runtime_ = std::make_unique<kvmem::KvMemRuntime>(rc);
        m->runtime_->register_append(s->n_blocks * s->block_tokens);
        kvmem::RawKvStoreConfig cfg;
        cfg.n_layer = s->n_layer;
        cfg.n_embd_k = E;
        cfg.n_embd_v = E;
        cfg.block_tokens = s->block_tokens;
        cfg.k_row_bytes = static_cast<uint64_t>(E) + 64;   // opaque rows: mean-K statistics only
        m->raw_ = std::make_unique<kvmem::RawKvStore>(cfg);
        for (uint32_t il = 0; il < s->n_layer; ++il) {
            for (uint32_t b = 0; b < s->n_blocks; ++b) {
                const size_t at = static_cast<size_t>(il) * s->n_blocks + b;
                if (counts[at]) {
                    m->raw_->write_layer_mean_sum(b * s->block_tokens, counts[at], il, sums + at * E);
                }
            }
        }
        m->n_layer_ = s->n_layer;
        m->n_embd_k_ = E;
        m->n_head_ = s->n_head;
        m->n_head_kv_ = s->n_head_kv;
        m->n_embd_head_ = s->head_dim;
        m->q_sum_.assign(s->n_layer, std::vector<float>(static_cast<size_t>(s->n_head) * s->head_dim));
        m->q_count_.assign(s->n_layer, 0u);
        return m.release();
    } catch (const std::exception &) {
        return nullptr;
    }
}

void ref_scorer_free(void *h) { delete static_cast<llama_memory_kvmem *>(h); }

// One score_retrieval for query sums q_sum [n_layer][n_head*head_dim] and
// q_count [n_layer]; scores [n_blocks] out (the store's retrieval_score).
// Returns 0, or -1 when the reference threw.
int ref_scorer_run(void *h, const float *q_sum, const uint32_t *q_count, double *scores) {
    try {
        auto *m = static_cast<llama_memory_kvmem *>(h);
        const size_t qrow = static_cast<size_t>(m->n_head_) * m->n_embd_head_;
        for (uint32_t il = 0; il < m->n_layer_; ++il) {
            std::copy(q_sum + il * qrow, q_sum + (il + 1) * qrow, m->q_sum_[il].begin());
            m->q_count_[il] = q_count[il];
        }
        m->score_retrieval();
        const auto &blocks = m->runtime_->store().blocks();
        for (size_t b = 0; b < blocks.size(); ++b) scores[b] = blocks[b].retrieval_score;
        return 0;
    } catch (const std::exception &) {
        return -1;
    }
}

// ref_scorer_new + ref_scorer_run + ref_scorer_free.
int ref_score_retrieval(const ref_score_shape *s, const float *sums, const uint32_t *counts,
                        const float *q_sum, const uint32_t *q_count, double *scores) {
    void *h = ref_scorer_new(s, sums, counts);
    if (!h) return -1;
    const int rc = ref_scorer_run(h, q_sum, q_count, scores);
    ref_scorer_free(h);
    return rc;
}

}  // extern "C"
