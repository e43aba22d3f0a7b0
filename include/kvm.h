/*
 * kvm.h -- C ABI of libkvm, a B200-native (sm_100a) implementation of
 * KVMem's per-step KV reselection path:
 *
 *     score every stored 128-token block against the captured query
 *  -> select the top-k blocks within the budget (sinks pinned, mandatory
 *     blocks newest-first, ties to the higher block id)
 *  -> diff the selection against the resident window (KvMemPlan) and lay the
 *     window out chronologically (slot i = i-th selected block)
 *  -> move retained blocks in place and gather + quantize the newly selected
 *     F16 K/V blocks into ggml q8_0 / q4_0 / q5_0 rows of the window.
 *
 * Plain C types only; every pointer is a host pointer unless its name starts
 * with `d_` (device) or the comment says "host or device".  All calls return
 * a kvm_status and never throw.  Calls that take a `stream` are
 * stream-ordered and do not block the host, except where noted.  One session
 * serves one sequence on one device; sessions are independent and may be
 * used from different threads; one session is single-threaded.
 *
 * Deferred launches: kvm_select and kvm_reset_window record their work and
 * the next kvm_diff performs both inside its own launch (one kernel for
 * select + diff).  Any other call that depends on that work -- one that
 * rewrites the scores or the plan, reads or writes the block table, appends
 * blocks, waits or reads results -- launches it first, on that call's own
 * stream.  A correct program orders such a call after kvm_select /
 * kvm_reset_window anyway (same stream, or a wait between streams), so every
 * sequence of calls has the effect of running them in order.
 *
 * Reference interfaces this ABI replaces (paths in CrKcel/kvmem-llama.cpp):
 *   - llama_memory_kvmem::score_retrieval        src/adapter/llama-memory-kvmem.cpp:2869-2916
 *   - KvMemStore::pick_topk_blocks(mandatory)    kvmem/src/host/kvmem_store.cpp:357-359, :482-623
 *   - KvMemStore::set_selection -> KvMemPlan     kvmem/src/host/kvmem_store.cpp:758-882
 *   - layout_gpu_slots_by_orig_pos               src/adapter/llama-memory-kvmem.cpp:931-1254
 *   - write_block_to_gpu / kvmem_stagein_*       src/adapter/llama-memory-kvmem.cpp:2726-2791,
 *                                                src/adapter/llama-kvmem-stagein.h:12-62
 *   - RawKvStore mean-K summaries                kvmem/src/host/raw_kv_store.cpp:204-223, :674-720, :976-1043
 */
#ifndef KVM_H
#define KVM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KVM_ABI_VERSION 1

typedef struct kvm_session kvm_session;
/* A cudaStream_t passed as an opaque handle (NULL = legacy default stream). */
typedef void *kvm_stream;

typedef enum kvm_status {
    KVM_OK = 0,
    KVM_EINVAL = 1,    /* bad argument or configuration (std::invalid_argument) */
    KVM_ENOMEM = 2,    /* device or pinned allocation failed */
    KVM_ECUDA = 3,     /* CUDA runtime error; see kvm_last_error */
    KVM_ETIMEOUT = 4,  /* bounded host wait or device wait ran out */
    KVM_ESTATE = 5,    /* call out of order (e.g. stage-in before a diff) */
    KVM_EDEVICE = 6    /* a kernel reported an error flag (bad index, timeout) */
} kvm_status;

/* ggml_type ids (ggml.h enum ggml_type): the window cache formats F16, Q4_0,
 * Q5_0, Q8_0, and the captured-activation formats F32, F16, BF16. */
typedef enum kvm_type {
    KVM_TYPE_F32 = 0,
    KVM_TYPE_F16 = 1,
    KVM_TYPE_Q4_0 = 2,
    KVM_TYPE_Q5_0 = 6,
    KVM_TYPE_Q8_0 = 8,
    KVM_TYPE_BF16 = 30
} kvm_type;

/* Block tiers, kvmem/include/kvmem/kvmem_store.hpp:31 (enum class KvTier). */
typedef enum kvm_tier { KVM_TIER_GPU = 0, KVM_TIER_CPU = 1, KVM_TIER_SSD = 2 } kvm_tier;

/*
 * Session configuration: the subset of KvMemStoreConfig
 * (kvmem/include/kvmem/kvmem_store.hpp:231-327) and llama_kvmem_params
 * (src/adapter/llama-kvmem-hooks.h:19-39) that the reselection path reads.
 */
typedef struct kvm_config {
    uint32_t block_tokens;     /* --kvmem-block-tokens (128) */
    uint32_t select_budget;    /* --kvmem-budget, tokens; budget blocks = budget / block_tokens */
    uint32_t gen_reserve;      /* --kvmem-gen-reserve, tokens; window slots = ceil((budget+gen)/bt) */
    uint32_t sink_blocks;      /* always-kept prefix blocks (make_runtime_cfg maps 0 tokens -> 1) */
    uint32_t recent_blocks;    /* always-kept suffix blocks (0 = literal none) */
    uint32_t n_layer;          /* attention layers owned by this session */
    uint32_t n_head_kv;
    uint32_t head_dim;
    uint32_t n_head_q;
    uint32_t max_blocks;       /* block-table capacity (<= 65536) */
    int32_t  type_k;           /* kvm_type of the window K cache */
    int32_t  type_v;           /* kvm_type of the window V cache */
    uint32_t optimize_stage_in;        /* 0 = reload every selected block (ablation) */
    uint32_t immutable_source_k;       /* KvMemStoreConfig::immutable_source_k */
    uint32_t immutable_refresh_remaps;
    uint32_t reserved0;
    uint64_t immutable_refresh_abs_delta_tokens;
    uint64_t immutable_max_baked_position;
    uint64_t staging_bytes;    /* HBM ring for host-resident sources, allocated on the first
                                  host-source stage-in; 0 = 256 MiB */
} kvm_config;

/* Fill `cfg` with the reference defaults (kvmem_store.hpp:231-327 and the
 * adapter's make_runtime_cfg, llama-memory-kvmem.cpp:282-317). */
void kvm_config_default(kvm_config *cfg);

/*
 * F16 K/V of the stored history (what RawKvStore keeps on the host).
 * Element (layer l, block b, token t, channel e) of K is at byte offset
 *     l*layer_stride + b*block_stride + t*row_stride + 2*e
 * from `k` (same for V).  `location` says whether k/v are device (HBM)
 * pointers or pinned host pointers (cudaHostAlloc / cudaHostRegister).
 */
typedef enum kvm_location { KVM_LOC_DEVICE = 0, KVM_LOC_HOST = 1 } kvm_location;
typedef struct kvm_source {
    const void *k;
    const void *v;
    uint64_t layer_stride;
    uint64_t block_stride;
    uint64_t row_stride;
    int32_t  location;
    int32_t  reserved0;
} kvm_source;

/*
 * Packed (already quantized) K/V rows of the stored history: what the
 * reference's RawKvStore keeps after the harvest (write_layer_k_gpu /
 * write_layer_v_gpu, fed by harvest_gpu_v) and what kvm_stageout writes.  The
 * n_tokens rows of block b, layer l are contiguous, row_bytes_k apart, at
 *     k + l*k_layer_stride + b*k_block_stride
 * (V alike with the v_ strides and row_bytes_v).  A kvm_stageout destination
 * whose ids were 0, 1, 2, ... is such a source with
 *     k = dst, v = dst + block_tokens*row_bytes_k,
 *     k_layer_stride = v_layer_stride = block_tokens*(row_bytes_k + row_bytes_v),
 *     k_block_stride = v_block_stride = kvm_stageout_item_bytes(s).
 * `location` as in kvm_source.
 */
typedef struct kvm_packed_source {
    const void *k;
    const void *v;
    uint64_t k_layer_stride;
    uint64_t k_block_stride;
    uint64_t v_layer_stride;
    uint64_t v_block_stride;
    int32_t  location;
    int32_t  reserved0;
} kvm_packed_source;

/*
 * The bounded window (llama.cpp KV cache tensors, owned by the caller).
 * d_k[l] / d_v[l] are device base pointers of layer l's K / V cache; token t
 * of slot s lives at base + (s*block_tokens + t) * ggml_row_size(type, E).
 * The arrays themselves are host arrays of n_layer pointers.
 */
typedef struct kvm_window {
    void *const *d_k;
    void *const *d_v;
} kvm_window;

/* KvMemPlan plus the chronological slot layout, as host arrays.  Arrays are
 * caller-owned with capacity `capacity` entries (>= max_blocks); NULL arrays
 * are skipped.  Semantics follow kvmem_store.hpp:108-124. */
typedef struct kvm_plan {
    uint32_t capacity;
    uint32_t n_selected;                 /* selected blocks (ascending ids) */
    uint32_t *selected;                  /* slot i holds selected[i] */
    uint32_t n_stage_in;
    uint32_t *stage_in;
    uint32_t n_stage_out;
    uint32_t *stage_out;
    uint32_t n_remaps;                   /* == n_selected */
    uint32_t *rm_block_id;
    uint32_t *rm_n_tokens;
    int32_t  *rm_from_base;
    int32_t  *rm_to_base;
    uint8_t  *rm_working_k_resident;
    uint8_t  *rm_skip;
    uint8_t  *rm_raw_refresh;
    uint32_t total_window_tokens;
    uint32_t selection_overlap_blocks;
    uint32_t gpu_reused_blocks;
    uint32_t retained_position_stable;
    uint32_t retained_position_moved;
    uint32_t n_moves;                    /* resident blocks moved to a new slot */
    uint32_t *mv_block;
    int32_t  *mv_from;
    int32_t  *mv_to;
    uint32_t n_cold;                     /* blocks gathered + quantized from the source */
    uint32_t *cold_block;
    int32_t  *cold_to;
} kvm_plan;

/* Stage timers of the last step (CUDA events), in milliseconds; field names
 * follow the reference's KVMEM_RETR_SUM line (llama-memory-kvmem.cpp:2918-2936). */
typedef struct kvm_timings {
    float score_ms;
    float plan_ms;      /* select + diff */
    float layout_ms;    /* in-place moves of retained blocks */
    float set_ms;       /* gather + quantize stage-in (incl. H2D for host sources) */
    float total_ms;
} kvm_timings;

/* ------------------------------------------------------------ sessions -- */

/* Allocates the session's device state on `device` (summaries, block table,
 * plan buffers, staging ring).  Replaces the adapter-owned state built in
 * llama_memory_kvmem's constructor (llama-memory-kvmem.cpp:430-600). */
kvm_status kvm_session_create(const kvm_config *cfg, int device, kvm_session **out);
void kvm_session_destroy(kvm_session *s);
/* Last error message of this session (never NULL). */
const char *kvm_last_error(const kvm_session *s);
/* Window slots: ceil((select_budget + gen_reserve) / block_tokens)
 * (kvmem_compute_pool, llama-memory-kvmem.cpp:363-426, without the VRAM cap). */
uint32_t kvm_window_slots(const kvm_session *s);
uint32_t kvm_block_count(const kvm_session *s);
/* ggml_row_size(type, n_embd) */
uint64_t kvm_row_bytes(int32_t type, uint32_t n_embd);

/* --------------------------------------------------------- block table -- */

/* KvMemStore::register_append (kvmem_store.cpp:179-205): extend the trailing
 * partial block, then start new blocks.  `resident` = 0: the tokens exist
 * only in the stored history (tier CPU).  `resident` = 1: the model wrote
 * them into the window (tier GPU); new blocks take the next free window
 * slots (alloc_slot, llama-memory-kvmem.cpp:693-700): the lowest slots not
 * holding a block, which requires the previous step's plan to have been read
 * with kvm_get_plan.  The device block table is updated on `stream`. */
kvm_status kvm_register_append(kvm_session *s, kvm_stream stream, uint32_t n_new_tokens,
                               int resident);
/* KvMemStore::set_block_tier (kvmem_store.cpp:250-276): a tier other than
 * GPU also drops the block's window slot.  Stream-ordered. */
kvm_status kvm_set_block_tier(kvm_session *s, kvm_stream stream, uint32_t block_id,
                              int32_t tier);
/* KvMemStore::set_block_gpu_slot (kvmem_store.cpp:278-281): record that the
 * block's rows are in window slot `slot` (-1 = none).  Stream-ordered. */
kvm_status kvm_set_block_gpu_slot(kvm_session *s, kvm_stream stream, uint32_t block_id,
                                  int32_t slot);
/* KvMemStore::clear_working_set + drop every window slot: the next step
 * treats the window as empty (cold).  Stream-ordered on `stream`; the reset
 * is applied by the next kvm_diff inside its own launch (deferred launches,
 * above). */
kvm_status kvm_reset_window(kvm_session *s, kvm_stream stream);

/* ------------------------------------------------- summaries and query -- */

/*
 * RawKvStore mean-K statistics for `n` blocks of one layer: `sums` holds
 * [n][n_head_kv*head_dim] F32 token sums, `counts` [n] the tokens behind each
 * sum (0 = no statistics).  host or device pointers.  The mean is computed on
 * read as sum * (1.0f / count) exactly like RawKvStore::mean_k.
 */
kvm_status kvm_upload_summaries(kvm_session *s, kvm_stream stream, uint32_t layer,
                                uint32_t block0, uint32_t n, const float *sums,
                                const uint32_t *counts);
/* The inverse of kvm_upload_summaries: copy n blocks' F32 sums ([n][E]) and
 * counts of one layer to `sums` / `counts` (host or device pointers; either
 * may be NULL).  Stream-ordered.  Serves checkpoint/resume of a session
 * (RawKvStore::mean_checkpoint, raw_kv_store.cpp:1131-1164). */
kvm_status kvm_download_summaries(kvm_session *s, kvm_stream stream, uint32_t layer,
                                  uint32_t block0, uint32_t n, float *sums, uint32_t *counts);
/* GPU producer of the same statistics from F16 K rows of the source
 * (RawKvStore::add_mean_f32 over F16->F32 values, ordered token sum).  The
 * source must be device-resident.  Counts are the blocks' n_tokens. */
kvm_status kvm_summarize(kvm_session *s, kvm_stream stream, uint32_t layer0,
                         uint32_t n_layers, uint32_t block0, uint32_t n,
                         const kvm_source *src);
/*
 * A captured activation tensor in device memory, laid out like the ggml
 * tensor the attention graph hands to the capture hook
 * (patches/0002-attn-qk-capture-hook.patch): element (token t, head h,
 * dim d) is at data + t*nb_tok + h*nb_head + d*nb_dim (ggml nb[2], nb[1],
 * nb[0]).  `type` is KVM_TYPE_F32, KVM_TYPE_F16 or KVM_TYPE_BF16; values are
 * widened to F32 exactly.  n_head * head_dim must equal the row width the
 * call expects (n_head_kv*head_dim for K, n_head_q*head_dim for Q).
 */
typedef struct kvm_rows {
    const void *data;
    int32_t type;
    uint32_t n_head;
    uint32_t head_dim;
    uint32_t reserved0;
    uint64_t nb_dim;
    uint64_t nb_head;
    uint64_t nb_tok;
} kvm_rows;

/* Device producers of the statistics the scorer reads.  Every one is an
 * ordered F32 sum that continues the reference's own association, so the
 * summaries and the query stay bit-identical to the reference host store
 * while never leaving HBM. */

/* RawKvStore::write_layer_mean_k (raw_kv_store.cpp:674-694, add_mean_f32
 * :204-223) for tokens [pos0, pos0+n) of one layer, row i of `k` holding
 * position pos0+i: per block, a write starting at offset 0 restarts the sum,
 * rows are added in token order, and the block's mean_tokens becomes `take`
 * (offset 0) or max(mean_tokens, offset+take).  Stream-ordered. */
kvm_status kvm_write_mean_k(kvm_session *s, kvm_stream stream, uint32_t layer, uint32_t pos0,
                            uint32_t n, const kvm_rows *k);
/* Decode accumulator of one layer (kvmem_meank_add, llama-kvmem-stagein.cu:
 * 269-315 and :1039-1063): acc[layer] += rows tok0 .. tok0+n-1 of `k`, in
 * order.  The session holds one F32 [n_head_kv*head_dim] accumulator per
 * layer, zero at creation. */
kvm_status kvm_meank_add(kvm_session *s, kvm_stream stream, uint32_t layer, uint32_t tok0,
                         uint32_t n, const kvm_rows *k);
/* decode_mean_flush (llama-memory-kvmem.cpp:2665-2724) for layers
 * [layer0, layer0+n_layers): RawKvStore::write_layer_mean_sum(pos0, n, il,
 * acc[il]) (raw_kv_store.cpp:696-720) on the device, then acc[il] = 0. */
kvm_status kvm_meank_flush(kvm_session *s, kvm_stream stream, uint32_t layer0,
                           uint32_t n_layers, uint32_t pos0, uint32_t n);
/* kvmem_meank_zero (llama-kvmem-stagein.cu:1031-1037) for layers
 * [layer0, layer0+n_layers) (decode_mean_zero_acc, llama-memory-kvmem.cpp:2470). */
kvm_status kvm_meank_zero(kvm_session *s, kvm_stream stream, uint32_t layer0,
                          uint32_t n_layers);
/* reset_query_acc (llama-memory-kvmem.cpp:2059-2064): q_sum = 0, q_count = 0. */
kvm_status kvm_query_reset(kvm_session *s, kvm_stream stream);
/* harvest 'q' (llama-memory-kvmem.cpp:2157-2173, :2206-2219) for one layer:
 * for each token i < n with keep[i] != 0 (keep = host array of
 * query_contains(pos_i); NULL keeps all), in order, q_sum[layer] += Q[i] and
 * q_count[layer] += 1.  The next score picks the accumulated query up. */
kvm_status kvm_query_add(kvm_session *s, kvm_stream stream, uint32_t layer, uint32_t n,
                         const kvm_rows *q, const uint8_t *keep);

/*
 * Captured query (harvest_from_host 'q', llama-memory-kvmem.cpp:2157-2173):
 * q_sum [n_layer][n_head_q*head_dim] F32 sums of pre-RoPE Q (host or device
 * pointer), q_count [n_layer] host array of tokens summed (0 = layer has no
 * query and does not vote).  Either way q_sum is read in stream order at
 * this call: a host query is copied; a query in this device's memory (and at
 * most 64 layers) is read by the query prep, which this call launches on
 * `stream` (one kernel, no copy), so the following kvm_score starts with the
 * scorer.  The caller may reuse its buffer for work ordered after the call.
 */
kvm_status kvm_set_query(kvm_session *s, kvm_stream stream, const float *q_sum,
                         const uint32_t *q_count);

/* ---------------------------------------------- stage-in transform mode -- */

/*
 * Optional per-head transforms applied to the F16 rows between the gather and
 * the quantizer (the reference's quantizing stage-in, llama-kvmem-stagein.cu:
 * 632-753: RoPE at the original position, then attn_rot, then quantize), so
 * F16 pre-RoPE history can feed a rotated quantized cache:
 *   K: NeoX RoPE of the first rope_n_rot dims of every head at the token's
 *      original position (block_id * block_tokens + row), then the
 *      Walsh-Hadamard transform of every rot_k chunk of every head;
 *   V: the Walsh-Hadamard transform of every rot_v chunk.
 * The RoPE frequencies follow kvmem::rope_neox_apply (kvmem/src/host/
 * rope.cpp:8-45): theta_i = powf(freq_base, -2i/n_rot) * freq_scale; the
 * Hadamard transform follows fwht_kernel (llama-kvmem-stagein.cu:104-130):
 * scale by 1/sqrtf(n) first, then butterflies h = 1, 2, 4, ...  Zero fields
 * switch a transform off.  rot_k / rot_v must be 64, 128, 256 or 512 and
 * divide head_dim; rope_n_rot a multiple of 64 up to head_dim.  The window
 * types must be quantized (Q8_0 / Q4_0 / Q5_0) for a Hadamard transform, as
 * kvmem_attn_rot_on requires; head_dim must be a multiple of 32.
 */
typedef struct kvm_transform {
    uint32_t rot_k;
    uint32_t rot_v;
    uint32_t rope_n_rot;
    uint32_t reserved0;
    float rope_freq_base;
    float rope_freq_scale;
} kvm_transform;

/* Set (or, with NULL, clear) the transforms of later stage-ins. */
kvm_status kvm_set_transform(kvm_session *s, const kvm_transform *t);
/* The reference's attn_rot rule (kvmem_attn_rot_on, kvmem_hadamard_nrot_k /
 * _v, src/adapter/llama-kvmem-quant.h:22-40): the Hadamard size a cache of
 * `type` gets for K (is_k = 1) or V, 0 when attn_rot is off for it.  The
 * LLAMA_ATTN_ROT_DISABLE environment switch is the caller's to read. */
uint32_t kvm_attn_rot_nrot(int32_t type, uint32_t head_dim, int is_k);

/* ----------------------------------------------------- reselection step -- */

/* Scores of every block (f64, score_retrieval); optional copy to d_scores. */
kvm_status kvm_score(kvm_session *s, kvm_stream stream, double *d_scores);
/* Per-layer score terms for layers [layer0, layer0+n_layers) of this session,
 * written to d_terms[(layer0 + i) * ldt + b] = layer_sum / n_head_kv (0 for a
 * layer without query).  Used to split one session's layers across GPUs. */
kvm_status kvm_score_terms(kvm_session *s, kvm_stream stream, uint32_t layer0,
                           uint32_t n_layers, double *d_terms, uint32_t ldt);
/* Ordered sum of per-layer terms: d_acc[b] = ((0 + t[0][b]) + t[1][b]) + ...
 * over the n_layers rows of d_terms (row stride ldt), the reference's
 * layer order (llama-memory-kvmem.cpp:2881-2912).  Rows of layers without a
 * query hold 0.0, which adds exactly.  Used to combine terms gathered from
 * the ranks of a layer-split session, or a rank's partial sum. */
kvm_status kvm_reduce_terms(kvm_session *s, kvm_stream stream, const double *d_terms,
                            uint32_t n_layers, uint32_t ldt, double *d_acc);
/* Install block scores from summed terms: score = acc / n_active (0 for blocks
 * without data).  d_acc [block_count] f64 device; n_active = layers with a
 * query across all partitions.  KvMemStore::set_retrieval_scores. */
kvm_status kvm_set_scores_from_sum(kvm_session *s, kvm_stream stream, const double *d_acc,
                                   uint32_t n_active);
/* Install externally computed scores (host or device pointer, f64 [n]). */
kvm_status kvm_set_scores(kvm_session *s, kvm_stream stream, const double *scores,
                          uint32_t n);
/* pick_topk_blocks(mandatory): mandatory is a host array in reference order
 * (walked from its end, newest first), copied before the call returns.  The
 * selection kernel runs fused with the next kvm_diff (deferred launches,
 * above). */
kvm_status kvm_select(kvm_session *s, kvm_stream stream, const uint32_t *mandatory,
                      uint32_t n_mandatory);
/* KvMemStore::pick_semantic_groups (kvmem/src/host/kvmem_store.cpp:625-756)
 * in place of kvm_select: the same sink / mandatory / recent pins, then whole
 * groups -- spans[2g], spans[2g+1] a half-open token span (host array),
 * scores[g] its f64 score (host or device) -- in score-descending,
 * group-descending order; a group is admitted with every block it overlaps
 * or skipped when they do not fit; the rest of the budget stays unused.
 * At most 8192 groups. */
kvm_status kvm_select_groups(kvm_session *s, kvm_stream stream, const uint32_t *spans,
                             const double *scores, uint32_t n_groups,
                             const uint32_t *mandatory, uint32_t n_mandatory);
/* Use a caller-chosen selection instead of kvm_select (any order, duplicates
 * and out-of-range ids are dropped like set_selection does). */
kvm_status kvm_set_selection_ids(kvm_session *s, kvm_stream stream, const uint32_t *ids,
                                 uint32_t n);
/* set_selection + chronological layout on the device; `force_raw_refresh`
 * as in KvMemStore::set_selection. */
kvm_status kvm_diff(kvm_session *s, kvm_stream stream, int force_raw_refresh);
/* Moves retained blocks to their new slots in place, then gathers and
 * quantizes the cold blocks from `src` into the window.  Window bases must be
 * 2-byte aligned (KVM_EINVAL before any launch otherwise).  A device source
 * is fully stream-ordered.  A host source is the one deliberate exception to
 * "no host wait inside a call": the call reads the plan's cold list back (a
 * bounded host wait for the plan header, then a copy of the list) to size the
 * copies through the HBM staging ring, then overlaps
 * each chunk's H2D with the quantize kernel of the previous one; the copy
 * runs at ~93 % of the measured pinned host-to-device bandwidth, which bounds
 * this path. */
kvm_status kvm_stagein(kvm_session *s, kvm_stream stream, const kvm_source *src,
                       const kvm_window *win);
/*
 * Stage-out (harvest) of resident blocks: the packed window rows of blocks
 * ids[0..n) -- harvest_gpu_v with kvmem_stageout_enqueue / _submit,
 * src/adapter/llama-memory-kvmem.cpp:2318-2410, llama-kvmem-stagein.cu:842-963.
 * Block ids[j] lands at dst + j * kvm_stageout_item_bytes(s): for every layer
 * l, at + l * block_tokens * (row_bytes_k + row_bytes_v), its n_tokens K rows
 * then (at + block_tokens * row_bytes_k) its V rows; bytes past a partial
 * block's rows are unspecified.  Window slots come from the device block
 * table, so the call needs no plan read-back.  dst is device memory (one
 * gather kernel) or host memory (pinned for asynchrony: chunks are packed in
 * the HBM staging ring and copied out on a second stream while the next chunk
 * is packed).  resident (host, optional) receives per block 1 when it had a
 * window slot and was copied, 0 when not (its bytes unspecified).  Everything
 * is stream-ordered on `stream`: dst and resident are complete once it is.
 */
kvm_status kvm_stageout(kvm_session *s, kvm_stream stream, const uint32_t *ids, uint32_t n,
                        const kvm_window *win, void *dst, uint8_t *resident);
/* Bytes one block occupies in a kvm_stageout destination. */
uint64_t kvm_stageout_item_bytes(const kvm_session *s);

/* kvm_stagein from packed rows, the reference's stage-in as it runs today
 * (write_block_to_gpu -> kvmem_stagein_enqueue_v / kvmem_stagein_flush,
 * llama-memory-kvmem.cpp:2726-2791, llama-kvmem-stagein.cu:632-753, 820-840):
 * the retained blocks are moved to their new slots, then the cold blocks' rows
 * are copied into theirs unchanged (no quantization: they are already in the
 * window's types).  A host source goes through the HBM staging ring, each
 * chunk's H2D overlapping the previous chunk's copy. */
kvm_status kvm_stagein_packed(kvm_session *s, kvm_stream stream, const kvm_packed_source *src,
                              const kvm_window *win);

/* score -> select -> diff -> stage-in in one call. */
kvm_status kvm_step(kvm_session *s, kvm_stream stream, const uint32_t *mandatory,
                    uint32_t n_mandatory, const kvm_source *src, const kvm_window *win);

/* Bounded host wait for all work queued on `stream`; checks the device error
 * flags.  KVM_ETIMEOUT if not done within timeout_ms. */
kvm_status kvm_wait(kvm_session *s, kvm_stream stream, uint32_t timeout_ms);

/* Test hook for the failure path (no reference counterpart).  With
 * KVM_TEST_SKIP_TILE_LOAD the next stage-in launch of this session leaves the
 * first tile of its first CTA unloaded: that CTA's bounded waits run out
 * (about 2 s each), it drains its other copies and returns, and the next
 * kvm_wait reports KVM_EDEVICE ("wait-timeout") and clears the flags.  The
 * hook applies to one launch; nothing faults and the session stays usable. */
#define KVM_TEST_SKIP_TILE_LOAD 1u
kvm_status kvm_test_inject(kvm_session *s, uint32_t flags);
/* Copy the last plan to host arrays (waits on `stream`, bounded by
 * timeout_ms) and refresh the host view of window slots. */
kvm_status kvm_get_plan(kvm_session *s, kvm_stream stream, kvm_plan *plan, uint32_t timeout_ms);
/* Copy scores (f64 [n]) to a host array after a wait. */
kvm_status kvm_get_scores(kvm_session *s, kvm_stream stream, double *scores, uint32_t n,
                          uint32_t timeout_ms);
/* Stage timers of the last kvm_step (needs a completed step). */
kvm_status kvm_get_timings(kvm_session *s, kvm_timings *t);
/* Number of kernels libkvm launched on this session since creation. */
uint64_t kvm_kernel_launches(const kvm_session *s);

/* -------------------------------------------------- standalone kernels -- */

/* Quantize n_rows F16 rows of n_embd values (device pointers, rows
 * contiguous) to `type` rows at d_dst -- the stage-in kernel on a plain
 * row range.  d_src must be 16-byte and d_dst 2-byte aligned.  Returns
 * KVM_EINVAL for unsupported widths or alignments, KVM_EDEVICE when a
 * bounded device wait ran out (message in kvm_last_error(NULL)).  Allocates
 * a small work list and waits on the host for the stream before it returns. */
kvm_status kvm_quantize_rows(kvm_stream stream, int32_t type, const void *d_src,
                             uint64_t n_rows, uint32_t n_embd, void *d_dst);

/*
 * kvm_quantize_rows without any device allocation.  No counterpart in the
 * reference: it exists for callers that cannot call cudaMalloc while they
 * run -- runtimes whose caching allocator owns all free HBM, latency-critical
 * loops that cannot take the device-wide synchronisation of
 * cudaMalloc/cudaFree.  Same arguments, alignment rules and bytes as
 * kvm_quantize_rows; stream-ordered, no host wait, so a bounded device wait
 * that runs out inside the kernel is not reported.
 * The work list lives in a fixed device array of 16384 row tiles (a tile is
 * 8192 / n_embd rows, at most 128: 131072 rows at n_embd 1024); larger calls
 * return KVM_EINVAL (message in kvm_last_error(NULL)).  The array is shared
 * by every call in the process, so calls that overlap on the GPU (for
 * example on two streams) race: serialise them.  The first call on each
 * device looks the array's device address up (cudaGetSymbolAddress) and
 * should come before any stream capture.
 */
kvm_status kvm_quantize_rows_noalloc(kvm_stream stream, int32_t type, const void *d_src,
                                     uint64_t n_rows, uint32_t n_embd, void *d_dst);

#ifdef __cplusplus
}
#endif

#endif /* KVM_H */
