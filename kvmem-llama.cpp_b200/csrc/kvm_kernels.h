// kvm_kernels.h -- launch arguments and launchers of libkvm's kernels.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "kvm_internal.cuh"

namespace kvm {

constexpr int kStageinConsumerWarps = 8;
constexpr int kStageinStages = 3;
// Transform mode.  attn_rot alone: 7 consumer warps + the producer, four
// CTAs an SM (64 registers a thread, 32 warps an SM), two stages and two
// output tiles -- measured faster than three CTAs with three and three (80
// registers) once output tiles are released as soon as their store has read
// them; with RoPE: 8 + 1 warps, two CTAs an SM (its sin/cos want the
// registers), four stages of input only.
constexpr int kXfConsumerWarps = 7;
constexpr int kXfMinBlocks = 4;
constexpr int kXfStages = 2;
constexpr int kXfOutStages = 2;
constexpr int kXfRopeWarps = 8;
constexpr int kXfRopeMinBlocks = 2;
constexpr int kXfRopeStages = 4;
constexpr int kPermuteThreads = 512;
constexpr uint32_t kSumGroup = 32;                 // blocks per summary tile
constexpr uint32_t kScoreRange = 32;               // blocks per scorer CTA (a warp's lanes)
static_assert(kScoreRange == kSumGroup, "a scorer CTA reads one summary tile per layer");
constexpr int kScoreStages = 12;                   // scorer: 16-byte vectors in flight per lane
constexpr int kSelectThreads = 1024;
constexpr int kDiffThreads = 1024;

// ------------------------------------------------------------- stage-in --
struct StageinArgs {
    // work list: items [item0, item0 + n) of cold_block / cold_to
    const uint32_t *cold_block;
    const int32_t *cold_to;
    const uint32_t *n_items_dev;   // device count (NULL: use n_items_host)
    uint32_t n_items_host;
    uint32_t item0;
    uint32_t max_items;
    uint32_t src_by_item;          // 1: source index = item - item0 (staging ring)
    uint32_t n_kv;                 // 2: K and V tasks; 1: K only
    // F16 source
    const uint8_t *src_k;
    const uint8_t *src_v;
    uint64_t layer_stride;
    uint64_t item_stride;
    uint64_t row_stride;
    // block table and window
    const uint32_t *n_tokens;
    uint32_t max_blocks;
    uint8_t *const *dst_k;         // device array [n_layer]
    uint8_t *const *dst_v;
    uint32_t n_layer;
    uint32_t block_tokens;
    uint32_t n_embd;
    uint32_t n_slots;
    int32_t type_k;
    int32_t type_v;
    uint32_t row_bytes_k;
    uint32_t row_bytes_v;
    uint32_t rows_per_tile;
    uint32_t tile_in_bytes;
    uint32_t tile_out_bytes;
    uint32_t bulk_store;
    uint32_t *status;
    // transform mode (kvm_set_transform): xform = head_dim / 32 when a
    // transform is on, 0 for the plain gather + quantize
    uint32_t xform;
    uint32_t rot_k;
    uint32_t rot_v;
    uint32_t rope_n_rot;
    const float *theta;            // device [rope_n_rot / 2]
    float xf_pre_k, xf_pre_v;      // Hadamard scale applied before the butterflies (1: none)
    float xf_post_k, xf_post_v;    // power-of-two Hadamard scale folded into the quantizer (1: none)
    uint32_t xf_heads;             // KV heads per row, n_embd / head_dim
    uint32_t xf_heads_magic;       // ceil(2^32 / xf_heads); 0 when xf_heads == 1
    uint32_t test_skip;            // kvm_test_inject: CTA 0 leaves its first tile unloaded
};

uint32_t stagein_rows_per_tile(uint32_t n_embd, uint32_t block_tokens);
// Fills the transform-mode fields of `a` (xform, rot_k/v, rope_n_rot, theta
// and the derived scales and head count); all zero / 1 when nothing is set.
void stagein_set_transform(StageinArgs &a, uint32_t head_dim, uint32_t n_embd, uint32_t rot_k,
                           uint32_t rot_v, uint32_t rope_n_rot, const float *theta);
size_t stagein_smem_bytes(const StageinArgs &a);
cudaError_t launch_stagein(const StageinArgs &a, cudaStream_t stream, uint32_t grid_cap);

// ------------------------------------------------------------ stage-out --
struct StageoutArgs {
    const uint32_t *ids;           // device block ids of this launch's items
    uint32_t n;                    // items in this launch
    uint32_t item0;                // index of ids[0] in the caller's list (resident flags)
    const int32_t *gpu_slot;       // block table
    const uint32_t *n_tokens;
    uint32_t n_blocks;
    uint32_t n_slots;
    uint32_t n_layer;
    uint32_t block_tokens;
    uint8_t *const *win_k;         // device arrays [n_layer]
    uint8_t *const *win_v;
    uint32_t row_bytes_k;
    uint32_t row_bytes_v;
    uint8_t *dst;                  // item j at dst + j * item_bytes
    uint64_t item_bytes;
    uint8_t *resident;             // optional device flags, [item0 + j]
    uint32_t bulk;                 // 1: every address and size 16-byte aligned
    uint32_t *status;
};

cudaError_t launch_stageout(const StageoutArgs &a, cudaStream_t stream);

// stage-in of packed rows: cold items [item0, item0 + n) of cold_block / cold_to
struct PackedInArgs {
    const uint32_t *cold_block;
    const int32_t *cold_to;
    const uint32_t *n_items_dev;   // device count (NULL: use n_items_host)
    uint32_t n_items_host;
    uint32_t item0;
    uint32_t max_items;
    uint32_t src_by_item;          // 1: source index = item - item0 (staging ring)
    const uint8_t *src_k;
    const uint8_t *src_v;
    uint64_t k_layer_stride;
    uint64_t k_block_stride;
    uint64_t v_layer_stride;
    uint64_t v_block_stride;
    const uint32_t *n_tokens;
    uint32_t max_blocks;
    uint32_t n_slots;
    uint32_t n_layer;
    uint32_t block_tokens;
    uint8_t *const *win_k;
    uint8_t *const *win_v;
    uint32_t row_bytes_k;
    uint32_t row_bytes_v;
    uint32_t bulk;                 // 1: every address and size 16-byte aligned
    uint32_t *status;
};

cudaError_t launch_packed_stagein(const PackedInArgs &a, cudaStream_t stream);

// -------------------------------------------------------------- permute --
struct PermuteArgs {
    const uint32_t *n_moves_dev;
    const uint32_t *mv_block;
    const int32_t *mv_from;
    const int32_t *mv_to;
    uint32_t max_moves;
    const uint32_t *n_tokens;
    uint32_t max_blocks;
    uint8_t *const *dst_k;
    uint8_t *const *dst_v;
    uint32_t n_layer;
    uint32_t block_tokens;
    uint32_t n_slots;
    uint32_t row_bytes_k;
    uint32_t row_bytes_v;
    uint32_t span_k;
    uint32_t span_v;
    uint32_t col_bytes;            // widest column a CTA stages (bytes, multiple of 16)
    uint32_t col_region;           // shared-memory bytes for the staged columns
    uint32_t vec16;
    uint32_t piece;                // streaming permute: bytes of a block span a stream moves
    uint32_t *status;
};

// shared-memory bytes of the per-move metadata table (12 bytes a move, 16-aligned)
__host__ __device__ inline size_t permute_meta_bytes(uint32_t max_moves) {
    return (static_cast<size_t>(max_moves) * 12u + 15u) & ~static_cast<size_t>(15u);
}

// Streaming permute: ring depth and the offset of its buffers in shared
// memory (a 256-byte header, the move table, the processing order).
constexpr int kChainStages = 4;
__host__ __device__ inline size_t permute_chain_buf_offset(uint32_t max_moves) {
    return (256u + permute_meta_bytes(max_moves) + 2u * static_cast<size_t>(max_moves) + 127u) &
           ~static_cast<size_t>(127u);
}
cudaError_t launch_permute(const PermuteArgs &a, cudaStream_t stream);

// ---------------------------------------------------------- summaries --
// Summary tensor, tiled: [layer][block group of 32][n_embd/4][32 blocks][4
// channels].  Four consecutive channels of one block are one 16-byte vector,
// and the vectors of the 32 blocks of a group sit side by side: a warp of
// threads, one per block, reads its blocks' next four channels as 512
// contiguous bytes, and one KV head of a group is head_dim * 128 contiguous
// bytes.  n_embd is a multiple of 32 (ggml blocks).
struct SummaryLayout {
    float *sum_t;          // [n_layer][ldb/32][n_embd/4][32][4]
    uint32_t *mean_tok;    // [n_layer][ldb]
    float *inv_tok;        // [n_layer][ldb]  1.0f / mean_tok (0 when none)
    uint32_t ldb;          // block capacity, a multiple of 32
    uint32_t n_layer;
    uint32_t n_embd;
};

__host__ __device__ inline size_t sum_index(const SummaryLayout &s, uint32_t l, uint32_t e,
                                            uint32_t b) {
    return (((static_cast<size_t>(l) * (s.ldb / kSumGroup) + b / kSumGroup) * (s.n_embd / 4u) + e / 4u) *
                kSumGroup + (b % kSumGroup)) * 4u + (e % 4u);
}

cudaError_t launch_upload_summaries(const SummaryLayout &s, uint32_t layer, uint32_t block0,
                                    uint32_t n, const float *d_sums, const uint32_t *d_counts,
                                    cudaStream_t stream);
cudaError_t launch_download_summaries(const SummaryLayout &s, uint32_t layer, uint32_t block0,
                                      uint32_t n, float *d_sums, cudaStream_t stream);

// ----------------------------------------------------------- producers --
// ggml type ids of captured activations
constexpr int32_t kActF32 = 0;
constexpr int32_t kActF16 = 1;
constexpr int32_t kActBF16 = 30;

struct MeanKArgs {
    SummaryLayout sum;
    const uint8_t *src;    // row addressing: see kvm_produce.cu
    int32_t type;          // kActF32 / kActF16 / kActBF16
    uint32_t vec;          // channels per lane: 8, 4 or 1 (mean_k_vec)
    uint32_t head_dim;
    uint64_t nb_dim;
    uint64_t nb_head;
    uint64_t nb_row;       // between consecutive tokens
    uint64_t nb_block;     // table mode: between blocks
    uint64_t nb_layer;     // table mode: between layers (0 in token mode)
    uint32_t layer0;
    uint32_t block0;
    uint32_t n_blk;
    uint32_t block_tokens;
    uint32_t pos0;         // token mode
    uint32_t n;            // token mode
    const uint32_t *n_tokens;  // table mode when non-null
};

struct AddRowsArgs {
    float *acc;
    uint32_t n_elem;
    const uint8_t *src;
    int32_t type;
    uint32_t head_dim;
    uint64_t nb_dim;
    uint64_t nb_head;
    uint64_t nb_tok;
    const uint32_t *tok_list;  // optional: token indices to add, in order
    uint32_t tok0;             // without a list: tokens tok0 .. tok0+n-1
    uint32_t n;
};

// channels per lane the mean-K kernel may use for this source; align_mask is
// the OR of the base pointer and every stride the rows are addressed with
uint32_t mean_k_vec(int32_t type, uint32_t head_dim, uint64_t nb_dim, uint64_t align_mask);
cudaError_t launch_mean_k(const MeanKArgs &a, uint32_t n_layers, cudaStream_t stream);
cudaError_t launch_add_rows(const AddRowsArgs &a, cudaStream_t stream);
cudaError_t launch_meank_flush(const SummaryLayout &s, float *meank, uint32_t layer0, uint32_t n_layers,
                               uint32_t pos0, uint32_t n, uint32_t block_tokens, cudaStream_t stream);

// --------------------------------------------------------------- query --
struct QueryState {
    float *q_sum;          // [n_layer][n_head_q*head_dim]  (device copy)
    uint32_t *q_count;     // [n_layer]
    float *qv;             // [n_layer][n_head_kv][head_dim] prepared query
    float *nq;             // [n_layer][n_head_kv] its squared norm
};

// kvm_set_query with a device-resident q_sum: the prep reads it in stream
// order at that call, keeps a copy in QueryState::q_sum (for later
// kvm_query_add) and takes q_count from the launch parameters.
constexpr uint32_t kQueryInlineLayers = 64;
struct QueryLoad {
    const float *src;                       // [n_layer][n_head_q*head_dim]
    uint32_t count[kQueryInlineLayers];     // q_count of each layer
};

// The query prep alone, as the programmatic dependent launch of whatever
// precedes it on the stream: it waits (griddepcontrol) before it reads
// `ld.src`, then lets a following scorer start.
cudaError_t launch_query_load(const QueryState &q, const QueryLoad &ld, uint32_t n_layer, uint32_t n_head_kv,
                              uint32_t n_head_q, uint32_t head_dim, cudaStream_t stream);

// -------------------------------------------------------------- scorer --
struct ScoreArgs {
    SummaryLayout sum;
    const float *qv;       // QueryState::qv / nq, made by the query prep
    const float *nq;
    const uint32_t *q_count;
    uint32_t n_head_kv;
    uint32_t n_head_q;
    uint32_t head_dim;
    uint32_t n_blocks;
    uint32_t layer0;       // first layer scored by this launch
    uint32_t n_layers;     // layers scored by this launch
    double *terms;         // [layer][ldt], indexed by the session's layer
    uint32_t ldt;
    uint32_t *status;
    // combine: the last CTA of each block range also forms the final scores
    // (only when n_layers == all layers of the session)
    int combine;
    uint32_t *range_done;  // [ldb / kScoreRange] arrival counters, zero between launches
    double *scores;        // [ldb]
};

// The query prep (when `prep`, qv / nq from q_sum for every layer), then the
// scorer.  After a prep -- this one, or launch_query_load as the stream's
// previous kernel (`after_prep_load`) -- the scorer is a programmatic
// dependent launch: its CTAs start their summary loads while the prep runs
// and wait for it (griddepcontrol) before they read the query and q_count.
cudaError_t launch_score(const ScoreArgs &a, const QueryState *prep, uint32_t n_layer_all, cudaStream_t stream,
                         bool after_prep_load = false);
cudaError_t launch_reduce_terms(const double *terms, uint32_t n_layers, uint32_t ldt,
                                uint32_t n_blocks, double *acc, cudaStream_t stream);
cudaError_t launch_scores_from_sum(const SummaryLayout &s, uint32_t n_blocks, const double *acc,
                                   uint32_t n_active, double *scores, cudaStream_t stream);

// -------------------------------------------------------------- select --
struct SelectArgs {
    const double *scores;
    uint32_t n_blocks;
    uint32_t budget;
    uint32_t sink;
    uint32_t recent;
    const uint32_t *mandatory;
    uint32_t n_mandatory;
    uint32_t *selected;
    PlanHeader *hdr;
};

cudaError_t launch_select(const SelectArgs &a, cudaStream_t stream);

// pick_semantic_groups
constexpr uint32_t kMaxGroups = 8192;
struct GroupSelectArgs {
    const uint32_t *spans;         // [n_groups][2] half-open token spans
    const double *scores;          // [n_groups]
    uint32_t n_groups;
    uint32_t n_blocks;
    uint32_t budget;
    uint32_t sink;
    uint32_t recent;
    uint32_t block_tokens;
    uint32_t covered_tokens;       // tokens registered (last block's start + its tokens)
    const uint32_t *mandatory;
    uint32_t n_mandatory;
    uint32_t *selected;
    PlanHeader *hdr;
};

size_t group_select_smem(uint32_t n_groups, uint32_t n_blocks);
cudaError_t launch_group_select(const GroupSelectArgs &a, cudaStream_t stream);

// Sort ascending + dedupe + drop >= n of a caller selection (device, n <= cap).
cudaError_t launch_canon_ids(const uint32_t *ids, uint32_t n_ids, uint32_t n_blocks,
                             uint32_t *selected, PlanHeader *hdr, cudaStream_t stream);

// ---------------------------------------------------------------- diff --
struct DiffArgs {
    BlockTable bt;
    uint32_t n_blocks;
    uint32_t n_slots;
    uint32_t optimize_stage_in;
    uint32_t immutable_source_k;
    uint32_t immutable_refresh_remaps;
    uint64_t immutable_refresh_abs_delta_tokens;
    uint64_t immutable_max_baked_position;
    int force_raw_refresh;
    uint32_t reset_window;         // apply a pending kvm_reset_window first
    PlanArrays plan;
    uint32_t *status;
};

cudaError_t launch_diff(const DiffArgs &a, cudaStream_t stream);
// kvm_select + kvm_diff as one launch
cudaError_t launch_select_diff(const SelectArgs &sa, const DiffArgs &da, cudaStream_t stream);
cudaError_t launch_reset_window(const BlockTable &bt, uint32_t n, cudaStream_t stream);

}  // namespace kvm
