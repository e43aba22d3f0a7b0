/*
 * kvm_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of CrKcel/kvmem-llama.cpp's per-step KV reselection path
 * (score -> select -> diff -> quantized stage-in).  It is the checker that the
 * sm_100a kernels are compared against.  Only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / `--impl reference` leg may load it; the
 * product library (libkvm) never links or calls it.
 *
 * Parity status of each piece:
 *   - selection (pick_topk) and diff (set_selection): pinned against the
 *     reference's own libkvmem compiled from its sources (oracle/_ref) and the
 *     inline expectations of kvmem/tests/kvmem_store_test.cpp.
 *   - mean-K (sum * 1/n): pinned against the compiled RawKvStore.
 *   - quantizers q8_0/q4_0/q5_0: pinned against gguf-py 0.19.0 (which states
 *     bit-exactness with ggml-quants.c) through tests/golden fixtures; q8_0
 *     also against the reference's own CUDA quant_q8_0 (bit-exact), q4_0
 *     against its quant_q4_0, which differs only where nvcc fuses x*id + 8.5f
 *     (oracle/ref_stagein.cu, tests/test_gpu_ref_kernels.py).
 *   - Walsh-Hadamard: bit-exact with the reference's own CUDA fwht_kernel<N>
 *     for N = 64, 128, 256, 512 (same files).
 *   - scorer: pinned against the reference's own score_retrieval
 *     (src/adapter/llama-memory-kvmem.cpp:2869-2916).  The adapter as a whole
 *     needs the absent llama.cpp submodule, so oracle/Makefile compiles that
 *     one function, cut from the reference file at build time, inside
 *     ref_score.cpp against the compiled libkvmem; tests compare live and
 *     through tests/golden/score_golden.npz.  The restatement follows it line
 *     by line, compiled with -ffp-contract=off like the reference's x86-64
 *     baseline build (no FMA contraction).
 */
#ifndef KVM_ORACLE_H
#define KVM_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids (ggml.h enum ggml_type values). */
#define ORA_TYPE_F16  1
#define ORA_TYPE_Q4_0 2
#define ORA_TYPE_Q5_0 6
#define ORA_TYPE_Q8_0 8

/* Store tier values, kvmem/include/kvmem/kvmem_store.hpp:31. */
#define ORA_TIER_GPU 0
#define ORA_TIER_CPU 1
#define ORA_TIER_SSD 2

float    ora_f16_to_f32(uint16_t h);
uint16_t ora_f32_to_f16(float f);

/* Bytes of one quantized row of n_embd values (ggml_row_size). */
uint64_t ora_row_bytes(int type, uint32_t n_embd);

/* ggml q8_0 / q4_0 / q5_0 reference quantizers over n floats (n % 32 == 0). */
void ora_quantize_q8_0(const float *x, int64_t n, uint8_t *y);
void ora_quantize_q4_0(const float *x, int64_t n, uint8_t *y);
void ora_quantize_q5_0(const float *x, int64_t n, uint8_t *y);

/* F16 rows [n_rows][n_embd] -> quantized rows of `type`; returns 0 or -1. */
int ora_quantize_rows_f16(int type, const uint16_t *src, int64_t n_rows,
                          uint32_t n_embd, uint8_t *dst, int n_threads);

/*
 * Stage-in transforms (the reference's quantizing stage-in,
 * src/adapter/llama-kvmem-stagein.cu:632-753).
 *   ora_rope_theta: theta_i = powf(base, -2i/n_rot) * scale, i < n_rot/2
 *                   (kvmem/src/host/rope.cpp:18-22).
 *   ora_rope_neox_rows: NeoX RoPE of rows [n_tokens][n_head][head_dim] at
 *                   positions pos0 + t (rope.cpp:26-43, rope_neox_kernel
 *                   stagein.cu:160-178); cosf / sinf, no FMA contraction.
 *   ora_fwht_rows:  Walsh-Hadamard of every nrot chunk of n_rows rows of
 *                   n_embd floats, fwht_kernel order (stagein.cu:104-130):
 *                   scale by 1.0f/sqrtf(nrot) first, butterflies h = 1, 2, ...
 *   ora_attn_rot_nrot: kvmem_attn_rot_on + kvmem_hadamard_nrot_k/_v
 *                   (src/adapter/llama-kvmem-quant.h:22-40).
 */
void ora_rope_theta(uint32_t n_rot, float freq_base, float freq_scale, float *theta);
void ora_rope_neox_rows(float *x, int64_t n_tokens, uint32_t n_head, uint32_t head_dim,
                        uint32_t n_rot, int32_t pos0, const float *theta);
void ora_fwht_rows(float *x, int64_t n_rows, uint32_t n_embd, uint32_t nrot);
uint32_t ora_attn_rot_nrot(int type, uint32_t head_dim, int is_k);

/* Ordered F32 sum over tokens of F16 K rows (RawKvStore::add_mean_f32). */
void ora_block_sum_f16(const uint16_t *k, uint32_t n_tokens, uint32_t n_embd,
                       uint64_t row_stride, float *sum);
/* RawKvStore::mean_k: sum * (1.0f / n), zeros when n == 0. */
void ora_mean_k(const float *sum, uint32_t mean_tokens, uint32_t n_embd,
                float *out);

/*
 * llama_memory_kvmem::score_retrieval.
 *   sums      [n_layer][n_blocks][n_head_kv*head_dim] F32 K sums
 *   mean_tok  [n_layer][n_blocks] token count behind each sum (0 = none)
 *   has_block [n_blocks] RawKvStore::has_block
 *   q_sum     [n_layer][n_head_q*head_dim], q_count [n_layer]
 *   scores    [n_blocks] out;  terms [n_layer][n_blocks] out (optional):
 *             layer/H_kv for layers with q_count > 0, else 0.
 */
void ora_score(const float *sums, const uint32_t *mean_tok,
               const uint8_t *has_block, uint32_t n_blocks, uint32_t n_layer,
               const float *q_sum, const uint32_t *q_count, uint32_t n_head_kv,
               uint32_t n_head_q, uint32_t head_dim, double *scores,
               double *terms, int n_threads);

typedef struct ora_cfg {
    uint32_t block_tokens;
    uint32_t budget_blocks;          /* KvMemStore::budget_blocks() */
    uint32_t sink_blocks;
    uint32_t recent_blocks;
    uint32_t optimize_stage_in;      /* 0 => force_full_reload */
    uint32_t immutable_source_k;
    uint32_t immutable_refresh_remaps;
    uint32_t pad0;
    uint64_t immutable_refresh_abs_delta_tokens;
    uint64_t immutable_max_baked_position;
} ora_cfg;

/* Block table, structure of arrays (KvMemBlock fields used by the path). */
typedef struct ora_blocks {
    uint32_t *n_tokens;
    uint8_t  *tier;
    int32_t  *gpu_slot;
    int64_t  *baked_pos;
    uint32_t *remap_count;
    uint64_t *remap_abs_delta;
    uint8_t  *in_working_set;
} ora_blocks;

/* KvMemPlan, caller-owned arrays of capacity n_blocks. */
typedef struct ora_plan {
    uint32_t *stage_in;
    uint32_t *stage_out;
    uint32_t *rm_block_id;
    uint32_t *rm_n_tokens;
    int32_t  *rm_from_base;
    int32_t  *rm_to_base;
    uint8_t  *rm_working_k_resident;
    uint8_t  *rm_skip;
    uint8_t  *rm_raw_refresh;
    uint32_t n_stage_in;
    uint32_t n_stage_out;
    uint32_t n_remaps;
    uint32_t total_window_tokens;
    uint32_t selection_overlap_blocks;
    uint32_t gpu_reused_blocks;
    uint32_t retained_position_stable;
    uint32_t retained_position_moved;
} ora_plan;

/* KvMemStore::pick_topk_blocks(mandatory), TopK policy. Returns count. */
uint32_t ora_pick_topk(const ora_cfg *cfg, const double *scores, uint32_t n,
                       const uint32_t *mandatory, uint32_t n_mandatory,
                       uint32_t *out);

/* KvMemStore::set_selection. Returns 0, or -1 where the reference throws. */
/*
 * KvMemStore::pick_semantic_groups (kvmem/src/host/kvmem_store.cpp:625-756).
 * spans: [n_groups][2] half-open token spans; covered_tokens: tokens of the
 * store (last block's start + its n_tokens).  Selected ids ascending in out.
 */
uint32_t ora_pick_semantic_groups(const ora_cfg *cfg, uint32_t n, uint64_t covered_tokens,
                                  const uint32_t *spans, const double *scores,
                                  uint32_t n_groups, const uint32_t *mandatory,
                                  uint32_t n_mandatory, uint32_t *out);

int ora_set_selection(const ora_cfg *cfg, ora_blocks *b, uint32_t n,
                      const uint32_t *ids, uint32_t n_ids,
                      int force_raw_refresh, ora_plan *plan);

/*
 * Chronological slot layout after a selection (layout_gpu_slots_by_orig_pos):
 * the i-th selected block (ascending id) ends in window slot i.  Inputs are
 * the ascending selection and each block's slot before the step (-1 = not
 * resident).  Outputs: moves (block, from, to) for resident blocks whose slot
 * changes, cold (block, to) for blocks that must be staged in, and the new
 * slot of every block.  Returns 0.
 */
int ora_layout(const uint32_t *sel, uint32_t n_sel, const int32_t *slot_before,
               uint32_t n_blocks, int32_t *slot_after, uint32_t *mv_block,
               int32_t *mv_from, int32_t *mv_to, uint32_t *n_moves,
               uint32_t *cold_block, int32_t *cold_to, uint32_t *n_cold);

#ifdef __cplusplus
}
#endif

#endif
