// kvm_session.cu -- the extern "C" ABI of libkvm (include/kvm.h).
//
// A session owns, on one device: the channel-major mean-K summary tensor,
// the captured query, the block table (KvMemBlock fields of the path), the
// plan buffers and the HBM staging ring for host-resident sources.  Host
// state is only what the host must know without a device round trip: the
// block count and token counts (KvMemStore::register_append is host logic)
// and, after kvm_get_plan, the window slot of every block.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>
#include <thread>
#include <vector>

#include "kvm_internal.cuh"
#include "kvm_kernels.h"

using namespace kvm;

namespace {

constexpr int kPinSlots = 8;

uint32_t align_tokens(uint32_t tokens, uint32_t bt) {
    // kvmem_align_tokens, llama-memory-kvmem.cpp:254-262
    if (bt == 0) return 0;
    if (tokens < bt) return bt;
    return (tokens / bt) * bt;
}

bool type_ok(int32_t t) {
    return t == KVM_TYPE_F16 || t == KVM_TYPE_Q8_0 || t == KVM_TYPE_Q4_0 || t == KVM_TYPE_Q5_0;
}

}  // namespace

struct kvm_session {
    kvm_config cfg{};
    int device = 0;
    uint32_t n_embd = 0;
    uint32_t budget_blocks = 0;
    uint32_t n_slots = 0;
    uint32_t max_blocks = 0;
    uint32_t row_bytes_k = 0;
    uint32_t row_bytes_v = 0;

    // host view
    uint32_t n_blocks = 0;
    uint32_t total_tokens = 0;
    std::vector<uint32_t> h_n_tokens;
    std::vector<int32_t> h_slot;       // valid when slots_known
    bool slots_known = true;           // a fresh session has no resident block
    // No block holds a window slot (fresh session, kvm_reset_window, no slot
    // set since): the next diff can produce no moves.
    bool window_empty = true;
    bool plan_moveless = false;        // the current plan came from an empty window
    uint32_t test_inject = 0;          // kvm_test_inject flags for the next stage-in launch
    bool have_selection = false;
    bool have_plan = false;
    // Deferred launches.  kvm_select records its selection here and the next
    // kvm_diff runs select + diff as one kernel; kvm_reset_window records the
    // reset and the next diff applies it while it reads the block table.
    // Every other entry point first launches what is pending (flush_pending),
    // so the order of the calls keeps its meaning.
    bool select_pending = false;
    uint32_t select_n_mandatory = 0;
    bool reset_pending = false;

    // device state
    SummaryLayout sum{};
    QueryState q{};
    double *d_terms = nullptr;
    uint32_t *d_range_done = nullptr;  // scorer arrival counters [ldb / kScoreRange]
    double *d_scores = nullptr;
    double *d_acc = nullptr;
    BlockTable bt{};
    PlanArrays plan{};
    uint32_t *d_mandatory = nullptr;
    uint32_t *d_ids = nullptr;
    uint32_t *d_status = nullptr;
    uint8_t **d_win = nullptr;         // [2][n_layer] window bases
    std::vector<void *> h_win;         // last uploaded window bases
    float *d_stage_sums = nullptr;     // upload staging
    uint32_t *d_stage_counts = nullptr;
    size_t stage_sums_cap = 0;
    uint8_t *d_ring = nullptr;
    size_t ring_bytes = 0;
    float *d_meank = nullptr;          // decode mean-K accumulators [L][E]
    uint32_t *d_keep = nullptr;        // kept query token indices
    uint32_t keep_cap = 0;
    std::vector<uint32_t> h_q_count;   // host copy of q_count
    kvm_transform xf{};                // stage-in transforms (all zero = off)
    float *d_theta = nullptr;          // RoPE frequencies [head_dim / 2]
    bool q_dirty = false;              // q_sum / q_count changed since the last query prep
    // kvm_set_query's own prep launch: `launches` right after it and its
    // stream, so that a scorer launched next on that stream can follow it
    // as a programmatic dependent launch
    uint64_t prep_load_mark = ~0ull;
    cudaStream_t prep_load_stream = nullptr;
    void *d_base = nullptr;            // one allocation for the small arrays

    // pinned ring for small host uploads / plan reads
    uint8_t *h_pin = nullptr;
    size_t pin_slot_bytes = 0;
    cudaEvent_t pin_ev[kPinSlots] = {};
    bool pin_used[kPinSlots] = {};
    int pin_next = 0;
    uint8_t *h_plan = nullptr;         // pinned plan read-back buffer
    size_t h_plan_bytes = 0;

    cudaStream_t copy_stream = nullptr;
    static constexpr int kRingSlots = 4;
    cudaEvent_t ring_copied[kRingSlots] = {};
    cudaEvent_t ring_free[kRingSlots] = {};
    cudaEvent_t out_gathered[kRingSlots] = {};   // stage-out: slot packed (on the caller's stream)
    cudaEvent_t out_done[kRingSlots] = {};       // stage-out: slot copied out (on copy_stream)
    uint32_t *d_out_ids = nullptr;               // stage-out block list
    uint8_t *d_out_flags = nullptr;              // stage-out resident flags
    uint32_t *d_group_spans = nullptr;           // semantic-group spans [kMaxGroups][2]
    double *d_group_scores = nullptr;            // semantic-group scores [kMaxGroups]
    cudaEvent_t ev[7] = {};   // 0-4 step stages, 5 plan read-back, 6 ring start
    bool timed = false;

    uint64_t launches = 0;
    std::string err;
};

namespace {

kvm_status fail(kvm_session *s, kvm_status st, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (s) s->err = buf;
    return st;
}

kvm_status cuda_fail(kvm_session *s, cudaError_t e, const char *what) {
    return fail(s, e == cudaErrorMemoryAllocation ? KVM_ENOMEM : KVM_ECUDA, "%s: %s", what,
                cudaGetErrorString(e));
}

#define KVM_CUDA(s, call, what)                                   \
    do {                                                          \
        cudaError_t e__ = (call);                                 \
        if (e__ != cudaSuccess) return cuda_fail((s), e__, what); \
    } while (0)

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

cudaStream_t as_stream(kvm_stream st) { return reinterpret_cast<cudaStream_t>(st); }

// Bounded host wait on an event.
kvm_status wait_event(kvm_session *s, cudaEvent_t ev, uint32_t timeout_ms) {
    const auto t0 = std::chrono::steady_clock::now();
    for (uint32_t spin = 0;; ++spin) {
        const cudaError_t e = cudaEventQuery(ev);
        if (e == cudaSuccess) return KVM_OK;
        if (e != cudaErrorNotReady) return cuda_fail(s, e, "event wait");
        const auto el = std::chrono::duration_cast<std::chrono::milliseconds>(
                            std::chrono::steady_clock::now() - t0)
                            .count();
        if (static_cast<uint64_t>(el) > timeout_ms)
            return fail(s, KVM_ETIMEOUT, "device work not done after %u ms", timeout_ms);
        if (spin > 64) std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

// Stream-ordered copy of a small host array to the device through the
// session's pinned ring (the host array may be reused on return).
kvm_status upload_small(kvm_session *s, cudaStream_t st, void *dst, const void *src, size_t bytes) {
    if (bytes == 0) return KVM_OK;
    if (bytes > s->pin_slot_bytes) {
        KVM_CUDA(s, cudaStreamSynchronize(st), "upload sync");
        KVM_CUDA(s, cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice), "upload");
        return KVM_OK;
    }
    const int i = s->pin_next;
    s->pin_next = (s->pin_next + 1) % kPinSlots;
    if (s->pin_used[i]) {
        const kvm_status r = wait_event(s, s->pin_ev[i], 10000);
        if (r != KVM_OK) return r;
    }
    uint8_t *slot = s->h_pin + static_cast<size_t>(i) * s->pin_slot_bytes;
    std::memcpy(slot, src, bytes);
    KVM_CUDA(s, cudaMemcpyAsync(dst, slot, bytes, cudaMemcpyHostToDevice, st), "upload");
    KVM_CUDA(s, cudaEventRecord(s->pin_ev[i], st), "upload event");
    s->pin_used[i] = true;
    return KVM_OK;
}

kvm_status check_status(kvm_session *s) {
    uint32_t st = 0;
    KVM_CUDA(s, cudaMemcpy(&st, s->d_status, sizeof st, cudaMemcpyDeviceToHost), "status read");
    if (st) {
        cudaMemset(s->d_status, 0, sizeof(uint32_t));
        return fail(s, KVM_EDEVICE, "device error flags 0x%x (%s%s%s%s)", st,
                    (st & kErrTimeout) ? "wait-timeout " : "", (st & kErrIndex) ? "bad-index " : "",
                    (st & kErrSlot) ? "bad-slot " : "", (st & kErrConfig) ? "bad-config" : "");
    }
    return KVM_OK;
}

SelectArgs select_args(kvm_session *s, uint32_t n_mandatory) {
    SelectArgs a{};
    a.scores = s->d_scores;
    a.n_blocks = s->n_blocks;
    a.budget = s->budget_blocks;
    a.sink = s->cfg.sink_blocks;
    a.recent = s->cfg.recent_blocks;
    a.mandatory = s->d_mandatory;
    a.n_mandatory = n_mandatory;
    a.selected = s->plan.selected;
    a.hdr = s->plan.hdr;
    return a;
}

// Launch the deferred select / window reset on the stream of the call that
// needs it.  A call that depends on the selection or the reset is ordered
// after kvm_select / kvm_reset_window by the caller (same stream, or a wait
// between streams), so that stream is where the work belongs: the mandatory
// list the select reads was uploaded before that point.  An entry point
// flushes what it depends on: the selection before anything that rewrites
// the scores, the plan or the block count; the reset before anything that
// reads or writes the block table.
kvm_status flush_select(kvm_session *s, cudaStream_t st) {
    if (!s->select_pending) return KVM_OK;
    s->select_pending = false;
    KVM_CUDA(s, launch_select(select_args(s, s->select_n_mandatory), st), "select launch");
    s->launches++;
    return KVM_OK;
}

kvm_status flush_reset(kvm_session *s, cudaStream_t st) {
    if (!s->reset_pending) return KVM_OK;
    s->reset_pending = false;
    KVM_CUDA(s, launch_reset_window(s->bt, s->n_blocks, st), "reset launch");
    s->launches++;
    return KVM_OK;
}

#define KVM_FLUSH_SEL(s)                                           \
    do {                                                           \
        const kvm_status f__ = flush_select(s, as_stream(stream)); \
        if (f__ != KVM_OK) return f__;                             \
    } while (0)
#define KVM_FLUSH_RESET(s)                                         \
    do {                                                           \
        const kvm_status f__ = flush_reset(s, as_stream(stream));  \
        if (f__ != KVM_OK) return f__;                             \
    } while (0)
#define KVM_FLUSH(s)                                               \
    do {                                                           \
        KVM_FLUSH_SEL(s);                                          \
        KVM_FLUSH_RESET(s);                                        \
    } while (0)

kvm_status upload_window(kvm_session *s, cudaStream_t st, const kvm_window *win) {
    const uint32_t L = s->cfg.n_layer;
    std::vector<void *> w(2u * L);
    for (uint32_t l = 0; l < L; ++l) {
        w[l] = win->d_k[l];
        w[L + l] = win->d_v[l];
        if (!w[l] || !w[L + l]) return fail(s, KVM_EINVAL, "window layer %u has a null base", l);
        // every copy into the window stores at least 2-byte words
        if ((reinterpret_cast<uintptr_t>(w[l]) | reinterpret_cast<uintptr_t>(w[L + l])) & 1u)
            return fail(s, KVM_EINVAL, "window layer %u base is not 2-byte aligned", l);
    }
    if (w != s->h_win) {
        const kvm_status r = upload_small(s, st, s->d_win, w.data(), w.size() * sizeof(void *));
        if (r != KVM_OK) return r;
        s->h_win = w;
    }
    return KVM_OK;
}

bool window_aligned16(const kvm_session *s) {
    for (void *p : s->h_win)
        if (reinterpret_cast<uintptr_t>(p) & 15u) return false;
    return true;
}

StageinArgs stagein_common(kvm_session *s) {
    StageinArgs a{};
    a.cold_block = s->plan.cold_block;
    a.cold_to = s->plan.cold_to;
    a.max_items = s->max_blocks;
    a.n_tokens = s->bt.n_tokens;
    a.max_blocks = s->max_blocks;
    a.dst_k = s->d_win;
    a.dst_v = s->d_win + s->cfg.n_layer;
    a.n_layer = s->cfg.n_layer;
    a.block_tokens = s->cfg.block_tokens;
    a.n_embd = s->n_embd;
    a.n_slots = s->n_slots;
    a.type_k = s->cfg.type_k;
    a.type_v = s->cfg.type_v;
    a.row_bytes_k = s->row_bytes_k;
    a.row_bytes_v = s->row_bytes_v;
    a.n_kv = 2;
    a.rows_per_tile = stagein_rows_per_tile(s->n_embd, s->cfg.block_tokens);
    a.tile_in_bytes = a.rows_per_tile * s->n_embd * 2u;
    const uint32_t out_max = a.rows_per_tile * std::max(s->row_bytes_k, s->row_bytes_v);
    a.tile_out_bytes = (out_max + 15u) & ~15u;
    a.bulk_store = (s->row_bytes_k % 16u == 0 && s->row_bytes_v % 16u == 0 && window_aligned16(s)) ? 1u : 0u;
    stagein_set_transform(a, s->cfg.head_dim, s->n_embd, s->xf.rot_k, s->xf.rot_v, s->xf.rope_n_rot,
                          s->d_theta);
    a.status = s->d_status;
    return a;
}

kvm_status launch_moves(kvm_session *s, cudaStream_t st) {
    // a plan made over an empty window moves nothing: skip the launch
    if (s->plan_moveless) return KVM_OK;
    PermuteArgs p{};
    p.n_moves_dev = &s->plan.hdr->n_moves;
    p.mv_block = s->plan.mv_block;
    p.mv_from = s->plan.mv_from;
    p.mv_to = s->plan.mv_to;
    p.max_moves = s->n_slots;
    p.n_tokens = s->bt.n_tokens;
    p.max_blocks = s->max_blocks;
    p.dst_k = s->d_win;
    p.dst_v = s->d_win + s->cfg.n_layer;
    p.n_layer = s->cfg.n_layer;
    p.block_tokens = s->cfg.block_tokens;
    p.n_slots = s->n_slots;
    p.row_bytes_k = s->row_bytes_k;
    p.row_bytes_v = s->row_bytes_v;
    p.span_k = s->row_bytes_k * s->cfg.block_tokens;
    p.span_v = s->row_bytes_v * s->cfg.block_tokens;
    // aligned windows: the streaming kernel, each (layer, K|V, piece) a stream,
    // pieces sized for about three streams an SM (2-16 KiB); otherwise the
    // SIMT column kernel, which sizes its column from the device move count
    // (any count up to n_slots fits 96 KiB at 16 bytes or more a move)
    p.vec16 = (p.span_k % 16u == 0 && p.span_v % 16u == 0 && s->row_bytes_k % 16u == 0 &&
               s->row_bytes_v % 16u == 0 && window_aligned16(s)) ? 1u : 0u;
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, s->device) != cudaSuccess || sms < 1)
        sms = 148;
    const uint64_t all = static_cast<uint64_t>(p.n_layer) * (p.span_k + p.span_v);
    uint64_t piece = (all / (3u * static_cast<uint64_t>(sms))) & ~static_cast<uint64_t>(15u);
    piece = std::min<uint64_t>(16384u, std::max<uint64_t>(2048u, piece));
    piece = std::max<uint64_t>(piece, (4u * s->n_slots + kChainStages - 1u) / kChainStages * 4u);
    p.piece = static_cast<uint32_t>((piece + 15u) & ~static_cast<uint64_t>(15u));
    p.col_region = std::max<uint32_t>(96u * 1024u, 16u * s->n_slots);
    p.col_bytes = 2048u;
    p.status = s->d_status;
    KVM_CUDA(s, launch_permute(p, st), "permute launch");
    s->launches++;
    return KVM_OK;
}

kvm_status source_check(kvm_session *s, const kvm_source *src) {
    if (!src || !src->k || !src->v) return fail(s, KVM_EINVAL, "null source");
    if (src->row_stride < 2ull * s->n_embd) return fail(s, KVM_EINVAL, "row_stride < 2*n_embd");
    if (src->location != KVM_LOC_DEVICE && src->location != KVM_LOC_HOST)
        return fail(s, KVM_EINVAL, "bad source location");
    if (src->location == KVM_LOC_DEVICE) {
        const uint64_t m = reinterpret_cast<uintptr_t>(src->k) | reinterpret_cast<uintptr_t>(src->v) |
                           src->layer_stride | src->block_stride | src->row_stride;
        if (m & 15u)
            return fail(s, KVM_EINVAL, "device source pointers and strides must be 16-byte aligned");
    }
    return KVM_OK;
}

// The plan's cold list on the host (one bounded wait for the header).
kvm_status read_cold_list(kvm_session *s, cudaStream_t st, std::vector<uint32_t> &cold) {
    cudaEvent_t ev_ready = s->ev[5];
    PlanHeader *hh = reinterpret_cast<PlanHeader *>(s->h_plan);
    KVM_CUDA(s, cudaMemcpyAsync(hh, s->plan.hdr, sizeof(PlanHeader), cudaMemcpyDeviceToHost, st), "hdr read");
    KVM_CUDA(s, cudaEventRecord(ev_ready, st), "hdr event");
    kvm_status r = wait_event(s, ev_ready, 30000);
    if (r != KVM_OK) return r;
    const uint32_t n_cold = std::min(hh->n_cold, s->max_blocks);
    cold.resize(n_cold);
    if (n_cold)
        KVM_CUDA(s, cudaMemcpy(cold.data(), s->plan.cold_block, n_cold * sizeof(uint32_t),
                               cudaMemcpyDeviceToHost), "cold read");
    return KVM_OK;
}

kvm_status ensure_ring(kvm_session *s, cudaStream_t st) {
    if (s->d_ring) return KVM_OK;
    // first host-source transfer: the ring is only needed on these paths
    KVM_CUDA(s, cudaStreamSynchronize(st), "ring allocation sync");
    KVM_CUDA(s, cudaMalloc(&s->d_ring, s->ring_bytes), "staging ring allocation");
    return KVM_OK;
}

PackedInArgs packed_common(kvm_session *s) {
    PackedInArgs a{};
    a.cold_block = s->plan.cold_block;
    a.cold_to = s->plan.cold_to;
    a.max_items = s->max_blocks;
    a.n_tokens = s->bt.n_tokens;
    a.max_blocks = s->max_blocks;
    a.n_slots = s->n_slots;
    a.n_layer = s->cfg.n_layer;
    a.block_tokens = s->cfg.block_tokens;
    a.win_k = s->d_win;
    a.win_v = s->d_win + s->cfg.n_layer;
    a.row_bytes_k = s->row_bytes_k;
    a.row_bytes_v = s->row_bytes_v;
    a.status = s->d_status;
    return a;
}

// Packed stage-in from pinned host memory: per chunk of cold blocks, H2D of
// their rows into a ring slot on the copy stream, then the copy kernel into
// the window slots on `st`.
kvm_status packed_from_host(kvm_session *s, cudaStream_t st, const kvm_packed_source *src) {
    const uint32_t L = s->cfg.n_layer;
    const uint32_t T = s->cfg.block_tokens;
    std::vector<uint32_t> cold;
    kvm_status r = read_cold_list(s, st, cold);
    if (r != KVM_OK) return r;
    const uint32_t n_cold = static_cast<uint32_t>(cold.size());
    if (n_cold == 0) return KVM_OK;
    const uint64_t span_k = static_cast<uint64_t>(T) * s->row_bytes_k;
    const uint64_t span_v = static_cast<uint64_t>(T) * s->row_bytes_v;
    const uint64_t item_bytes = static_cast<uint64_t>(L) * (span_k + span_v);
    const uint64_t slot_cap = s->ring_bytes / kvm_session::kRingSlots;
    if (item_bytes > slot_cap)
        return fail(s, KVM_ENOMEM, "staging ring slot (%llu B) smaller than one block (%llu B)",
                    static_cast<unsigned long long>(slot_cap), static_cast<unsigned long long>(item_bytes));
    r = ensure_ring(s, st);
    if (r != KVM_OK) return r;
    const uint32_t per_slot = static_cast<uint32_t>(slot_cap / item_bytes);
    PackedInArgs a = packed_common(s);
    a.src_by_item = 1;
    a.k_layer_stride = span_k;
    a.k_block_stride = item_bytes;
    a.v_layer_stride = span_v;
    a.v_block_stride = item_bytes;
    a.bulk = (s->row_bytes_k % 16u == 0 && s->row_bytes_v % 16u == 0 && window_aligned16(s)) ? 1u : 0u;
    KVM_CUDA(s, cudaEventRecord(s->ev[6], st), "ring start");
    KVM_CUDA(s, cudaStreamWaitEvent(s->copy_stream, s->ev[6], 0), "ring start wait");
    const uint8_t *hk = static_cast<const uint8_t *>(src->k);
    const uint8_t *hv = static_cast<const uint8_t *>(src->v);
    uint32_t chunk = 0;
    for (uint32_t i0 = 0; i0 < n_cold; i0 += per_slot, ++chunk) {
        const uint32_t m = std::min(per_slot, n_cold - i0);
        const int rs = static_cast<int>(chunk % kvm_session::kRingSlots);
        uint8_t *ring = s->d_ring + static_cast<uint64_t>(rs) * slot_cap;
        if (chunk >= static_cast<uint32_t>(kvm_session::kRingSlots))
            KVM_CUDA(s, cudaStreamWaitEvent(s->copy_stream, s->ring_free[rs], 0), "ring free wait");
        for (uint32_t j = 0; j < m; ++j) {
            const uint32_t b = cold[i0 + j];
            if (b >= s->n_blocks) return fail(s, KVM_EDEVICE, "cold block %u out of range", b);
            const uint32_t nt = std::min(s->h_n_tokens[b], T);
            if (nt == 0) continue;
            uint8_t *dk = ring + static_cast<uint64_t>(j) * item_bytes;
            KVM_CUDA(s, cudaMemcpy2DAsync(dk, span_k, hk + static_cast<uint64_t>(b) * src->k_block_stride,
                                          src->k_layer_stride, static_cast<size_t>(nt) * s->row_bytes_k, L,
                                          cudaMemcpyHostToDevice, s->copy_stream),
                     "packed ring H2D (K)");
            KVM_CUDA(s, cudaMemcpy2DAsync(dk + L * span_k, span_v, hv + static_cast<uint64_t>(b) * src->v_block_stride,
                                          src->v_layer_stride, static_cast<size_t>(nt) * s->row_bytes_v, L,
                                          cudaMemcpyHostToDevice, s->copy_stream),
                     "packed ring H2D (V)");
        }
        KVM_CUDA(s, cudaEventRecord(s->ring_copied[rs], s->copy_stream), "ring copied");
        KVM_CUDA(s, cudaStreamWaitEvent(st, s->ring_copied[rs], 0), "ring copied wait");
        a.src_k = ring;
        a.src_v = ring + L * span_k;
        a.item0 = i0;
        a.n_items_host = m;
        a.n_items_dev = nullptr;
        KVM_CUDA(s, launch_packed_stagein(a, st), "packed stage-in launch");
        s->launches++;
        KVM_CUDA(s, cudaEventRecord(s->ring_free[rs], st), "ring free");
    }
    return KVM_OK;
}

// Stage-in of cold blocks from pinned host memory: read the cold list back,
// then per chunk of blocks copy the F16 spans into an HBM ring slot on the
// copy stream and quantize that slot on `st` once its copy is done.
kvm_status stagein_from_host(kvm_session *s, cudaStream_t st, const kvm_source *src) {
    const uint32_t L = s->cfg.n_layer;
    const uint32_t T = s->cfg.block_tokens;
    std::vector<uint32_t> cold;
    kvm_status r = read_cold_list(s, st, cold);
    if (r != KVM_OK) return r;
    const uint32_t n_cold = static_cast<uint32_t>(cold.size());
    if (n_cold == 0) return KVM_OK;
    const uint64_t span = static_cast<uint64_t>(T) * s->n_embd * 2u;   // one (layer, K|V) of a block
    const uint64_t item_bytes = 2ull * L * span;
    const uint32_t per_slot = static_cast<uint32_t>(
        std::max<uint64_t>(1, (s->ring_bytes / kvm_session::kRingSlots) / item_bytes));
    if (item_bytes * per_slot * kvm_session::kRingSlots > s->ring_bytes)
        return fail(s, KVM_ENOMEM, "staging ring (%zu B) smaller than one block (%llu B) per slot",
                    s->ring_bytes, static_cast<unsigned long long>(item_bytes));
    const uint64_t slot_bytes = item_bytes * per_slot;
    r = ensure_ring(s, st);
    if (r != KVM_OK) return r;
    StageinArgs a = stagein_common(s);
    a.src_by_item = 1;
    a.layer_stride = span;
    a.item_stride = item_bytes;
    a.row_stride = 2ull * s->n_embd;
    // the ring is reused across calls: its previous consumers must be done
    KVM_CUDA(s, cudaEventRecord(s->ev[6], st), "ring start");
    KVM_CUDA(s, cudaStreamWaitEvent(s->copy_stream, s->ev[6], 0), "ring start wait");
    const uint8_t *hk = static_cast<const uint8_t *>(src->k);
    const uint8_t *hv = static_cast<const uint8_t *>(src->v);
    uint32_t chunk = 0;
    for (uint32_t i0 = 0; i0 < n_cold; i0 += per_slot, ++chunk) {
        const uint32_t m = std::min(per_slot, n_cold - i0);
        const int rs = static_cast<int>(chunk % kvm_session::kRingSlots);
        uint8_t *ring = s->d_ring + rs * slot_bytes;
        if (chunk >= static_cast<uint32_t>(kvm_session::kRingSlots))
            KVM_CUDA(s, cudaStreamWaitEvent(s->copy_stream, s->ring_free[rs], 0), "ring free wait");
        for (uint32_t j = 0; j < m; ++j) {
            const uint32_t b = cold[i0 + j];
            if (b >= s->n_blocks) return fail(s, KVM_EDEVICE, "cold block %u out of range", b);
            const uint32_t nt = std::min(s->h_n_tokens[b], T);
            for (int kv = 0; kv < 2; ++kv) {
                const uint8_t *hs = (kv ? hv : hk) + static_cast<uint64_t>(b) * src->block_stride;
                uint8_t *ds = ring + j * item_bytes + kv * L * span;
                const size_t row_in = 2ull * s->n_embd;
                if (src->row_stride == row_in) {
                    // one 2-D copy: L layer spans of nt rows each
                    KVM_CUDA(s, cudaMemcpy2DAsync(ds, span, hs, src->layer_stride, nt * row_in, L,
                                                  cudaMemcpyHostToDevice, s->copy_stream),
                             "ring H2D");
                } else {
                    for (uint32_t l = 0; l < L; ++l) {
                        KVM_CUDA(s, cudaMemcpy2DAsync(ds + l * span, row_in, hs + l * src->layer_stride,
                                                      src->row_stride, row_in, nt,
                                                      cudaMemcpyHostToDevice, s->copy_stream),
                                 "ring H2D");
                    }
                }
            }
        }
        KVM_CUDA(s, cudaEventRecord(s->ring_copied[rs], s->copy_stream), "ring copied");
        KVM_CUDA(s, cudaStreamWaitEvent(st, s->ring_copied[rs], 0), "ring copied wait");
        a.src_k = ring;
        a.src_v = ring + static_cast<uint64_t>(L) * span;
        a.item0 = i0;
        a.n_items_host = m;
        a.n_items_dev = nullptr;
        KVM_CUDA(s, launch_stagein(a, st, 0), "stage-in launch");
        s->launches++;
        KVM_CUDA(s, cudaEventRecord(s->ring_free[rs], st), "ring free");
    }
    return KVM_OK;
}

}  // namespace

static thread_local std::string g_create_err;

namespace kvm {
// Message for kvm_last_error(NULL) from entry points that take no session.
void set_sessionless_error(const char *msg) { g_create_err = msg ? msg : ""; }
}  // namespace kvm

// ==================================================================== ABI ==

extern "C" {

void kvm_config_default(kvm_config *c) {
    if (!c) return;
    std::memset(c, 0, sizeof *c);
    c->block_tokens = 128;
    c->select_budget = 131072;
    c->gen_reserve = 32768;
    c->sink_blocks = 1;
    c->recent_blocks = 0;
    c->n_layer = 1;
    c->n_head_kv = 4;
    c->head_dim = 256;
    c->n_head_q = 24;
    c->max_blocks = 8192;
    c->type_k = KVM_TYPE_Q8_0;
    c->type_v = KVM_TYPE_Q8_0;
    c->optimize_stage_in = 1;
    c->immutable_source_k = 0;
    c->immutable_refresh_remaps = 8;
    c->immutable_refresh_abs_delta_tokens = 262144;
    c->immutable_max_baked_position = 262144;
    c->staging_bytes = 256ull << 20;
}

uint64_t kvm_row_bytes(int32_t type, uint32_t n_embd) {
    switch (type) {
        case KVM_TYPE_F16: return 2ull * n_embd;
        case KVM_TYPE_Q8_0: return (n_embd / 32ull) * 34ull;
        case KVM_TYPE_Q4_0: return (n_embd / 32ull) * 18ull;
        case KVM_TYPE_Q5_0: return (n_embd / 32ull) * 22ull;
        default: return 0;
    }
}


const char *kvm_last_error(const kvm_session *s) {
    if (!s) return g_create_err.c_str();
    return s->err.c_str();
}

uint32_t kvm_window_slots(const kvm_session *s) { return s ? s->n_slots : 0; }
uint32_t kvm_block_count(const kvm_session *s) { return s ? s->n_blocks : 0; }
uint64_t kvm_kernel_launches(const kvm_session *s) { return s ? s->launches : 0; }

void kvm_session_destroy(kvm_session *s) {
    if (!s) return;
    {
        DeviceGuard g(s->device);
        cudaDeviceSynchronize();
        cudaFree(s->sum.sum_t);
        cudaFree(s->d_base);
        cudaFree(s->d_ring);
        cudaFree(s->d_keep);
        if (s->h_pin) cudaFreeHost(s->h_pin);
        if (s->h_plan) cudaFreeHost(s->h_plan);
        for (auto &e : s->pin_ev) if (e) cudaEventDestroy(e);
        for (auto &e : s->ring_copied) if (e) cudaEventDestroy(e);
        for (auto &e : s->ring_free) if (e) cudaEventDestroy(e);
        for (auto &e : s->out_gathered) if (e) cudaEventDestroy(e);
        for (auto &e : s->out_done) if (e) cudaEventDestroy(e);
        for (auto &e : s->ev) if (e) cudaEventDestroy(e);
        if (s->copy_stream) cudaStreamDestroy(s->copy_stream);
    }
    delete s;
}

kvm_status kvm_session_create(const kvm_config *cfg, int device, kvm_session **out) {
    g_create_err.clear();
    if (!out) return KVM_EINVAL;
    *out = nullptr;
    if (!cfg) {
        g_create_err = "null config";
        return KVM_EINVAL;
    }
    const kvm_config &c = *cfg;
    auto bad = [&](const char *m) {
        g_create_err = m;
        return KVM_EINVAL;
    };
    if (c.block_tokens == 0) return bad("block_tokens must be > 0");
    if (c.n_layer == 0 || c.n_layer > kMaxLayers) return bad("n_layer must be in [1, 256]");
    if (c.n_head_kv == 0 || c.n_head_kv > 32) return bad("n_head_kv must be in [1, 32]");
    if (c.head_dim == 0 || c.head_dim > kMaxHeadDim) return bad("head_dim must be in [1, 1024]");
    if (c.n_head_q == 0) return bad("n_head_q must be > 0");
    const uint32_t E = c.n_head_kv * c.head_dim;
    if (E % 32u != 0) return bad("n_head_kv * head_dim must be a multiple of 32 (ggml block)");
    if (E > 16384u) return bad("n_head_kv * head_dim must be <= 16384");
    if (c.max_blocks == 0 || c.max_blocks > kMaxBlocks) return bad("max_blocks must be in [1, 65536]");
    if (!type_ok(c.type_k) || !type_ok(c.type_v)) return bad("type_k/type_v must be F16, Q8_0, Q4_0 or Q5_0");
    const uint32_t budget = align_tokens(c.select_budget, c.block_tokens);
    const uint32_t gen = align_tokens(c.gen_reserve ? c.gen_reserve : 256u, c.block_tokens);
    // Like KvMemStore, sink + recent beyond the budget is accepted: the pins
    // are best effort in the selector (kvmem_store.cpp:505-535).
    const uint32_t budget_blocks = budget / c.block_tokens;
    const uint64_t slots = (static_cast<uint64_t>(budget) + gen) / c.block_tokens;
    if (slots > kMaxBlocks) return bad("window slots exceed 65536");

    kvm_session *s = new (std::nothrow) kvm_session();
    if (!s) {
        g_create_err = "host allocation failed";
        return KVM_ENOMEM;
    }
    s->cfg = c;
    s->cfg.select_budget = budget;
    s->cfg.gen_reserve = gen;
    s->device = device;
    s->n_embd = E;
    s->budget_blocks = budget_blocks;
    s->n_slots = static_cast<uint32_t>(slots);
    s->max_blocks = c.max_blocks;
    s->row_bytes_k = static_cast<uint32_t>(kvm_row_bytes(c.type_k, E));
    s->row_bytes_v = static_cast<uint32_t>(kvm_row_bytes(c.type_v, E));
    s->h_n_tokens.reserve(c.max_blocks);
    s->h_slot.reserve(c.max_blocks);
    DeviceGuard g(device);
    auto cleanup = [&](cudaError_t e, const char *what) {
        g_create_err = std::string(what) + ": " + cudaGetErrorString(e);
        const kvm_status st = e == cudaErrorMemoryAllocation ? KVM_ENOMEM : KVM_ECUDA;
        kvm_session_destroy(s);
        return st;
    };
    cudaError_t e;
    const uint32_t ldb = (c.max_blocks + kSumGroup - 1u) / kSumGroup * kSumGroup;
    const uint32_t L = c.n_layer;
    s->sum.ldb = ldb;
    s->sum.n_layer = L;
    s->sum.n_embd = E;
    e = cudaMalloc(&s->sum.sum_t, static_cast<size_t>(L) * E * ldb * sizeof(float));
    if (e != cudaSuccess) return cleanup(e, "summary allocation");
    e = cudaMemset(s->sum.sum_t, 0, static_cast<size_t>(L) * E * ldb * sizeof(float));
    if (e != cudaSuccess) return cleanup(e, "summary clear");

    // one allocation for everything small (256-byte aligned sub-buffers)
    struct Item { void **p; size_t bytes; };
    const size_t nb = c.max_blocks;
    const size_t stage_cap = std::min<size_t>(nb, 1024);
    s->stage_sums_cap = stage_cap;
    std::vector<Item> items = {
        {reinterpret_cast<void **>(&s->sum.mean_tok), sizeof(uint32_t) * L * ldb},
        {reinterpret_cast<void **>(&s->sum.inv_tok), sizeof(float) * L * ldb},
        {reinterpret_cast<void **>(&s->q.q_sum), sizeof(float) * L * c.n_head_q * c.head_dim},
        {reinterpret_cast<void **>(&s->q.q_count), sizeof(uint32_t) * L},
        {reinterpret_cast<void **>(&s->q.qv), sizeof(float) * L * E},
        {reinterpret_cast<void **>(&s->q.nq), sizeof(float) * L * c.n_head_kv},
        {reinterpret_cast<void **>(&s->d_terms), sizeof(double) * L * ldb},
        {reinterpret_cast<void **>(&s->d_range_done), sizeof(uint32_t) * (ldb / kScoreRange)},
        {reinterpret_cast<void **>(&s->d_scores), sizeof(double) * ldb},
        {reinterpret_cast<void **>(&s->d_acc), sizeof(double) * ldb},
        {reinterpret_cast<void **>(&s->bt.n_tokens), sizeof(uint32_t) * nb},
        {reinterpret_cast<void **>(&s->bt.tier), nb},
        {reinterpret_cast<void **>(&s->bt.gpu_slot), sizeof(int32_t) * nb},
        {reinterpret_cast<void **>(&s->bt.baked_pos), sizeof(int64_t) * nb},
        {reinterpret_cast<void **>(&s->bt.remap_count), sizeof(uint32_t) * nb},
        {reinterpret_cast<void **>(&s->bt.remap_abs_delta), sizeof(uint64_t) * nb},
        {reinterpret_cast<void **>(&s->bt.in_ws), nb},
        {reinterpret_cast<void **>(&s->plan.hdr), sizeof(PlanHeader)},
        {reinterpret_cast<void **>(&s->plan.selected), sizeof(uint32_t) * nb},
        {reinterpret_cast<void **>(&s->plan.stage_in), sizeof(uint32_t) * nb},
        {reinterpret_cast<void **>(&s->plan.stage_out), sizeof(uint32_t) * nb},
        {reinterpret_cast<void **>(&s->plan.rm_block_id), sizeof(uint32_t) * nb},
        {reinterpret_cast<void **>(&s->plan.rm_n_tokens), sizeof(uint32_t) * nb},
        {reinterpret_cast<void **>(&s->plan.rm_from_base), sizeof(int32_t) * nb},
        {reinterpret_cast<void **>(&s->plan.rm_to_base), sizeof(int32_t) * nb},
        {reinterpret_cast<void **>(&s->plan.rm_wkr), nb},
        {reinterpret_cast<void **>(&s->plan.rm_skip), nb},
        {reinterpret_cast<void **>(&s->plan.rm_raw), nb},
        {reinterpret_cast<void **>(&s->plan.mv_block), sizeof(uint32_t) * nb},
        {reinterpret_cast<void **>(&s->plan.mv_from), sizeof(int32_t) * nb},
        {reinterpret_cast<void **>(&s->plan.mv_to), sizeof(int32_t) * nb},
        {reinterpret_cast<void **>(&s->plan.cold_block), sizeof(uint32_t) * nb},
        {reinterpret_cast<void **>(&s->plan.cold_to), sizeof(int32_t) * nb},
        {reinterpret_cast<void **>(&s->d_mandatory), sizeof(uint32_t) * nb},
        {reinterpret_cast<void **>(&s->d_ids), sizeof(uint32_t) * nb},
        {reinterpret_cast<void **>(&s->d_status), sizeof(uint32_t)},
        {reinterpret_cast<void **>(&s->d_win), sizeof(void *) * 2 * L},
        {reinterpret_cast<void **>(&s->d_stage_sums), sizeof(float) * stage_cap * E},
        {reinterpret_cast<void **>(&s->d_stage_counts), sizeof(uint32_t) * stage_cap},
        {reinterpret_cast<void **>(&s->d_meank), sizeof(float) * L * E},
        {reinterpret_cast<void **>(&s->d_theta), sizeof(float) * (kMaxHeadDim / 2)},
        {reinterpret_cast<void **>(&s->d_out_ids), sizeof(uint32_t) * nb},
        {reinterpret_cast<void **>(&s->d_out_flags), nb},
        {reinterpret_cast<void **>(&s->d_group_spans), sizeof(uint32_t) * 2 * kMaxGroups},
        {reinterpret_cast<void **>(&s->d_group_scores), sizeof(double) * kMaxGroups},
    };
    size_t total = 0;
    for (auto &it : items) total += (it.bytes + 255u) & ~static_cast<size_t>(255u);
    e = cudaMalloc(&s->d_base, total);
    if (e != cudaSuccess) return cleanup(e, "state allocation");
    e = cudaMemset(s->d_base, 0, total);
    if (e != cudaSuccess) return cleanup(e, "state clear");
    {
        uint8_t *p = static_cast<uint8_t *>(s->d_base);
        for (auto &it : items) {
            *it.p = p;
            p += (it.bytes + 255u) & ~static_cast<size_t>(255u);
        }
    }
    // gpu_slot = -1 everywhere
    e = cudaMemset(s->bt.gpu_slot, 0xff, sizeof(int32_t) * nb);
    if (e != cudaSuccess) return cleanup(e, "slot clear");
    // the HBM staging ring is allocated on the first stage-in from a host source
    s->ring_bytes = c.staging_bytes ? c.staging_bytes : (256ull << 20);
    s->pin_slot_bytes = std::max<size_t>(64u * 1024u, std::max<size_t>(4u * nb, sizeof(void *) * 2 * L));
    e = cudaHostAlloc(reinterpret_cast<void **>(&s->h_pin), s->pin_slot_bytes * kPinSlots, cudaHostAllocDefault);
    if (e != cudaSuccess) return cleanup(e, "pinned ring allocation");
    s->h_plan_bytes = sizeof(PlanHeader);
    e = cudaHostAlloc(reinterpret_cast<void **>(&s->h_plan), s->h_plan_bytes, cudaHostAllocDefault);
    if (e != cudaSuccess) return cleanup(e, "pinned plan allocation");
    for (auto &ev : s->pin_ev) {
        e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
        if (e != cudaSuccess) return cleanup(e, "event");
    }
    for (int i = 0; i < kvm_session::kRingSlots; ++i) {
        e = cudaEventCreateWithFlags(&s->ring_copied[i], cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s->ring_free[i], cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s->out_gathered[i], cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s->out_done[i], cudaEventDisableTiming);
        if (e != cudaSuccess) return cleanup(e, "event");
    }
    for (auto &ev : s->ev) {
        e = cudaEventCreate(&ev);
        if (e != cudaSuccess) return cleanup(e, "event");
    }
    e = cudaStreamCreateWithFlags(&s->copy_stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) return cleanup(e, "copy stream");
    *out = s;
    return KVM_OK;
}

kvm_status kvm_register_append(kvm_session *s, kvm_stream stream, uint32_t n_new, int resident) {
    if (!s) return KVM_EINVAL;
    if (n_new == 0) return KVM_OK;
    DeviceGuard g(s->device);
    KVM_FLUSH(s);
    cudaStream_t st = as_stream(stream);
    const uint32_t bt = s->cfg.block_tokens;
    // plan the append on the host (KvMemStore::register_append)
    std::vector<uint32_t> nt = s->h_n_tokens;
    uint32_t total = s->total_tokens;
    uint32_t first_changed = static_cast<uint32_t>(nt.size());
    uint32_t remaining = n_new;
    if (!nt.empty() && nt.back() < bt) {
        const uint32_t take = std::min(bt - nt.back(), remaining);
        nt.back() += take;
        remaining -= take;
        total += take;
        first_changed = static_cast<uint32_t>(nt.size() - 1);
    }
    const uint32_t first_new = static_cast<uint32_t>(nt.size());
    while (remaining > 0) {
        const uint32_t take = std::min(bt, remaining);
        nt.push_back(take);
        total += take;
        remaining -= take;
    }
    const uint32_t n = static_cast<uint32_t>(nt.size());
    if (n > s->max_blocks)
        return fail(s, KVM_EINVAL, "block table full: %u blocks > max_blocks %u", n, s->max_blocks);
    const uint32_t n_add = n - first_new;
    std::vector<uint8_t> tier(n_add, resident ? KVM_TIER_GPU : KVM_TIER_CPU);
    std::vector<int32_t> slot(n_add, -1);
    std::vector<int64_t> baked(n_add);
    for (uint32_t i = 0; i < n_add; ++i) baked[i] = static_cast<int64_t>(first_new + i) * bt;
    std::vector<int32_t> hs = s->h_slot;
    hs.resize(n, -1);
    if (resident) {
        if (!s->slots_known)
            return fail(s, KVM_ESTATE, "resident append needs the previous plan (kvm_get_plan) first");
        if (first_changed < first_new && hs[first_changed] < 0)
            return fail(s, KVM_ESTATE, "resident append extends block %u, which is not in the window",
                        first_changed);
        std::vector<uint8_t> used(s->n_slots, 0);
        for (uint32_t i = 0; i < first_new; ++i)
            if (hs[i] >= 0 && static_cast<uint32_t>(hs[i]) < s->n_slots) used[hs[i]] = 1;
        uint32_t next = 0;
        for (uint32_t i = 0; i < n_add; ++i) {
            while (next < s->n_slots && used[next]) ++next;
            if (next >= s->n_slots)
                return fail(s, KVM_ENOMEM, "no free window slot for appended block %u", first_new + i);
            slot[i] = static_cast<int32_t>(next);
            used[next] = 1;
            hs[first_new + i] = slot[i];
        }
    }
    kvm_status r = upload_small(s, st, s->bt.n_tokens + first_changed, nt.data() + first_changed,
                                sizeof(uint32_t) * (n - first_changed));
    if (r == KVM_OK && n_add) {
        r = upload_small(s, st, s->bt.tier + first_new, tier.data(), n_add);
        if (r == KVM_OK) r = upload_small(s, st, s->bt.gpu_slot + first_new, slot.data(), 4u * n_add);
        if (r == KVM_OK && resident) s->window_empty = false;
        if (r == KVM_OK) r = upload_small(s, st, s->bt.baked_pos + first_new, baked.data(), 8u * n_add);
        if (r == KVM_OK) KVM_CUDA(s, cudaMemsetAsync(s->bt.remap_count + first_new, 0, 4u * n_add, st), "clear");
        if (r == KVM_OK) KVM_CUDA(s, cudaMemsetAsync(s->bt.remap_abs_delta + first_new, 0, 8u * n_add, st), "clear");
        if (r == KVM_OK) KVM_CUDA(s, cudaMemsetAsync(s->bt.in_ws + first_new, 0, n_add, st), "clear");
    }
    if (r != KVM_OK) return r;
    s->h_n_tokens.swap(nt);
    s->h_slot.swap(hs);
    s->n_blocks = n;
    s->total_tokens = total;
    return KVM_OK;
}

kvm_status kvm_set_block_tier(kvm_session *s, kvm_stream stream, uint32_t block_id, int32_t tier) {
    if (!s) return KVM_EINVAL;
    if (block_id >= s->n_blocks) return KVM_OK;   // the reference ignores unknown ids
    if (tier != KVM_TIER_GPU && tier != KVM_TIER_CPU && tier != KVM_TIER_SSD)
        return fail(s, KVM_EINVAL, "bad tier %d", tier);
    DeviceGuard g(s->device);
    KVM_FLUSH_RESET(s);
    cudaStream_t st = as_stream(stream);
    const uint8_t t = static_cast<uint8_t>(tier);
    kvm_status r = upload_small(s, st, s->bt.tier + block_id, &t, 1);
    if (r == KVM_OK && tier != KVM_TIER_GPU) {
        const int32_t none = -1;
        r = upload_small(s, st, s->bt.gpu_slot + block_id, &none, sizeof none);
        if (r == KVM_OK && block_id < s->h_slot.size()) s->h_slot[block_id] = -1;
    }
    return r;
}

kvm_status kvm_set_block_gpu_slot(kvm_session *s, kvm_stream stream, uint32_t block_id, int32_t slot) {
    if (!s) return KVM_EINVAL;
    if (block_id >= s->n_blocks) return KVM_OK;
    if (slot >= static_cast<int32_t>(s->n_slots)) return fail(s, KVM_EINVAL, "slot %d >= window slots", slot);
    DeviceGuard g(s->device);
    KVM_FLUSH_RESET(s);
    const int32_t v = slot < 0 ? -1 : slot;
    kvm_status r = upload_small(s, as_stream(stream), s->bt.gpu_slot + block_id, &v, sizeof v);
    if (r == KVM_OK && block_id < s->h_slot.size()) s->h_slot[block_id] = v;
    if (r == KVM_OK && v >= 0) s->window_empty = false;
    return r;
}

kvm_status kvm_reset_window(kvm_session *s, kvm_stream stream) {
    if (!s) return KVM_EINVAL;
    DeviceGuard g(s->device);
    // a pending select does not read the block table: it may stay pending
    // and fuse with the next diff, which also applies this reset (the
    // stream argument orders nothing until a later call launches the reset)
    (void)stream;
    if (s->n_blocks) s->reset_pending = true;
    std::fill(s->h_slot.begin(), s->h_slot.end(), -1);
    s->slots_known = true;
    s->window_empty = true;
    s->have_plan = false;
    return KVM_OK;
}

kvm_status kvm_upload_summaries(kvm_session *s, kvm_stream stream, uint32_t layer, uint32_t block0,
                                uint32_t n, const float *sums, const uint32_t *counts) {
    if (!s) return KVM_EINVAL;
    if (layer >= s->cfg.n_layer) return fail(s, KVM_EINVAL, "layer %u >= n_layer", layer);
    if (static_cast<uint64_t>(block0) + n > s->max_blocks) return fail(s, KVM_EINVAL, "blocks beyond max_blocks");
    if (n && (!sums || !counts)) return fail(s, KVM_EINVAL, "null sums/counts");
    DeviceGuard g(s->device);
    cudaStream_t st = as_stream(stream);
    const uint32_t E = s->n_embd;
    for (uint32_t off = 0; off < n;) {
        const uint32_t m = std::min<uint32_t>(n - off, static_cast<uint32_t>(s->stage_sums_cap));
        KVM_CUDA(s, cudaMemcpyAsync(s->d_stage_sums, sums + static_cast<size_t>(off) * E,
                                    sizeof(float) * m * E, cudaMemcpyDefault, st), "sums copy");
        KVM_CUDA(s, cudaMemcpyAsync(s->d_stage_counts, counts + off, sizeof(uint32_t) * m,
                                    cudaMemcpyDefault, st), "counts copy");
        KVM_CUDA(s, launch_upload_summaries(s->sum, layer, block0 + off, m, s->d_stage_sums,
                                            s->d_stage_counts, st), "summary upload");
        s->launches++;
        off += m;
    }
    return KVM_OK;
}

kvm_status kvm_download_summaries(kvm_session *s, kvm_stream stream, uint32_t layer, uint32_t block0,
                                  uint32_t n, float *sums, uint32_t *counts) {
    if (!s) return KVM_EINVAL;
    if (layer >= s->cfg.n_layer) return fail(s, KVM_EINVAL, "layer %u >= n_layer", layer);
    if (static_cast<uint64_t>(block0) + n > s->max_blocks) return fail(s, KVM_EINVAL, "blocks beyond max_blocks");
    DeviceGuard g(s->device);
    cudaStream_t st = as_stream(stream);
    const uint32_t E = s->n_embd;
    if (counts && n)
        KVM_CUDA(s, cudaMemcpyAsync(counts, s->sum.mean_tok + static_cast<size_t>(layer) * s->sum.ldb + block0,
                                    sizeof(uint32_t) * n, cudaMemcpyDefault, st), "counts copy");
    for (uint32_t off = 0; sums && off < n;) {
        const uint32_t m = std::min<uint32_t>(n - off, static_cast<uint32_t>(s->stage_sums_cap));
        KVM_CUDA(s, launch_download_summaries(s->sum, layer, block0 + off, m, s->d_stage_sums, st),
                 "summary download");
        s->launches++;
        KVM_CUDA(s, cudaMemcpyAsync(sums + static_cast<size_t>(off) * E, s->d_stage_sums,
                                    sizeof(float) * m * E, cudaMemcpyDefault, st), "sums copy");
        off += m;
    }
    return KVM_OK;
}

kvm_status kvm_summarize(kvm_session *s, kvm_stream stream, uint32_t layer0, uint32_t n_layers,
                         uint32_t block0, uint32_t n, const kvm_source *src) {
    if (!s) return KVM_EINVAL;
    if (static_cast<uint64_t>(layer0) + n_layers > s->cfg.n_layer) return fail(s, KVM_EINVAL, "layers out of range");
    if (static_cast<uint64_t>(block0) + n > s->n_blocks) return fail(s, KVM_EINVAL, "blocks beyond block_count");
    if (!src || !src->k || src->location != KVM_LOC_DEVICE)
        return fail(s, KVM_EINVAL, "kvm_summarize needs a device-resident source");
    if ((reinterpret_cast<uintptr_t>(src->k) | src->row_stride | src->layer_stride | src->block_stride) & 1u)
        return fail(s, KVM_EINVAL, "F16 source must be 2-byte aligned");
    DeviceGuard g(s->device);
    MeanKArgs a{};
    a.sum = s->sum;
    a.src = static_cast<const uint8_t *>(src->k);
    a.type = kActF16;
    a.head_dim = s->cfg.head_dim;
    a.nb_dim = 2;
    a.nb_head = 2ull * s->cfg.head_dim;
    a.nb_row = src->row_stride;
    a.nb_block = src->block_stride;
    a.nb_layer = src->layer_stride;
    a.vec = mean_k_vec(a.type, a.head_dim, a.nb_dim,
                       reinterpret_cast<uintptr_t>(src->k) | src->row_stride | src->block_stride |
                           src->layer_stride | a.nb_head);
    a.layer0 = layer0;
    a.block0 = block0;
    a.n_blk = n;
    a.block_tokens = s->cfg.block_tokens;
    a.n_tokens = s->bt.n_tokens;
    KVM_CUDA(s, launch_mean_k(a, n_layers, as_stream(stream)), "summarize launch");
    s->launches++;
    return KVM_OK;
}

namespace {

kvm_status check_rows(kvm_session *s, const kvm_rows *r, uint32_t width, const char *what) {
    if (!r || !r->data) return fail(s, KVM_EINVAL, "%s: null rows", what);
    if (r->type != KVM_TYPE_F32 && r->type != KVM_TYPE_F16 && r->type != KVM_TYPE_BF16)
        return fail(s, KVM_EINVAL, "%s: rows must be F32, F16 or BF16", what);
    if (r->head_dim == 0 || static_cast<uint64_t>(r->n_head) * r->head_dim != width)
        return fail(s, KVM_EINVAL, "%s: n_head*head_dim must be %u", what, width);
    const uint64_t es = r->type == KVM_TYPE_F32 ? 4u : 2u;
    const uint64_t m = reinterpret_cast<uintptr_t>(r->data) | r->nb_dim | r->nb_head | r->nb_tok;
    if (m & (es - 1u)) return fail(s, KVM_EINVAL, "%s: rows not aligned to their element size", what);
    return KVM_OK;
}

AddRowsArgs add_rows_args(const kvm_rows *r, float *acc, uint32_t n_elem) {
    AddRowsArgs a{};
    a.acc = acc;
    a.n_elem = n_elem;
    a.src = static_cast<const uint8_t *>(r->data);
    a.type = r->type;
    a.head_dim = r->head_dim;
    a.nb_dim = r->nb_dim;
    a.nb_head = r->nb_head;
    a.nb_tok = r->nb_tok;
    return a;
}

// After the query changed: upload q_count; *prep tells the scorer launch to
// run the query prep (qv, nq) first.
kvm_status ensure_query(kvm_session *s, cudaStream_t st, bool *prep) {
    *prep = s->q_dirty;
    if (!s->q_dirty) return KVM_OK;
    const uint32_t L = s->cfg.n_layer;
    return upload_small(s, st, s->q.q_count, s->h_q_count.data(), sizeof(uint32_t) * L);
}

}  // namespace

uint32_t kvm_attn_rot_nrot(int32_t type, uint32_t head_dim, int is_k) {
    // kvmem_attn_rot_on: quantized cache, head_dim a multiple of 64
    if (type != KVM_TYPE_Q8_0 && type != KVM_TYPE_Q4_0 && type != KVM_TYPE_Q5_0) return 0u;
    if (head_dim < 64u || head_dim % 64u != 0u) return 0u;
    if (!is_k) return 64u;                              // kvmem_hadamard_nrot_v
    uint32_t nrot = 64u;                                // kvmem_hadamard_nrot_k
    do {
        nrot *= 2u;
    } while (head_dim % nrot == 0u);
    return nrot / 2u;
}

kvm_status kvm_set_transform(kvm_session *s, const kvm_transform *t) {
    if (!s) return KVM_EINVAL;
    if (!t) {
        s->xf = kvm_transform{};
        return KVM_OK;
    }
    const uint32_t D = s->cfg.head_dim;
    auto rot_ok = [&](uint32_t n) {
        return n == 0u || ((n == 64u || n == 128u || n == 256u || n == 512u) && D % n == 0u);
    };
    if (!rot_ok(t->rot_k) || !rot_ok(t->rot_v))
        return fail(s, KVM_EINVAL, "rot_k / rot_v must be 0, 64, 128, 256 or 512 and divide head_dim");
    if (t->rope_n_rot % 64u != 0u || t->rope_n_rot > D)
        return fail(s, KVM_EINVAL, "rope_n_rot must be a multiple of 64 up to head_dim");
    const bool on = t->rot_k || t->rot_v || t->rope_n_rot;
    if (on && (D % 32u != 0u || D > 1024u))
        return fail(s, KVM_EINVAL, "transforms need head_dim a multiple of 32, at most 1024");
    auto quantized = [](int32_t ty) {
        return ty == KVM_TYPE_Q8_0 || ty == KVM_TYPE_Q4_0 || ty == KVM_TYPE_Q5_0;
    };
    if ((t->rot_k && !quantized(s->cfg.type_k)) || (t->rot_v && !quantized(s->cfg.type_v)))
        return fail(s, KVM_EINVAL, "a Hadamard transform needs a quantized window type");
    if (t->rope_n_rot) {
        // kvmem::rope_neox_apply, kvmem/src/host/rope.cpp:18-22
        const uint32_t half = t->rope_n_rot / 2u;
        std::vector<float> theta(half);
        for (uint32_t i = 0; i < half; ++i) {
            theta[i] = powf(t->rope_freq_base,
                            -2.0f * static_cast<float>(i) / static_cast<float>(t->rope_n_rot));
            theta[i] *= t->rope_freq_scale;
        }
        DeviceGuard g(s->device);
        // later stage-ins read the table: wait for earlier ones to finish with it
        KVM_CUDA(s, cudaDeviceSynchronize(), "transform sync");
        KVM_CUDA(s, cudaMemcpy(s->d_theta, theta.data(), sizeof(float) * half, cudaMemcpyHostToDevice),
                 "theta upload");
    }
    s->xf = *t;
    return KVM_OK;
}

kvm_status kvm_write_mean_k(kvm_session *s, kvm_stream stream, uint32_t layer, uint32_t pos0, uint32_t n,
                            const kvm_rows *k) {
    if (!s) return KVM_EINVAL;
    if (n == 0) return KVM_OK;
    if (layer >= s->cfg.n_layer) return fail(s, KVM_EINVAL, "layer out of range");
    const uint32_t T = s->cfg.block_tokens;
    if (static_cast<uint64_t>(pos0) + n > static_cast<uint64_t>(s->max_blocks) * T)
        return fail(s, KVM_EINVAL, "positions beyond max_blocks");
    kvm_status r = check_rows(s, k, s->n_embd, "kvm_write_mean_k");
    if (r != KVM_OK) return r;
    DeviceGuard g(s->device);
    MeanKArgs a{};
    a.sum = s->sum;
    a.src = static_cast<const uint8_t *>(k->data);
    a.type = k->type;
    a.head_dim = k->head_dim;
    a.nb_dim = k->nb_dim;
    a.nb_head = k->nb_head;
    a.nb_row = k->nb_tok;
    a.vec = mean_k_vec(a.type, a.head_dim, a.nb_dim,
                       reinterpret_cast<uintptr_t>(k->data) | k->nb_head | k->nb_tok);
    a.layer0 = layer;
    a.block0 = pos0 / T;
    a.n_blk = (pos0 + n - 1u) / T - a.block0 + 1u;
    a.block_tokens = T;
    a.pos0 = pos0;
    a.n = n;
    KVM_CUDA(s, launch_mean_k(a, 1, as_stream(stream)), "mean-k launch");
    s->launches++;
    return KVM_OK;
}

kvm_status kvm_meank_add(kvm_session *s, kvm_stream stream, uint32_t layer, uint32_t tok0, uint32_t n,
                         const kvm_rows *k) {
    if (!s) return KVM_EINVAL;
    if (n == 0) return KVM_OK;
    if (layer >= s->cfg.n_layer) return fail(s, KVM_EINVAL, "layer out of range");
    kvm_status r = check_rows(s, k, s->n_embd, "kvm_meank_add");
    if (r != KVM_OK) return r;
    DeviceGuard g(s->device);
    AddRowsArgs a = add_rows_args(k, s->d_meank + static_cast<size_t>(layer) * s->n_embd, s->n_embd);
    a.tok0 = tok0;
    a.n = n;
    KVM_CUDA(s, launch_add_rows(a, as_stream(stream)), "meank add");
    s->launches++;
    return KVM_OK;
}

kvm_status kvm_meank_flush(kvm_session *s, kvm_stream stream, uint32_t layer0, uint32_t n_layers, uint32_t pos0,
                           uint32_t n) {
    if (!s) return KVM_EINVAL;
    if (n == 0 || n_layers == 0) return KVM_OK;
    if (static_cast<uint64_t>(layer0) + n_layers > s->cfg.n_layer) return fail(s, KVM_EINVAL, "layers out of range");
    if (pos0 / s->cfg.block_tokens >= s->max_blocks) return fail(s, KVM_EINVAL, "position beyond max_blocks");
    DeviceGuard g(s->device);
    KVM_CUDA(s, launch_meank_flush(s->sum, s->d_meank, layer0, n_layers, pos0, n, s->cfg.block_tokens,
                                   as_stream(stream)),
             "meank flush");
    s->launches++;
    return KVM_OK;
}

kvm_status kvm_meank_zero(kvm_session *s, kvm_stream stream, uint32_t layer0, uint32_t n_layers) {
    if (!s) return KVM_EINVAL;
    if (static_cast<uint64_t>(layer0) + n_layers > s->cfg.n_layer) return fail(s, KVM_EINVAL, "layers out of range");
    DeviceGuard g(s->device);
    KVM_CUDA(s, cudaMemsetAsync(s->d_meank + static_cast<size_t>(layer0) * s->n_embd, 0,
                                sizeof(float) * n_layers * s->n_embd, as_stream(stream)),
             "meank zero");
    return KVM_OK;
}

kvm_status kvm_query_reset(kvm_session *s, kvm_stream stream) {
    if (!s) return KVM_EINVAL;
    DeviceGuard g(s->device);
    const uint32_t L = s->cfg.n_layer;
    KVM_CUDA(s, cudaMemsetAsync(s->q.q_sum, 0, sizeof(float) * L * s->cfg.n_head_q * s->cfg.head_dim,
                                as_stream(stream)),
             "query reset");
    s->h_q_count.assign(L, 0u);
    s->q_dirty = true;
    return KVM_OK;
}

kvm_status kvm_query_add(kvm_session *s, kvm_stream stream, uint32_t layer, uint32_t n, const kvm_rows *q,
                         const uint8_t *keep) {
    if (!s) return KVM_EINVAL;
    if (layer >= s->cfg.n_layer) return fail(s, KVM_EINVAL, "layer out of range");
    if (n == 0) return KVM_OK;
    const uint32_t qdim = s->cfg.n_head_q * s->cfg.head_dim;
    kvm_status r = check_rows(s, q, qdim, "kvm_query_add");
    if (r != KVM_OK) return r;
    DeviceGuard g(s->device);
    cudaStream_t st = as_stream(stream);
    AddRowsArgs a = add_rows_args(q, s->q.q_sum + static_cast<size_t>(layer) * qdim, qdim);
    uint32_t kept = n;
    if (keep) {
        std::vector<uint32_t> list;
        list.reserve(n);
        for (uint32_t i = 0; i < n; ++i)
            if (keep[i]) list.push_back(i);
        kept = static_cast<uint32_t>(list.size());
        if (kept == 0) return KVM_OK;
        if (kept < n) {
            if (kept > s->keep_cap) {
                KVM_CUDA(s, cudaStreamSynchronize(st), "keep list sync");
                if (s->d_keep) cudaFree(s->d_keep);
                s->d_keep = nullptr;
                s->keep_cap = 0;
                const uint32_t cap = std::max(kept, 1024u);
                KVM_CUDA(s, cudaMalloc(&s->d_keep, sizeof(uint32_t) * cap), "keep list allocation");
                s->keep_cap = cap;
            }
            r = upload_small(s, st, s->d_keep, list.data(), sizeof(uint32_t) * kept);
            if (r != KVM_OK) return r;
            a.tok_list = s->d_keep;
        }
    }
    a.tok0 = 0;
    a.n = kept;
    KVM_CUDA(s, launch_add_rows(a, st), "query add");
    s->launches++;
    if (s->h_q_count.size() != s->cfg.n_layer) s->h_q_count.assign(s->cfg.n_layer, 0u);
    s->h_q_count[layer] += kept;
    s->q_dirty = true;
    return KVM_OK;
}

kvm_status kvm_set_query(kvm_session *s, kvm_stream stream, const float *q_sum, const uint32_t *q_count) {
    if (!s) return KVM_EINVAL;
    if (!q_sum || !q_count) return fail(s, KVM_EINVAL, "null query");
    DeviceGuard g(s->device);
    cudaStream_t st = as_stream(stream);
    const uint32_t L = s->cfg.n_layer;
    s->h_q_count.assign(q_count, q_count + L);
    // A query in this device's memory is read by the prep itself, in stream
    // order here: no copy or count upload of its own, and the prep runs as
    // the programmatic dependent launch of the stream's previous kernel.
    cudaPointerAttributes pa{};
    const bool known = cudaPointerGetAttributes(&pa, q_sum) == cudaSuccess;
    if (!known) (void)cudaGetLastError();      // not a CUDA pointer: plain host memory
    const bool on_device = known && (pa.type == cudaMemoryTypeDevice || pa.type == cudaMemoryTypeManaged) &&
                           pa.device == s->device;
    if (on_device && L <= kQueryInlineLayers) {
        QueryLoad ld{};
        ld.src = q_sum;
        for (uint32_t l = 0; l < L; ++l) ld.count[l] = q_count[l];
        KVM_CUDA(s, launch_query_load(s->q, ld, L, s->cfg.n_head_kv, s->cfg.n_head_q, s->cfg.head_dim, st),
                 "query prep launch");
        s->launches++;
        s->q_dirty = false;
        s->prep_load_mark = s->launches;
        s->prep_load_stream = st;
        return KVM_OK;
    }
    KVM_CUDA(s, cudaMemcpyAsync(s->q.q_sum, q_sum, sizeof(float) * L * s->cfg.n_head_q * s->cfg.head_dim,
                                cudaMemcpyDefault, st), "query copy");
    s->q_dirty = true;
    return KVM_OK;
}

static ScoreArgs score_args(kvm_session *s) {
    ScoreArgs a{};
    a.sum = s->sum;
    a.qv = s->q.qv;
    a.nq = s->q.nq;
    a.q_count = s->q.q_count;
    a.n_head_kv = s->cfg.n_head_kv;
    a.n_head_q = s->cfg.n_head_q;
    a.head_dim = s->cfg.head_dim;
    a.n_blocks = s->n_blocks;
    a.terms = s->d_terms;
    a.ldt = s->sum.ldb;
    a.status = s->d_status;
    a.range_done = s->d_range_done;
    a.scores = s->d_scores;
    return a;
}

// The scorer launch, after the query prep when the query changed (the prep
// covers every layer; nothing runs when there are no blocks or layers).
static kvm_status run_score(kvm_session *s, const ScoreArgs &a, bool prep, cudaStream_t st) {
    if (s->n_blocks == 0 || a.n_layers == 0) return KVM_OK;
    // kvm_set_query's prep was this session's last launch, on this stream
    const bool after_load = !prep && s->launches == s->prep_load_mark && st == s->prep_load_stream;
    KVM_CUDA(s, launch_score(a, prep ? &s->q : nullptr, s->cfg.n_layer, st, after_load), "score launch");
    s->launches += prep ? 2u : 1u;
    if (prep) s->q_dirty = false;
    return KVM_OK;
}

kvm_status kvm_score(kvm_session *s, kvm_stream stream, double *d_scores) {
    if (!s) return KVM_EINVAL;
    DeviceGuard g(s->device);
    KVM_FLUSH_SEL(s);
    cudaStream_t st = as_stream(stream);
    bool prep = false;
    kvm_status r = ensure_query(s, st, &prep);
    if (r != KVM_OK) return r;
    ScoreArgs a = score_args(s);
    a.layer0 = 0;
    a.n_layers = s->cfg.n_layer;
    a.combine = 1;
    r = run_score(s, a, prep, st);
    if (r != KVM_OK) return r;
    if (d_scores && s->n_blocks)
        KVM_CUDA(s, cudaMemcpyAsync(d_scores, s->d_scores, sizeof(double) * s->n_blocks,
                                    cudaMemcpyDeviceToDevice, st), "score copy");
    return KVM_OK;
}

kvm_status kvm_score_terms(kvm_session *s, kvm_stream stream, uint32_t layer0, uint32_t n_layers,
                           double *d_terms, uint32_t ldt) {
    if (!s) return KVM_EINVAL;
    if (static_cast<uint64_t>(layer0) + n_layers > s->cfg.n_layer) return fail(s, KVM_EINVAL, "layers out of range");
    if (!d_terms || ldt < s->n_blocks) return fail(s, KVM_EINVAL, "bad terms buffer");
    DeviceGuard g(s->device);
    KVM_FLUSH_SEL(s);
    bool prep = false;
    kvm_status r = ensure_query(s, as_stream(stream), &prep);
    if (r != KVM_OK) return r;
    ScoreArgs a = score_args(s);
    a.layer0 = layer0;
    a.n_layers = n_layers;
    a.terms = d_terms;
    a.ldt = ldt;
    a.combine = 0;
    return run_score(s, a, prep, as_stream(stream));
}

kvm_status kvm_reduce_terms(kvm_session *s, kvm_stream stream, const double *d_terms, uint32_t n_layers,
                            uint32_t ldt, double *d_acc) {
    if (!s) return KVM_EINVAL;
    if (!d_terms || !d_acc || ldt < s->n_blocks) return fail(s, KVM_EINVAL, "bad terms/acc buffer");
    DeviceGuard g(s->device);
    KVM_CUDA(s, launch_reduce_terms(d_terms, n_layers, ldt, s->n_blocks, d_acc, as_stream(stream)),
             "reduce terms");
    s->launches++;
    return KVM_OK;
}

kvm_status kvm_set_scores_from_sum(kvm_session *s, kvm_stream stream, const double *d_acc, uint32_t n_active) {
    if (!s || !d_acc) return KVM_EINVAL;
    DeviceGuard g(s->device);
    KVM_FLUSH_SEL(s);
    KVM_CUDA(s, launch_scores_from_sum(s->sum, s->n_blocks, d_acc, n_active, s->d_scores, as_stream(stream)),
             "scores from sum");
    s->launches++;
    return KVM_OK;
}

kvm_status kvm_set_scores(kvm_session *s, kvm_stream stream, const double *scores, uint32_t n) {
    if (!s) return KVM_EINVAL;
    DeviceGuard g(s->device);
    KVM_FLUSH_SEL(s);
    cudaStream_t st = as_stream(stream);
    // KvMemStore::set_retrieval_scores: entries beyond `n` read as 0
    if (s->n_blocks) KVM_CUDA(s, cudaMemsetAsync(s->d_scores, 0, sizeof(double) * s->n_blocks, st), "clear");
    const uint32_t m = std::min(n, s->n_blocks);
    if (m) {
        if (!scores) return fail(s, KVM_EINVAL, "null scores");
        KVM_CUDA(s, cudaMemcpyAsync(s->d_scores, scores, sizeof(double) * m, cudaMemcpyDefault, st), "scores");
    }
    return KVM_OK;
}

kvm_status kvm_select(kvm_session *s, kvm_stream stream, const uint32_t *mandatory, uint32_t n_mandatory) {
    if (!s) return KVM_EINVAL;
    if (n_mandatory > s->max_blocks) return fail(s, KVM_EINVAL, "too many mandatory blocks");
    if (n_mandatory && !mandatory) return fail(s, KVM_EINVAL, "null mandatory");
    DeviceGuard g(s->device);
    // an earlier select still pending runs now; a pending reset may wait for the diff
    KVM_FLUSH_SEL(s);
    cudaStream_t st = as_stream(stream);
    kvm_status r = upload_small(s, st, s->d_mandatory, mandatory, sizeof(uint32_t) * n_mandatory);
    if (r != KVM_OK) return r;
    // the selection kernel runs with the next kvm_diff (one fused launch) or
    // with whatever entry point comes first
    s->select_pending = true;
    s->select_n_mandatory = n_mandatory;
    s->have_selection = true;
    return KVM_OK;
}

kvm_status kvm_select_groups(kvm_session *s, kvm_stream stream, const uint32_t *spans, const double *scores,
                             uint32_t n_groups, const uint32_t *mandatory, uint32_t n_mandatory) {
    if (!s) return KVM_EINVAL;
    if (n_groups > kMaxGroups) return fail(s, KVM_EINVAL, "at most %u groups", kMaxGroups);
    if (n_groups && (!spans || !scores)) return fail(s, KVM_EINVAL, "null spans or scores");
    if (n_mandatory > s->max_blocks) return fail(s, KVM_EINVAL, "too many mandatory blocks");
    if (n_mandatory && !mandatory) return fail(s, KVM_EINVAL, "null mandatory");
    if (group_select_smem(n_groups, s->n_blocks) > 200u * 1024u)
        return fail(s, KVM_EINVAL, "too many groups for %u blocks", s->n_blocks);
    DeviceGuard g(s->device);
    KVM_FLUSH_SEL(s);
    cudaStream_t st = as_stream(stream);
    kvm_status r = upload_small(s, st, s->d_mandatory, mandatory, sizeof(uint32_t) * n_mandatory);
    if (r != KVM_OK) return r;
    r = upload_small(s, st, s->d_group_spans, spans, sizeof(uint32_t) * 2 * n_groups);
    if (r != KVM_OK) return r;
    if (n_groups) {
        cudaPointerAttributes pa{};
        if (cudaPointerGetAttributes(&pa, scores) != cudaSuccess) {
            (void)cudaGetLastError();
            pa.type = cudaMemoryTypeUnregistered;
        }
        if (pa.type == cudaMemoryTypeDevice || pa.type == cudaMemoryTypeManaged) {
            KVM_CUDA(s, cudaMemcpyAsync(s->d_group_scores, scores, sizeof(double) * n_groups,
                                        cudaMemcpyDeviceToDevice, st), "group scores copy");
        } else {
            r = upload_small(s, st, s->d_group_scores, scores, sizeof(double) * n_groups);
            if (r != KVM_OK) return r;
        }
    }
    GroupSelectArgs a{};
    a.spans = s->d_group_spans;
    a.scores = s->d_group_scores;
    a.n_groups = n_groups;
    a.n_blocks = s->n_blocks;
    a.budget = s->budget_blocks;
    a.sink = s->cfg.sink_blocks;
    a.recent = s->cfg.recent_blocks;
    a.block_tokens = s->cfg.block_tokens;
    a.covered_tokens = s->total_tokens;
    a.mandatory = s->d_mandatory;
    a.n_mandatory = n_mandatory;
    a.selected = s->plan.selected;
    a.hdr = s->plan.hdr;
    KVM_CUDA(s, launch_group_select(a, st), "group select launch");
    s->launches++;
    s->have_selection = true;
    return KVM_OK;
}

kvm_status kvm_set_selection_ids(kvm_session *s, kvm_stream stream, const uint32_t *ids, uint32_t n) {
    if (!s) return KVM_EINVAL;
    if (n > s->max_blocks) return fail(s, KVM_EINVAL, "too many ids");
    if (n && !ids) return fail(s, KVM_EINVAL, "null ids");
    DeviceGuard g(s->device);
    KVM_FLUSH_SEL(s);
    cudaStream_t st = as_stream(stream);
    kvm_status r = upload_small(s, st, s->d_ids, ids, sizeof(uint32_t) * n);
    if (r != KVM_OK) return r;
    KVM_CUDA(s, launch_canon_ids(s->d_ids, n, s->n_blocks, s->plan.selected, s->plan.hdr, st), "canon launch");
    s->launches++;
    s->have_selection = true;
    return KVM_OK;
}

kvm_status kvm_diff(kvm_session *s, kvm_stream stream, int force_raw_refresh) {
    if (!s) return KVM_EINVAL;
    if (!s->have_selection) return fail(s, KVM_ESTATE, "kvm_diff needs a selection (kvm_select)");
    DeviceGuard g(s->device);
    cudaStream_t st = as_stream(stream);
    // a pending select and reset run inside this launch, on this stream
    DiffArgs a{};
    a.bt = s->bt;
    a.n_blocks = s->n_blocks;
    a.n_slots = s->n_slots;
    a.optimize_stage_in = s->cfg.optimize_stage_in;
    a.immutable_source_k = s->cfg.immutable_source_k;
    a.immutable_refresh_remaps = s->cfg.immutable_refresh_remaps;
    a.immutable_refresh_abs_delta_tokens = s->cfg.immutable_refresh_abs_delta_tokens;
    a.immutable_max_baked_position = s->cfg.immutable_max_baked_position;
    a.force_raw_refresh = force_raw_refresh;
    a.plan = s->plan;
    a.status = s->d_status;
    a.reset_window = s->reset_pending ? 1u : 0u;
    s->reset_pending = false;
    if (s->select_pending) {
        s->select_pending = false;
        KVM_CUDA(s, launch_select_diff(select_args(s, s->select_n_mandatory), a, st), "select+diff launch");
    } else {
        KVM_CUDA(s, launch_diff(a, st), "diff launch");
    }
    s->launches++;
    s->have_selection = false;
    s->have_plan = true;
    s->slots_known = false;
    s->plan_moveless = s->window_empty;
    s->window_empty = false;
    return KVM_OK;
}

kvm_status kvm_stagein(kvm_session *s, kvm_stream stream, const kvm_source *src, const kvm_window *win) {
    if (!s) return KVM_EINVAL;
    if (!s->have_plan) return fail(s, KVM_ESTATE, "kvm_stagein needs a plan (kvm_diff)");
    if (!win || !win->d_k || !win->d_v) return fail(s, KVM_EINVAL, "null window");
    kvm_status r = source_check(s, src);
    if (r != KVM_OK) return r;
    DeviceGuard g(s->device);
    KVM_FLUSH(s);
    cudaStream_t st = as_stream(stream);
    r = upload_window(s, st, win);
    if (r != KVM_OK) return r;
    if (s->timed) KVM_CUDA(s, cudaEventRecord(s->ev[2], st), "event");
    r = launch_moves(s, st);
    if (r != KVM_OK) return r;
    if (s->timed) KVM_CUDA(s, cudaEventRecord(s->ev[3], st), "event");
    if (src->location == KVM_LOC_HOST) return stagein_from_host(s, st, src);
    StageinArgs a = stagein_common(s);
    a.n_items_dev = &s->plan.hdr->n_cold;
    a.item0 = 0;
    a.src_by_item = 0;
    a.src_k = static_cast<const uint8_t *>(src->k);
    a.src_v = static_cast<const uint8_t *>(src->v);
    a.layer_stride = src->layer_stride;
    a.item_stride = src->block_stride;
    a.row_stride = src->row_stride;
    a.test_skip = (s->test_inject & KVM_TEST_SKIP_TILE_LOAD) ? 1u : 0u;
    s->test_inject = 0;
    KVM_CUDA(s, launch_stagein(a, st, 0), "stage-in launch");
    s->launches++;
    return KVM_OK;
}

kvm_status kvm_stagein_packed(kvm_session *s, kvm_stream stream, const kvm_packed_source *src,
                              const kvm_window *win) {
    if (!s) return KVM_EINVAL;
    if (!s->have_plan) return fail(s, KVM_ESTATE, "kvm_stagein_packed needs a plan (kvm_diff)");
    if (!win || !win->d_k || !win->d_v) return fail(s, KVM_EINVAL, "null window");
    if (!src || !src->k || !src->v) return fail(s, KVM_EINVAL, "null source");
    if (src->location != KVM_LOC_DEVICE && src->location != KVM_LOC_HOST)
        return fail(s, KVM_EINVAL, "bad source location");
    DeviceGuard g(s->device);
    KVM_FLUSH(s);
    cudaStream_t st = as_stream(stream);
    kvm_status r = upload_window(s, st, win);
    if (r != KVM_OK) return r;
    r = launch_moves(s, st);
    if (r != KVM_OK) return r;
    if (src->location == KVM_LOC_HOST) return packed_from_host(s, st, src);
    PackedInArgs a = packed_common(s);
    a.n_items_dev = &s->plan.hdr->n_cold;
    a.src_k = static_cast<const uint8_t *>(src->k);
    a.src_v = static_cast<const uint8_t *>(src->v);
    a.k_layer_stride = src->k_layer_stride;
    a.k_block_stride = src->k_block_stride;
    a.v_layer_stride = src->v_layer_stride;
    a.v_block_stride = src->v_block_stride;
    const uint64_t m = reinterpret_cast<uintptr_t>(src->k) | reinterpret_cast<uintptr_t>(src->v) |
                       src->k_layer_stride | src->k_block_stride | src->v_layer_stride | src->v_block_stride;
    a.bulk = ((m & 15u) == 0 && s->row_bytes_k % 16u == 0 && s->row_bytes_v % 16u == 0 && window_aligned16(s))
                 ? 1u : 0u;
    KVM_CUDA(s, launch_packed_stagein(a, st), "packed stage-in launch");
    s->launches++;
    return KVM_OK;
}

uint64_t kvm_stageout_item_bytes(const kvm_session *s) {
    return s ? static_cast<uint64_t>(s->cfg.n_layer) * s->cfg.block_tokens * (s->row_bytes_k + s->row_bytes_v)
             : 0u;
}

kvm_status kvm_stageout(kvm_session *s, kvm_stream stream, const uint32_t *ids, uint32_t n,
                        const kvm_window *win, void *dst, uint8_t *resident) {
    if (!s) return KVM_EINVAL;
    if (n == 0) return KVM_OK;
    if (!ids || !dst) return fail(s, KVM_EINVAL, "null block list or destination");
    if (n > s->max_blocks) return fail(s, KVM_EINVAL, "at most max_blocks (%u) blocks per call", s->max_blocks);
    if (!win || !win->d_k || !win->d_v) return fail(s, KVM_EINVAL, "null window");
    DeviceGuard g(s->device);
    KVM_FLUSH(s);
    cudaStream_t st = as_stream(stream);
    kvm_status r = upload_window(s, st, win);
    if (r != KVM_OK) return r;
    r = upload_small(s, st, s->d_out_ids, ids, sizeof(uint32_t) * n);
    if (r != KVM_OK) return r;
    cudaPointerAttributes pa{};
    if (cudaPointerGetAttributes(&pa, dst) != cudaSuccess) {
        (void)cudaGetLastError();
        pa.type = cudaMemoryTypeUnregistered;
    }
    const bool on_device = pa.type == cudaMemoryTypeDevice || pa.type == cudaMemoryTypeManaged;
    const uint64_t item_bytes = kvm_stageout_item_bytes(s);
    StageoutArgs a{};
    a.gpu_slot = s->bt.gpu_slot;
    a.n_tokens = s->bt.n_tokens;
    a.n_blocks = s->n_blocks;
    a.n_slots = s->n_slots;
    a.n_layer = s->cfg.n_layer;
    a.block_tokens = s->cfg.block_tokens;
    a.win_k = s->d_win;
    a.win_v = s->d_win + s->cfg.n_layer;
    a.row_bytes_k = s->row_bytes_k;
    a.row_bytes_v = s->row_bytes_v;
    a.item_bytes = item_bytes;
    a.resident = s->d_out_flags;
    a.status = s->d_status;
    const bool rows16 = s->row_bytes_k % 16u == 0 && s->row_bytes_v % 16u == 0 && window_aligned16(s);
    if (on_device) {
        a.ids = s->d_out_ids;
        a.n = n;
        a.item0 = 0;
        a.dst = static_cast<uint8_t *>(dst);
        a.bulk = rows16 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0 ? 1u : 0u;
        KVM_CUDA(s, launch_stageout(a, st), "stage-out launch");
        s->launches++;
    } else {
        // host destination: pack chunks into the HBM ring on `st`, copy each
        // slot out on the copy stream while the next one is packed
        const uint64_t slot_cap = s->ring_bytes / kvm_session::kRingSlots;
        if (item_bytes > slot_cap)
            return fail(s, KVM_ENOMEM, "staging ring slot (%llu B) smaller than one block (%llu B)",
                        static_cast<unsigned long long>(slot_cap), static_cast<unsigned long long>(item_bytes));
        if (!s->d_ring) {
            KVM_CUDA(s, cudaStreamSynchronize(st), "ring allocation sync");
            KVM_CUDA(s, cudaMalloc(&s->d_ring, s->ring_bytes), "staging ring allocation");
        }
        const uint32_t per_slot = static_cast<uint32_t>(slot_cap / item_bytes);
        a.bulk = rows16 ? 1u : 0u;
        uint8_t *out = static_cast<uint8_t *>(dst);
        int last = 0;
        uint32_t chunk = 0;
        for (uint32_t i0 = 0; i0 < n; i0 += per_slot, ++chunk) {
            const uint32_t m = std::min(per_slot, n - i0);
            const int rs = static_cast<int>(chunk % kvm_session::kRingSlots);
            uint8_t *ring = s->d_ring + static_cast<uint64_t>(rs) * slot_cap;
            // the slot's previous copy-out must be done before it is packed again
            KVM_CUDA(s, cudaStreamWaitEvent(st, s->out_done[rs], 0), "ring slot wait");
            a.ids = s->d_out_ids + i0;
            a.n = m;
            a.item0 = i0;
            a.dst = ring;
            KVM_CUDA(s, launch_stageout(a, st), "stage-out launch");
            s->launches++;
            KVM_CUDA(s, cudaEventRecord(s->out_gathered[rs], st), "stage-out packed");
            KVM_CUDA(s, cudaStreamWaitEvent(s->copy_stream, s->out_gathered[rs], 0), "stage-out packed wait");
            KVM_CUDA(s, cudaMemcpyAsync(out + static_cast<uint64_t>(i0) * item_bytes, ring, m * item_bytes,
                                        cudaMemcpyDeviceToHost, s->copy_stream),
                     "stage-out D2H");
            KVM_CUDA(s, cudaEventRecord(s->out_done[rs], s->copy_stream), "stage-out copied");
            last = rs;
        }
        // work queued on `st` after this call sees the copies done
        KVM_CUDA(s, cudaStreamWaitEvent(st, s->out_done[last], 0), "stage-out join");
    }
    if (resident)
        KVM_CUDA(s, cudaMemcpyAsync(resident, s->d_out_flags, n, cudaMemcpyDeviceToHost, st), "resident flags");
    return KVM_OK;
}

kvm_status kvm_step(kvm_session *s, kvm_stream stream, const uint32_t *mandatory, uint32_t n_mandatory,
                    const kvm_source *src, const kvm_window *win) {
    if (!s) return KVM_EINVAL;
    DeviceGuard g(s->device);
    cudaStream_t st = as_stream(stream);
    s->timed = true;
    KVM_CUDA(s, cudaEventRecord(s->ev[0], st), "event");
    kvm_status r = kvm_score(s, stream, nullptr);
    if (r == KVM_OK) {
        KVM_CUDA(s, cudaEventRecord(s->ev[1], st), "event");
        r = kvm_select(s, stream, mandatory, n_mandatory);
    }
    if (r == KVM_OK) r = kvm_diff(s, stream, 0);
    if (r == KVM_OK) r = kvm_stagein(s, stream, src, win);
    if (r == KVM_OK) KVM_CUDA(s, cudaEventRecord(s->ev[4], st), "event");
    s->timed = false;
    return r;
}

kvm_status kvm_test_inject(kvm_session *s, uint32_t flags) {
    if (!s) return KVM_EINVAL;
    if (flags & ~KVM_TEST_SKIP_TILE_LOAD) return fail(s, KVM_EINVAL, "unknown test flags 0x%x", flags);
    s->test_inject = flags;
    return KVM_OK;
}

kvm_status kvm_wait(kvm_session *s, kvm_stream stream, uint32_t timeout_ms) {
    if (!s) return KVM_EINVAL;
    DeviceGuard g(s->device);
    KVM_FLUSH(s);
    cudaEvent_t ev;
    KVM_CUDA(s, cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "event");
    cudaError_t e = cudaEventRecord(ev, as_stream(stream));
    kvm_status r = e == cudaSuccess ? wait_event(s, ev, timeout_ms) : cuda_fail(s, e, "event record");
    cudaEventDestroy(ev);
    if (r != KVM_OK) return r;
    return check_status(s);
}

kvm_status kvm_get_plan(kvm_session *s, kvm_stream stream, kvm_plan *p, uint32_t timeout_ms) {
    if (!s || !p) return KVM_EINVAL;
    kvm_status r = kvm_wait(s, stream, timeout_ms);
    if (r != KVM_OK) return r;
    DeviceGuard g(s->device);
    PlanHeader h{};
    KVM_CUDA(s, cudaMemcpy(&h, s->plan.hdr, sizeof h, cudaMemcpyDeviceToHost), "plan header");
    const uint32_t cap = p->capacity;
    auto get = [&](void *dst, const void *src, uint32_t n, size_t esz) -> kvm_status {
        if (!dst || n == 0) return KVM_OK;
        if (n > cap) return fail(s, KVM_EINVAL, "plan capacity %u < %u", cap, n);
        KVM_CUDA(s, cudaMemcpy(dst, src, n * esz, cudaMemcpyDeviceToHost), "plan read");
        return KVM_OK;
    };
    p->n_selected = h.n_selected;
    p->n_stage_in = h.n_stage_in;
    p->n_stage_out = h.n_stage_out;
    p->n_remaps = h.n_remaps;
    p->total_window_tokens = h.total_window_tokens;
    p->selection_overlap_blocks = h.selection_overlap_blocks;
    p->gpu_reused_blocks = h.gpu_reused_blocks;
    p->retained_position_stable = h.retained_position_stable;
    p->retained_position_moved = h.retained_position_moved;
    p->n_moves = h.n_moves;
    p->n_cold = h.n_cold;
    std::vector<uint32_t> sel(h.n_selected);
    if (h.n_selected)
        KVM_CUDA(s, cudaMemcpy(sel.data(), s->plan.selected, 4u * h.n_selected, cudaMemcpyDeviceToHost), "sel");
    if (p->selected && h.n_selected) {
        if (h.n_selected > cap) return fail(s, KVM_EINVAL, "plan capacity %u < %u", cap, h.n_selected);
        std::memcpy(p->selected, sel.data(), 4u * h.n_selected);
    }
    if ((r = get(p->stage_in, s->plan.stage_in, h.n_stage_in, 4)) != KVM_OK) return r;
    if ((r = get(p->stage_out, s->plan.stage_out, h.n_stage_out, 4)) != KVM_OK) return r;
    if ((r = get(p->rm_block_id, s->plan.rm_block_id, h.n_remaps, 4)) != KVM_OK) return r;
    if ((r = get(p->rm_n_tokens, s->plan.rm_n_tokens, h.n_remaps, 4)) != KVM_OK) return r;
    if ((r = get(p->rm_from_base, s->plan.rm_from_base, h.n_remaps, 4)) != KVM_OK) return r;
    if ((r = get(p->rm_to_base, s->plan.rm_to_base, h.n_remaps, 4)) != KVM_OK) return r;
    if ((r = get(p->rm_working_k_resident, s->plan.rm_wkr, h.n_remaps, 1)) != KVM_OK) return r;
    if ((r = get(p->rm_skip, s->plan.rm_skip, h.n_remaps, 1)) != KVM_OK) return r;
    if ((r = get(p->rm_raw_refresh, s->plan.rm_raw, h.n_remaps, 1)) != KVM_OK) return r;
    if ((r = get(p->mv_block, s->plan.mv_block, h.n_moves, 4)) != KVM_OK) return r;
    if ((r = get(p->mv_from, s->plan.mv_from, h.n_moves, 4)) != KVM_OK) return r;
    if ((r = get(p->mv_to, s->plan.mv_to, h.n_moves, 4)) != KVM_OK) return r;
    if ((r = get(p->cold_block, s->plan.cold_block, h.n_cold, 4)) != KVM_OK) return r;
    if ((r = get(p->cold_to, s->plan.cold_to, h.n_cold, 4)) != KVM_OK) return r;
    // host view of the window after this plan: slot i = i-th selected block
    // (only when the selection read back is the one the last diff laid out)
    if (s->have_plan && !s->have_selection && h.n_blocks == s->n_blocks) {
        std::fill(s->h_slot.begin(), s->h_slot.end(), -1);
        for (uint32_t i = 0; i < h.n_selected; ++i)
            if (sel[i] < s->h_slot.size()) s->h_slot[sel[i]] = static_cast<int32_t>(i);
        s->slots_known = true;
    }
    return KVM_OK;
}

kvm_status kvm_get_scores(kvm_session *s, kvm_stream stream, double *scores, uint32_t n, uint32_t timeout_ms) {
    if (!s || (!scores && n)) return KVM_EINVAL;
    kvm_status r = kvm_wait(s, stream, timeout_ms);
    if (r != KVM_OK) return r;
    DeviceGuard g(s->device);
    const uint32_t m = std::min(n, s->n_blocks);
    if (m) KVM_CUDA(s, cudaMemcpy(scores, s->d_scores, sizeof(double) * m, cudaMemcpyDeviceToHost), "scores read");
    return KVM_OK;
}

kvm_status kvm_get_timings(kvm_session *s, kvm_timings *t) {
    if (!s || !t) return KVM_EINVAL;
    DeviceGuard g(s->device);
    if (cudaEventQuery(s->ev[4]) != cudaSuccess) return fail(s, KVM_ESTATE, "no completed step");
    KVM_CUDA(s, cudaEventElapsedTime(&t->score_ms, s->ev[0], s->ev[1]), "timing");
    KVM_CUDA(s, cudaEventElapsedTime(&t->plan_ms, s->ev[1], s->ev[2]), "timing");
    KVM_CUDA(s, cudaEventElapsedTime(&t->layout_ms, s->ev[2], s->ev[3]), "timing");
    KVM_CUDA(s, cudaEventElapsedTime(&t->set_ms, s->ev[3], s->ev[4]), "timing");
    KVM_CUDA(s, cudaEventElapsedTime(&t->total_ms, s->ev[0], s->ev[4]), "timing");
    return KVM_OK;
}

kvm_status kvm_quantize_rows(kvm_stream stream, int32_t type, const void *d_src, uint64_t n_rows,
                             uint32_t n_embd, void *d_dst) {
    if (!type_ok(type) || n_embd == 0 || n_embd % 32u != 0 || n_embd > 16384u) return KVM_EINVAL;
    if (n_rows == 0) return KVM_OK;
    if (!d_src || !d_dst || (reinterpret_cast<uintptr_t>(d_src) & 15u)) return KVM_EINVAL;
    if (reinterpret_cast<uintptr_t>(d_dst) & 1u) {
        set_sessionless_error("kvm_quantize_rows: d_dst must be 2-byte aligned");
        return KVM_EINVAL;
    }
    // rows as one pseudo-block per tile run: item i = rows [i*R, (i+1)*R)
    const uint32_t rb = static_cast<uint32_t>(kvm_row_bytes(type, n_embd));
    const uint32_t R = stagein_rows_per_tile(n_embd, 128u);
    const uint64_t n_items64 = (n_rows + R - 1) / R;
    if (n_items64 > (1ull << 24)) return KVM_EINVAL;
    const uint32_t n_items = static_cast<uint32_t>(n_items64);
    // device work list: identity block ids / slots, per-item row counts
    uint32_t *d_list = nullptr;
    uint8_t **d_dst_arr = nullptr;
    const size_t list_bytes = (3ull * n_items * sizeof(uint32_t) + 255u) & ~static_cast<size_t>(255u);
    if (cudaMalloc(&d_list, list_bytes + 512) != cudaSuccess) return KVM_ENOMEM;
    d_dst_arr = reinterpret_cast<uint8_t **>(reinterpret_cast<uint8_t *>(d_list) + list_bytes);
    uint32_t *d_stat = reinterpret_cast<uint32_t *>(reinterpret_cast<uint8_t *>(d_list) + list_bytes + 256);
    std::vector<uint32_t> h(3ull * n_items);
    for (uint32_t i = 0; i < n_items; ++i) {
        h[i] = i;
        h[n_items + i] = i;
        const uint64_t left = n_rows - static_cast<uint64_t>(i) * R;
        h[2ull * n_items + i] = static_cast<uint32_t>(left < R ? left : R);
    }
    cudaStream_t st = as_stream(stream);
    uint8_t *dst_ptrs[2] = {static_cast<uint8_t *>(d_dst), static_cast<uint8_t *>(d_dst)};
    cudaError_t e = cudaMemcpyAsync(d_list, h.data(), h.size() * sizeof(uint32_t),
                                    cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_dst_arr, dst_ptrs, sizeof dst_ptrs, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(d_stat, 0, sizeof(uint32_t), st);
    StageinArgs a{};
    a.cold_block = d_list;
    a.cold_to = reinterpret_cast<const int32_t *>(d_list + n_items);
    a.n_items_dev = nullptr;
    a.n_items_host = n_items;
    a.item0 = 0;
    a.max_items = n_items;
    a.src_by_item = 1;
    a.n_kv = 1;
    a.src_k = static_cast<const uint8_t *>(d_src);
    a.src_v = static_cast<const uint8_t *>(d_src);
    a.layer_stride = 0;
    a.item_stride = static_cast<uint64_t>(R) * n_embd * 2u;
    a.row_stride = 2ull * n_embd;
    a.n_tokens = d_list + 2ull * n_items;
    a.max_blocks = n_items;
    a.dst_k = d_dst_arr;
    a.dst_v = d_dst_arr;
    a.n_layer = 1;
    a.block_tokens = R;
    a.n_embd = n_embd;
    a.n_slots = n_items;
    a.type_k = type;
    a.type_v = type;
    a.row_bytes_k = rb;
    a.row_bytes_v = rb;
    a.rows_per_tile = R;
    a.tile_in_bytes = R * n_embd * 2u;
    a.tile_out_bytes = (R * rb + 15u) & ~15u;
    a.bulk_store = (rb % 16u == 0 && (reinterpret_cast<uintptr_t>(d_dst) & 15u) == 0) ? 1u : 0u;
    a.status = d_stat;
    if (e == cudaSuccess) e = launch_stagein(a, st, 0);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    uint32_t stat = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&stat, d_stat, sizeof stat, cudaMemcpyDeviceToHost);
    cudaFree(d_list);
    if (e != cudaSuccess) {
        set_sessionless_error(cudaGetErrorString(e));
        return e == cudaErrorMemoryAllocation ? KVM_ENOMEM : KVM_ECUDA;
    }
    if (stat) {
        set_sessionless_error(stat & kErrTimeout ? "kvm_quantize_rows: a bounded device wait timed out"
                                                 : "kvm_quantize_rows: device error flag");
        return KVM_EDEVICE;
    }
    return KVM_OK;
}

}  // extern "C"
