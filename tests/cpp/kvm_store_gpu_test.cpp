// The reference's KvMemStore expectations (kvmem/tests/kvmem_store_test.cpp)
// run against kvm::KvMemStore, the C++ mirror whose selector and diff execute
// on the GPU.  Plain main() + CHECK like the reference's tests; exit code 0
// when every check passes.
#include "kvm_store.hpp"

#include <algorithm>
#include <cstdio>
#include <vector>

static int g_fail = 0;
#define CHECK(cond)                                                            \
    do {                                                                       \
        if (!(cond)) {                                                         \
            std::printf("FAIL %s:%d  %s\n", __FILE__, __LINE__, #cond);        \
            ++g_fail;                                                          \
        }                                                                      \
    } while (0)

using kvm::KvMemStore;
using kvm::KvMemStoreConfig;
using kvm::KvTier;

static bool has(const std::vector<uint32_t> &v, uint32_t id) {
    return std::find(v.begin(), v.end(), id) != v.end();
}

static KvMemStoreConfig base(uint32_t bt, uint32_t budget_blocks, uint32_t sink, uint32_t recent) {
    KvMemStoreConfig c;
    c.block_tokens = bt;
    c.select_budget = bt * budget_blocks;
    c.gen_budget = bt * 4;
    c.sink_blocks = sink;
    c.recent_blocks = recent;
    c.n_layer = 1;
    c.n_head_kv = 1;
    c.head_dim = 32;
    c.n_head_q = 1;
    c.max_blocks = 256;
    return c;
}

// kvmem_store_test.cpp:53-110
static void test_selection_diff_and_remap() {
    KvMemStore s(base(128, 1024, 1, 0));
    s.register_append(128 * 5);
    CHECK(s.block_count() == 5);
    auto plan = s.set_selection({4, 0, 2});
    CHECK(plan.stage_in.size() == 3);
    CHECK(plan.stage_out.size() == 2);
    CHECK(plan.stage_out[0] == 1 && plan.stage_out[1] == 3);
    CHECK(plan.remaps.size() == 3);
    CHECK(plan.total_window_tokens == 128 * 3);
    CHECK(plan.remaps[0].block_id == 0 && plan.remaps[0].from_base == 0 &&
          plan.remaps[0].to_base == 0 && plan.remaps[0].skip);
    CHECK(plan.remaps[1].block_id == 2 && plan.remaps[1].from_base == 256 &&
          plan.remaps[1].to_base == 128 && !plan.remaps[1].skip);
    CHECK(plan.remaps[2].block_id == 4 && plan.remaps[2].from_base == 512 &&
          plan.remaps[2].to_base == 256);
    for (uint32_t id : plan.stage_out) s.set_block_tier(id, KvTier::CPU, static_cast<int32_t>(id), -1);
    auto plan2 = s.set_selection({0, 2, 3});
    CHECK(plan2.stage_in.size() == 1 && plan2.stage_in[0] == 3);
    CHECK(plan2.stage_out.size() == 1 && plan2.stage_out[0] == 4);
    CHECK(plan2.remaps.size() == 3);
    CHECK(plan2.remaps[0].skip && plan2.remaps[1].skip && !plan2.remaps[2].skip);
    CHECK(plan2.remaps[2].from_base == 128 * 3 && plan2.remaps[2].to_base == 128 * 2);
    CHECK(plan2.total_window_tokens == 128 * 3);
    // chronological layout: slot i holds the i-th selected block
    CHECK(plan2.selected == std::vector<uint32_t>({0, 2, 3}));
}

// kvmem_store_test.cpp:284-314
static void test_topk_budget_sink_recent() {
    KvMemStore s(base(128, 4, 1, 1));
    s.register_append(128 * 10);
    CHECK(s.budget_blocks() == 4);
    std::vector<double> scores(10, 0.0);
    scores[5] = 100.0;
    scores[6] = 90.0;
    scores[3] = 10.0;
    s.set_retrieval_scores(scores);
    auto sel = s.pick_topk_blocks();
    CHECK(sel.size() == 4);
    CHECK(has(sel, 0) && has(sel, 9) && has(sel, 5) && has(sel, 6));
    for (size_t i = 1; i < sel.size(); ++i) CHECK(sel[i] > sel[i - 1]);
}

// kvmem_store_test.cpp:316-339
static void test_topk_zero_recent_keeps_no_suffix() {
    KvMemStore s(base(128, 4, 1, 0));
    s.register_append(128 * 10);
    std::vector<double> scores(10, 0.0);
    scores[3] = 80.0;
    scores[5] = 100.0;
    scores[6] = 90.0;
    scores[9] = -100.0;
    s.set_retrieval_scores(scores);
    const auto sel = s.pick_topk_blocks();
    CHECK(sel.size() == 4);
    CHECK(has(sel, 0) && has(sel, 3) && has(sel, 5) && has(sel, 6) && !has(sel, 9));
}

// kvmem_store_test.cpp:433-458
static void test_topk_mandatory_blocks_stay_inside_budget() {
    KvMemStore s(base(32, 4, 1, 0));
    s.register_append(32 * 10);
    std::vector<double> scores(10, 0.0);
    scores[2] = 100.0;
    scores[3] = 90.0;
    scores[4] = 80.0;
    scores[8] = -10.0;
    scores[9] = -20.0;
    s.set_retrieval_scores(scores);
    const auto sel = s.pick_topk_blocks({8, 9});
    CHECK(sel.size() == 4);
    CHECK(has(sel, 0) && has(sel, 2) && has(sel, 8) && has(sel, 9) && !has(sel, 3));
}

// kvmem_store_test.cpp:460-477
static void test_mandatory_overlap_deduplicates_and_recent_is_best_effort() {
    KvMemStore s(base(32, 4, 2, 3));
    s.register_append(32 * 10);
    s.set_retrieval_scores(std::vector<double>(10, 0.0));
    const auto sel = s.pick_topk_blocks({0, 0, 5});
    CHECK(sel.size() == 4);
    for (uint32_t id : {0u, 1u, 5u, 9u}) CHECK(has(sel, id));
    CHECK(!has(sel, 8));
}

// kvmem_store_test.cpp:479-504
static void test_mandatory_hard_union_overflow_trims_newest() {
    KvMemStore s(base(32, 4, 1, 2));
    s.register_append(32 * 10);
    s.set_retrieval_scores(std::vector<double>(10, 0.0));
    const auto sel = s.pick_topk_blocks({1, 2, 3, 4});
    CHECK(sel.size() == 4);
    for (uint32_t id : {0u, 2u, 3u, 4u}) CHECK(has(sel, id));
    CHECK(!has(sel, 1));
}

// kvmem_store_test.cpp:763-781
static void test_topk_all_fit_and_empty() {
    KvMemStore s(base(128, 100, 1, 0));
    s.register_append(128 * 3);
    s.set_retrieval_scores({0.0, 0.0, 0.0});
    auto sel = s.pick_topk_blocks();
    CHECK(sel.size() == 3 && sel[0] == 0 && sel[1] == 1 && sel[2] == 2);
    KvMemStore e(base(128, 100, 1, 0));
    CHECK(e.pick_topk_blocks().empty());
    auto plan = e.set_selection({0, 1});
    CHECK(plan.remaps.empty());
    CHECK(plan.total_window_tokens == 0);
}

// kvmem_store_test.cpp:1017-1053
static void test_round_groups_are_selected_whole() {
    KvMemStore s(base(32, 8, 1, 1));
    s.register_append(32 * 20);
    const std::vector<std::pair<uint32_t, uint32_t>> groups{
        {32, 32 * 4}, {32 * 4 + 3, 32 * 8 - 5}, {32 * 8, 32 * 11}, {32 * 12, 32 * 14}};
    const auto selected = s.pick_semantic_groups(groups, {1.0, 10.0, 9.0, 2.0});
    CHECK(selected.size() <= 8);
    CHECK(has(selected, 0) && has(selected, 19));
    for (uint32_t id = 4; id <= 7; ++id) CHECK(has(selected, id));
    for (uint32_t id = 8; id <= 10; ++id) CHECK(!has(selected, id));
}

// kvmem_store_test.cpp:1055-1076
static void test_round_groups_charge_shared_boundary_once() {
    KvMemStore s(base(64, 4, 0, 0));
    s.register_append(64 * 8);
    const std::vector<std::pair<uint32_t, uint32_t>> groups{{64, 64 * 2 + 10}, {64 * 2 + 10, 64 * 4}};
    const auto selected = s.pick_semantic_groups(groups, {2.0, 1.0}, {7});
    CHECK(selected.size() == 4);
    for (uint32_t id : {1u, 2u, 3u, 7u}) CHECK(has(selected, id));
}

// kvmem_store_test.cpp:479-503 (the semantic half)
static void test_semantic_mandatory_overflow_trims_newest() {
    KvMemStore s(base(32, 4, 1, 2));
    s.register_append(32 * 10);
    const auto sem = s.pick_semantic_groups({{32 * 5, 32 * 7}}, {1.0}, {1, 2, 3, 4});
    CHECK(sem.size() == 4);
    for (uint32_t id : {0u, 2u, 3u, 4u}) CHECK(has(sem, id));
    CHECK(!has(sem, 1));
    bool threw = false;
    try {
        s.pick_semantic_groups({{0, 32}}, {});
    } catch (const std::runtime_error &) {
        threw = true;
    }
    CHECK(threw);
}

// A shape the device path cannot serve is rejected with std::invalid_argument,
// the exception type the reference uses for bad configurations.
static void test_invalid_config_throws() {
    bool threw = false;
    try {
        KvMemStoreConfig c = base(32, 4, 1, 0);
        c.head_dim = 10;                   // n_head_kv * head_dim not a ggml block multiple
        KvMemStore s(c);
    } catch (const std::invalid_argument &) {
        threw = true;
    }
    CHECK(threw);
}

int main() {
    test_selection_diff_and_remap();
    test_topk_budget_sink_recent();
    test_topk_zero_recent_keeps_no_suffix();
    test_topk_mandatory_blocks_stay_inside_budget();
    test_mandatory_overlap_deduplicates_and_recent_is_best_effort();
    test_mandatory_hard_union_overflow_trims_newest();
    test_topk_all_fit_and_empty();
    test_round_groups_are_selected_whole();
    test_round_groups_charge_shared_boundary_once();
    test_semantic_mandatory_overflow_trims_newest();
    test_invalid_config_throws();
    if (g_fail) {
        std::printf("%d check(s) failed\n", g_fail);
        return 1;
    }
    std::printf("kvm_store_gpu_test: all checks passed\n");
    return 0;
}
