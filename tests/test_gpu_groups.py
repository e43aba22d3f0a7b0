"""kvm_select_groups (pick_semantic_groups on the device) against the oracle
restatement -- itself pinned to the reference's compiled KvMemStore -- through
the C ABI: the reference's inline test cases, the golden sequence of seeded
cases, device-resident scores, and the diff that follows."""
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _session(kvm, T, budget, sink, recent, max_blocks):
    cfg = kvm.default_config(block_tokens=T, select_budget=budget * T, gen_reserve=T, sink_blocks=sink,
                             recent_blocks=recent, n_layer=1, n_head_kv=1, head_dim=32, n_head_q=1,
                             max_blocks=max_blocks, type_k=8, type_v=8)
    return kvm.Session(cfg, 0)


def _gpu_select(kvm, cfg, total, spans, scores, mand, device_scores=False):
    import torch
    T = cfg["block_tokens"]
    n = (total + T - 1) // T
    s = _session(kvm, T, cfg["budget_blocks"], cfg["sink_blocks"], cfg["recent_blocks"], n + 4)
    try:
        s.register_append(total)
        sc = torch.from_numpy(np.asarray(scores, np.float64)).cuda() if device_scores else scores
        s.select_groups(spans, sc, mand)
        s.diff()
        return s.plan()["selected"]
    finally:
        s.close()


def test_reference_inline_cases(kvm_lib):
    c = dict(block_tokens=32, budget_blocks=8, sink_blocks=1, recent_blocks=1)
    sel = _gpu_select(kvm_lib, c, 32 * 20, [(32, 128), (131, 251), (256, 352), (384, 448)],
                      [1.0, 10.0, 9.0, 2.0], [])
    assert {0, 19, 4, 5, 6, 7} <= set(sel.tolist()) and not ({8, 9, 10} & set(sel.tolist()))
    c = dict(block_tokens=64, budget_blocks=4, sink_blocks=0, recent_blocks=0)
    assert _gpu_select(kvm_lib, c, 64 * 8, [(64, 138), (138, 256)], [2.0, 1.0], [7]).tolist() == [1, 2, 3, 7]
    c = dict(block_tokens=32, budget_blocks=4, sink_blocks=1, recent_blocks=2)
    assert _gpu_select(kvm_lib, c, 320, [(160, 224)], [1.0], [1, 2, 3, 4]).tolist() == [0, 2, 3, 4]


def test_golden_cases_and_device_scores(kvm_lib, oracle):
    g = json.load(open(os.path.join(GOLD, "groups_golden.json")))
    for i, c in enumerate(g["cases"]):
        if c["cfg"]["budget_blocks"] == 0:
            # the raw store selects everything at budget 0; a session's budget
            # is aligned to at least one block like the adapter's
            # kvmem_align_tokens (llama-memory-kvmem.cpp:254-262)
            continue
        scores = np.array([-0.0 if (x == 0.0 and sb) else x for x, sb in zip(c["scores"], c["signbits"])],
                          np.float64)
        spans = np.array(c["spans"], np.uint32).reshape(-1, 2)
        got = _gpu_select(kvm_lib, c["cfg"], c["total_tokens"], spans, scores, c["mandatory"],
                          device_scores=(i % 2 == 1))
        assert got.tolist() == c["selected"], i


def test_many_groups_random(kvm_lib, oracle):
    """Thousands of groups over 4096 blocks: the bitonic sort at full width."""
    rng = np.random.default_rng(5)
    T, n = 128, 4096
    for G, ties in ((8192, False), (3000, True), (1, False)):
        b0 = rng.integers(0, n * T, G)
        spans = np.stack([b0, b0 + rng.integers(1, 8 * T, G)], 1).astype(np.uint32)
        scores = rng.integers(0, 5, G).astype(np.float64) if ties else rng.standard_normal(G)
        mand = rng.integers(0, n, 6)
        c = dict(block_tokens=T, budget_blocks=300, sink_blocks=1, recent_blocks=2)
        got = _gpu_select(kvm_lib, c, n * T, spans, scores, mand)
        want = oracle.pick_semantic_groups(oracle.make_cfg(T, 300, 1, 2), n, n * T, spans, scores, mand)
        assert np.array_equal(got, want), G


def test_group_argument_checks(kvm_lib):
    s = _session(kvm_lib, 32, 4, 1, 0, 16)
    try:
        s.register_append(320)
        with pytest.raises(kvm_lib.KvmError):
            s.select_groups(np.zeros((8193, 2), np.uint32), np.zeros(8193))
        s.select_groups(np.zeros((0, 2), np.uint32), np.zeros(0))     # pins only
        s.diff()
        assert s.plan()["selected"].tolist() == [0]
    finally:
        s.close()
