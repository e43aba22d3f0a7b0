"""Pin the CPU oracle (oracle/kvm_oracle.c) before trusting it as the checker.

  * quantizers vs gguf-py 0.19.0 golden bytes (tests/golden/quant_golden.npz)
  * selection + KvMemPlan vs sequences recorded from the reference's own
    kvmem::KvMemStore (tests/golden/store_golden.json), and live against the
    compiled reference when oracle/_ref is present
  * mean-K vs the reference's own RawKvStore (memcmp-exact)
  * the reference's inline store expectations (kvmem/tests/kvmem_store_test.cpp)
  * the scorer vs the reference adapter's own score_retrieval, compiled from
    its file by oracle/Makefile (live when oracle/_ref is present, and through
    tests/golden/score_golden.npz everywhere), and vs an independent numpy
    restatement (float32 sequential sums)
"""
import json
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")


# ----------------------------------------------------------------- F16 ---

def test_f16_conversions_exhaustive(oracle):
    L = oracle.lib()
    h = np.arange(0, 65536, dtype=np.uint16)
    ref = h.view(np.float16).astype(np.float32)
    got = np.array([L.ora_f16_to_f32(int(v)) for v in h], dtype=np.float32)
    ok = ~np.isnan(ref)
    assert np.array_equal(got[ok].view(np.uint32), ref[ok].view(np.uint32))
    assert np.all(np.isnan(got[~ok]))
    rng = np.random.default_rng(3)
    vals = (rng.standard_normal(20000) * 10.0 ** rng.integers(-9, 5, 20000)).astype(np.float32)
    vals = np.concatenate([vals, np.float32([65504, 65519.99, 65520, -65520, 2**-24, 2**-25,
                                              3 * 2**-26, 0.0, -0.0, np.inf, -np.inf])])
    got16 = np.array([L.ora_f32_to_f16(float(v)) for v in vals], dtype=np.uint16)
    with np.errstate(over="ignore"):
        assert np.array_equal(got16, vals.astype(np.float16).view(np.uint16))


# ---------------------------------------------------------- quantizers ---

def _neg_zero_first_blocks(rows, bs):
    """Blocks whose first max-|x| element is -0.0 (all-zero blocks starting with -0)."""
    blk = rows.astype(np.float32).reshape(-1, 32)
    return np.all(blk == 0, axis=1) & np.signbit(blk[:, 0])


@pytest.mark.parametrize("name,type_id,bs", [("q8_0", 8, 34), ("q4_0", 2, 18), ("q5_0", 6, 22)])
def test_quantizers_match_gguf_golden(oracle, name, type_id, bs):
    g = np.load(os.path.join(GOLD, "quant_golden.npz"))
    rows = g["rows_f16"].view(np.float16)
    got = oracle.quantize_rows_f16(type_id, rows).reshape(-1, bs)
    want = g[name].reshape(-1, bs)
    assert got.shape == want.shape
    differ = np.any(got != want, axis=1)
    # gguf-py takes the signed zero of the argmax element; the reference
    # (stagein.cu:207-214, ggml ref) keeps vmax = +0.0f, giving d = -0.0.
    # No golden row has such a block for q8_0 (d = +0/127 either way).
    assert not np.any(differ & ~_neg_zero_first_blocks(rows, bs))


def test_quantizer_edge_cases(oracle):
    # all-zero blocks: q8_0 d = +0, q4_0/q5_0 d = 0/-8 = -0.0 (0x8000), mid codes
    z = np.zeros(32, np.float32)
    q8 = oracle.quantize(oracle.TYPE_Q8_0, z)
    assert q8[:2].tolist() == [0, 0] and not q8[2:].any()
    q4 = oracle.quantize(oracle.TYPE_Q4_0, z)
    assert q4[:2].tolist() == [0x00, 0x80] and np.all(q4[2:] == 0x88)
    q5 = oracle.quantize(oracle.TYPE_Q5_0, z)
    assert q5[:2].tolist() == [0x00, 0x80]
    assert q5[2:6].tolist() == [0xff] * 4 and np.all(q5[6:] == 0)   # 16 -> high bit set
    # q8_0 round-half-away-from-zero: amax 127 -> id 1 -> x = 0.5 rounds to 1, -0.5 to -1
    x = np.zeros(32, np.float32)
    x[0], x[1], x[2], x[3] = 127.0, 0.5, -0.5, 2.5
    q = oracle.quantize(oracle.TYPE_Q8_0, x).view(np.int8)
    assert q[2 + 0] == 127 and q[2 + 1] == 1 and q[2 + 2] == -1 and q[2 + 3] == 3
    # q4_0 first-max tie: |3| at index 0 (+3) and 1 (-3): vmax = +3 -> d = -0.375
    x = np.zeros(32, np.float32)
    x[0], x[1] = 3.0, -3.0
    q4 = oracle.quantize(oracle.TYPE_Q4_0, x)
    assert q4[:2].view(np.float16)[0] == np.float16(-0.375)


# ---------------------------------------------------------------- mean-K ---

def test_mean_k_matches_reference_rawkvstore(oracle):
    g = np.load(os.path.join(GOLD, "meank_golden.npz"))
    bt = int(g["block_tokens"])
    for il, key in enumerate(("k0", "k1")):
        k = g[key]
        nb = (k.shape[0] + bt - 1) // bt
        for b in range(nb):
            rows = k[b * bt:(b + 1) * bt]
            s = np.zeros(k.shape[1], np.float32)
            for r in rows:
                s = (s + r).astype(np.float32)       # ordered F32 sum
            got = oracle.mean_k(s, rows.shape[0])
            assert got.tobytes() == g["means"][il, b].tobytes()


def test_block_sum_f16_ordered(oracle):
    rng = np.random.default_rng(5)
    k = oracle.synth_f16(rng, (128, 64), 64)
    got = oracle.block_sum_f16(k)
    want = np.zeros(64, np.float32)
    for r in k.astype(np.float32):
        want = (want + r).astype(np.float32)
    assert got.tobytes() == want.tobytes()


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(HERE), "oracle", "_ref",
                                                    "libkvmem_ref.so")),
                    reason="reference library not built here")
def test_mean_k_live_vs_reference(oracle):
    rng = np.random.default_rng(11)
    E, bt = 128, 32
    k = rng.standard_normal((3 * bt + 5, E)).astype(np.float32) * 100
    raw = oracle.RefRaw(1, E, bt)
    pos = 0
    while pos < k.shape[0]:          # uneven write batches across block edges
        n = min(11, k.shape[0] - pos)
        raw.write_layer_mean_k(pos, k[pos:pos + n], 0)
        pos += n
    for b in range(4):
        rows = k[b * bt:(b + 1) * bt]
        s = np.zeros(E, np.float32)
        for r in rows:
            s = (s + r).astype(np.float32)
        assert oracle.mean_k(s, rows.shape[0]).tobytes() == raw.mean_k(b, 0).tobytes()
    assert not raw.has_block(9)


def test_mean_store_sequence_matches_reference_golden(oracle):
    from kvm_testlib import load_meank_seq
    ops, g = load_meank_seq()
    L, E, bt = int(g["n_layer"]), int(g["n_embd"]), int(g["block_tokens"])
    nb = g["means"].shape[1]
    ms = oracle.MeanStore(L, nb, E, bt)
    for op in ops:
        if op[0] == "k":
            ms.write_layer_mean_k(op[2], op[3], op[1])
        else:
            ms.write_layer_mean_sum(op[2], op[3], op[1], op[4])
    for il in range(L):
        for b in range(nb):
            assert ms.mean_k(b, il).tobytes() == g["means"][il, b].tobytes(), (il, b)
    # the sequence covers mid-block flushes, block-start flushes and partial blocks
    kinds = {(op[0], op[2] % bt == 0) for op in ops}
    assert ("s", False) in kinds and ("s", True) in kinds and ("k", False) in kinds


def test_add_rows_is_the_ordered_f32_sum(oracle):
    rows = np.array([[1e8], [1.0], [-1e8], [1.0]], np.float32)
    # (((0 + 1e8) + 1) - 1e8) + 1 = 1 in F32 order; a pairwise sum would give 2
    assert oracle.add_rows(np.zeros(1, np.float32), rows)[0] == np.float32(1.0)
    assert oracle.add_rows(np.array([-0.0], np.float32), np.array([[-0.0]], np.float32))[0] == 0.0


# ------------------------------------------------------- semantic groups ---

def _group_case_scores(c):
    return np.array([-0.0 if (x == 0.0 and sb) else x for x, sb in zip(c["scores"], c["signbits"])],
                    np.float64)


def test_semantic_groups_reference_inline_cases(oracle):
    """The expectations of kvmem/tests/kvmem_store_test.cpp for
    pick_semantic_groups (whole-group admission, shared boundary charged once,
    newest mandatory ids kept under budget pressure)."""
    # four variable-length groups, budget 8, sink 1, recent 1 (:1020-1058)
    sel = oracle.pick_semantic_groups(oracle.make_cfg(32, 8, 1, 1), 20, 32 * 20,
                                      [(32, 128), (131, 251), (256, 352), (384, 448)],
                                      [1.0, 10.0, 9.0, 2.0])
    assert sel.size <= 8 and {0, 19, 4, 5, 6, 7} <= set(sel.tolist())
    assert not ({8, 9, 10} & set(sel.tolist()))
    # two groups sharing block 2, mandatory {7} (:1060-1080)
    sel = oracle.pick_semantic_groups(oracle.make_cfg(64, 4, 0, 0), 8, 64 * 8,
                                      [(64, 138), (138, 256)], [2.0, 1.0], [7])
    assert sel.tolist() == [1, 2, 3, 7]
    # sink {0} + mandatory {1,2,3,4} > budget 4: newest mandatory ids (:480-503)
    sel = oracle.pick_semantic_groups(oracle.make_cfg(32, 4, 1, 2), 10, 320, [(160, 224)], [1.0],
                                      [1, 2, 3, 4])
    assert sel.tolist() == [0, 2, 3, 4]


def test_semantic_groups_match_reference_golden(oracle):
    g = json.load(open(os.path.join(GOLD, "groups_golden.json")))
    for i, c in enumerate(g["cases"]):
        cfg = c["cfg"]
        n = (c["total_tokens"] + cfg["block_tokens"] - 1) // cfg["block_tokens"]
        sel = oracle.pick_semantic_groups(
            oracle.make_cfg(cfg["block_tokens"], cfg["budget_blocks"], cfg["sink_blocks"],
                            cfg["recent_blocks"]),
            n, c["total_tokens"], np.array(c["spans"], np.uint32).reshape(-1, 2),
            _group_case_scores(c), c["mandatory"])
        assert sel.tolist() == c["selected"], i


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(HERE), "oracle", "_ref",
                                                    "libkvmem_ref.so")),
                    reason="reference library not built here")
def test_semantic_groups_live_vs_reference(oracle):
    import sys
    sys.path.insert(0, GOLD)
    from make_golden import groups_case
    rng = np.random.default_rng(99)
    for _ in range(400):
        cfg, total, spans, scores, mand = groups_case(rng)
        rs = oracle.RefStore(block_tokens=cfg["block_tokens"],
                             select_budget=cfg["budget_blocks"] * cfg["block_tokens"],
                             sink_blocks=cfg["sink_blocks"], recent_blocks=cfg["recent_blocks"])
        rs.register_append(total)
        want = rs.pick_semantic_groups(spans, scores, mand)
        got = oracle.pick_semantic_groups(
            oracle.make_cfg(cfg["block_tokens"], cfg["budget_blocks"], cfg["sink_blocks"],
                            cfg["recent_blocks"]), rs.block_count(), total, spans, scores, mand)
        assert np.array_equal(got, want)


# ------------------------------------------------- stage-in transforms ---

def test_rope_oracle_matches_reference_golden(oracle):
    """The oracle's NeoX RoPE against kvmem::rope_neox_apply outputs (fixture
    made by the compiled reference), bit for bit."""
    g = np.load(os.path.join(GOLD, "rope_golden.npz"))
    for i in range(int(g["n_cases"])):
        H, D, n_rot, pos0, base, scale = g[f"case{i}"]
        H, D, n_rot, pos0 = int(H), int(D), int(n_rot), int(pos0)
        th = oracle.rope_theta(n_rot, float(np.float32(base)), float(np.float32(scale)))
        got = oracle.rope_neox_rows(g[f"x{i}"], H, D, n_rot, pos0, th)
        assert got.tobytes() == g[f"out{i}"].tobytes(), i


def test_fwht_oracle_exact_cases_and_inverse(oracle):
    n = 64
    e0 = np.zeros((1, n), np.float32)
    e0[0, 0] = 1.0
    assert np.all(oracle.fwht_rows(e0, n) == np.float32(0.125))     # first column of H/8
    ones = np.ones((1, 2 * n), np.float32)
    y = oracle.fwht_rows(ones, n)                                   # two chunks of 64
    assert y[0, 0] == 8.0 and y[0, n] == 8.0 and not np.any(np.delete(y[0], [0, n]))
    rng = np.random.default_rng(4)
    x = rng.standard_normal((5, 512)).astype(np.float32)
    for nrot in (64, 128, 256, 512):
        z = oracle.fwht_rows(oracle.fwht_rows(x, nrot), nrot)       # H is orthonormal, H^2 = I
        assert np.allclose(z, x, atol=1e-5)
        assert np.allclose(np.linalg.norm(oracle.fwht_rows(x, nrot), axis=1),
                           np.linalg.norm(x, axis=1), rtol=1e-5)


def test_attn_rot_sizes_follow_the_reference_rule(oracle):
    # kvmem_hadamard_nrot_k: the largest power of two >= 64 dividing head_dim;
    # V always 64; only quantized caches with head_dim % 64 == 0 rotate
    want_k = {64: 64, 128: 128, 192: 64, 256: 256, 320: 64, 384: 128, 512: 512}
    for d, n in want_k.items():
        assert oracle.attn_rot_nrot(oracle.TYPE_Q8_0, d, True) == n
        assert oracle.attn_rot_nrot(oracle.TYPE_Q4_0, d, False) == 64
    assert oracle.attn_rot_nrot(oracle.TYPE_F16, 256, True) == 0
    assert oracle.attn_rot_nrot(oracle.TYPE_Q8_0, 96, True) == 0


def test_attn_rot_rule_of_the_library_matches_oracle(oracle):
    import kvm
    kvm.build()
    L = kvm.lib()
    for ty in (oracle.TYPE_F16, oracle.TYPE_Q8_0, oracle.TYPE_Q4_0, oracle.TYPE_Q5_0):
        for d in (32, 64, 96, 128, 192, 256, 320, 384, 512, 1024):
            for k in (0, 1):
                assert L.kvm_attn_rot_nrot(ty, d, k) == oracle.attn_rot_nrot(ty, d, bool(k))


# ------------------------------------------------------ selection + diff ---

def _cfg_from(oracle, c):
    return oracle.make_cfg(c["block_tokens"], c["select_budget"] // c["block_tokens"],
                           c["sink_blocks"], c["recent_blocks"], c["optimize_stage_in"],
                           c["immutable_source_k"], c["immutable_refresh_remaps"],
                           c["immutable_refresh_abs_delta_tokens"],
                           c["immutable_max_baked_position"])


def test_store_golden_replay(oracle):
    with open(os.path.join(GOLD, "store_golden.json")) as f:
        gold = json.load(f)
    assert len(gold["cases"]) >= 20
    for case in gold["cases"]:
        c = case["cfg"]
        cfg = _cfg_from(oracle, c)
        blocks = oracle.Blocks.appended(case["n_tokens"], c["block_tokens"])
        for st in case["steps"]:
            sel = oracle.pick_topk(cfg, np.array(st["scores"]), st["mandatory"])
            assert sel.tolist() == st["selected"]
            plan = oracle.set_selection(cfg, blocks, sel)
            assert plan.stage_in.tolist() == st["stage_in"]
            assert plan.stage_out.tolist() == st["stage_out"]
            assert plan.rm_block_id.tolist() == st["rm_block_id"]
            assert plan.rm_from_base.tolist() == st["rm_from_base"]
            assert plan.rm_to_base.tolist() == st["rm_to_base"]
            assert plan.rm_skip.tolist() == st["rm_skip"]
            assert plan.rm_raw_refresh.tolist() == st["rm_raw_refresh"]
            assert plan.rm_working_k_resident.tolist() == st["rm_working_k_resident"]
            assert list(plan.counters()) == st["counters"]
            # the runtime's tier transitions (stage_out -> CPU, stage_in -> GPU)
            blocks.tier[plan.stage_out] = oracle.TIER_CPU
            blocks.gpu_slot[plan.stage_out] = -1
            blocks.tier[plan.stage_in] = oracle.TIER_GPU


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(HERE), "oracle", "_ref",
                                                    "libkvmem_ref.so")),
                    reason="reference library not built here")
def test_select_diff_live_vs_reference(oracle):
    rng = np.random.default_rng(1)
    for case in range(120):
        bt = int(rng.choice([32, 128]))
        nb = int(rng.integers(0, 300))
        ntok = nb * bt - (int(rng.integers(0, bt)) if nb else 0)
        bb = int(rng.integers(1, 80))
        sink, recent = int(rng.integers(0, 4)), int(rng.integers(0, 3))
        imm, osi = bool(rng.integers(0, 2)), bool(rng.integers(0, 5) > 0)
        kw = dict(block_tokens=bt, select_budget=bb * bt, sink_blocks=sink, recent_blocks=recent,
                  optimize_stage_in=osi, immutable_source_k=imm,
                  immutable_refresh_remaps=int(rng.integers(0, 4)),
                  immutable_refresh_abs_delta_tokens=int(rng.integers(0, 3)) * bt * 20,
                  immutable_max_baked_position=int(rng.integers(0, 2)) * bt * 200)
        R = oracle.RefStore(**kw)
        R.register_append(ntok)
        n = R.block_count()
        cfg = oracle.make_cfg(bt, bb, sink, recent, osi, imm, kw["immutable_refresh_remaps"],
                              kw["immutable_refresh_abs_delta_tokens"],
                              kw["immutable_max_baked_position"])
        blocks = R.blocks()
        for step in range(5):
            scores = rng.standard_normal(n)
            if step % 2:
                scores = np.round(scores * 2) / 2
            mand = rng.integers(0, n + 3, size=int(rng.integers(0, 6))).astype(np.uint32)
            R.set_retrieval_scores(scores)
            a = R.pick_topk_blocks(mand)
            assert np.array_equal(a, oracle.pick_topk(cfg, scores, mand))
            pa = R.set_selection(a)
            pb = oracle.set_selection(cfg, blocks, a)
            for f in pa.__dataclass_fields__:
                assert np.array_equal(getattr(pa, f), getattr(pb, f)), f
            for b in pa.stage_out:
                R.set_block_tier(int(b), oracle.TIER_CPU, int(b), -1)
                blocks.tier[b], blocks.gpu_slot[b] = oracle.TIER_CPU, -1
            for b in pa.stage_in:
                R.set_block_tier(int(b), oracle.TIER_GPU, -1, -1)
                blocks.tier[b] = oracle.TIER_GPU
            rb = R.blocks()
            for f in ("n_tokens", "tier", "baked_pos", "remap_count", "remap_abs_delta",
                      "in_working_set"):
                assert np.array_equal(getattr(rb, f), getattr(blocks, f)), f


# The reference's inline expectations (kvmem/tests/kvmem_store_test.cpp), restated.

def test_ref_case_selection_diff_and_remap(oracle):
    # kvmem_store_test.cpp:53-110
    cfg = oracle.make_cfg(block_tokens=128, budget_blocks=1024)
    b = oracle.Blocks.appended(128 * 5, 128)
    plan = oracle.set_selection(cfg, b, [4, 0, 2])
    assert plan.stage_in.tolist() == [0, 2, 4]
    assert plan.stage_out.tolist() == [1, 3]
    assert plan.total_window_tokens == 128 * 3
    assert plan.rm_block_id.tolist() == [0, 2, 4]
    assert plan.rm_from_base.tolist() == [0, 256, 512]
    assert plan.rm_to_base.tolist() == [0, 128, 256]
    assert plan.rm_skip.tolist() == [1, 0, 0]
    assert b.remap_count[[0, 2, 4]].tolist() == [0, 1, 1]
    b.tier[plan.stage_out] = oracle.TIER_CPU
    plan2 = oracle.set_selection(cfg, b, [0, 2, 3])
    assert plan2.stage_in.tolist() == [3] and plan2.stage_out.tolist() == [4]
    assert plan2.rm_skip.tolist() == [1, 1, 0]
    assert plan2.rm_from_base[2] == 384 and plan2.rm_to_base[2] == 256
    assert b.remap_count[2] == 1 and b.remap_count[3] == 1


def test_ref_case_topk_sink_recent(oracle):
    # kvmem_store_test.cpp:284-314 (accumulate_attn == attn_score)
    cfg = oracle.make_cfg(block_tokens=128, budget_blocks=4, sink_blocks=1, recent_blocks=1)
    s = np.zeros(10)
    s[5], s[6], s[3] = 100.0, 90.0, 10.0
    assert oracle.pick_topk(cfg, s).tolist() == [0, 5, 6, 9]


def test_ref_case_topk_zero_recent(oracle):
    # kvmem_store_test.cpp:316-339
    cfg = oracle.make_cfg(block_tokens=128, budget_blocks=4, sink_blocks=1, recent_blocks=0)
    s = np.zeros(10)
    s[3], s[5], s[6], s[9] = 80.0, 100.0, 90.0, -100.0
    assert oracle.pick_topk(cfg, s).tolist() == [0, 3, 5, 6]


def test_ref_case_mandatory_inside_budget(oracle):
    # kvmem_store_test.cpp:433-458
    cfg = oracle.make_cfg(block_tokens=32, budget_blocks=4, sink_blocks=1, recent_blocks=0)
    s = np.zeros(10)
    s[2], s[3], s[4], s[8], s[9] = 100.0, 90.0, 80.0, -10.0, -20.0
    assert oracle.pick_topk(cfg, s, [8, 9]).tolist() == [0, 2, 8, 9]


def test_ref_case_mandatory_dedupe_recent_best_effort(oracle):
    # kvmem_store_test.cpp:460-477
    cfg = oracle.make_cfg(block_tokens=32, budget_blocks=4, sink_blocks=2, recent_blocks=3)
    assert oracle.pick_topk(cfg, np.zeros(10), [0, 0, 5]).tolist() == [0, 1, 5, 9]


def test_ref_case_mandatory_overflow_trims_oldest(oracle):
    # kvmem_store_test.cpp:479-504
    cfg = oracle.make_cfg(block_tokens=32, budget_blocks=4, sink_blocks=1, recent_blocks=2)
    assert oracle.pick_topk(cfg, np.zeros(10), [1, 2, 3, 4]).tolist() == [0, 2, 3, 4]


def test_ref_case_all_fit_and_empty(oracle):
    # kvmem_store_test.cpp:763-781
    cfg = oracle.make_cfg(block_tokens=128, budget_blocks=100)
    assert oracle.pick_topk(cfg, np.zeros(3)).tolist() == [0, 1, 2]
    assert oracle.pick_topk(cfg, np.zeros(0)).tolist() == []
    b = oracle.Blocks.appended(0, 128)
    plan = oracle.set_selection(cfg, b, [0, 1])
    assert plan.rm_block_id.size == 0 and plan.total_window_tokens == 0


def test_layout_chronological(oracle):
    slot_before = np.array([-1, 3, 0, -1, 1, 2], dtype=np.int32)
    slot_after, moves, cold = oracle.layout(np.array([1, 2, 3, 5], np.uint32), slot_before)
    assert slot_after.tolist() == [-1, 0, 1, 2, -1, 3]
    assert moves.tolist() == [[1, 3, 0], [2, 0, 1], [5, 2, 3]]
    assert cold.tolist() == [[3, 2]]


# ---------------------------------------------------------------- scorer ---

def _score_numpy(sums, cnt, has, q, qc, Hkv, Hq, D):
    """Independent restatement with numpy float32 sequential sums (cumsum)."""
    L, B, E = sums.shape
    g = Hq // Hkv
    out = np.zeros(B)
    for b in range(B):
        if not has[b]:
            continue
        acc, nl = 0.0, 0
        for il in range(L):
            if qc[il] == 0:
                continue
            if cnt[il, b]:
                mk = sums[il, b] * (np.float32(1.0) / np.float32(cnt[il, b]))
            else:
                mk = np.zeros(E, np.float32)
            invq = np.float32(1.0) / np.float32(qc[il] * g)
            layer = 0.0
            for h in range(Hkv):
                qh = np.zeros(D, np.float32)
                for gi in range(g):
                    qh = (qh + q[il, (h * g + gi) * D:(h * g + gi + 1) * D]).astype(np.float32)
                qv = (qh * invq).astype(np.float32)
                kh = mk[h * D:(h + 1) * D]
                dot = np.cumsum((qv * kh).astype(np.float32), dtype=np.float32)[-1]
                nq = np.cumsum((qv * qv).astype(np.float32), dtype=np.float32)[-1]
                nk = np.cumsum((kh * kh).astype(np.float32), dtype=np.float32)[-1]
                den = np.float32(np.sqrt(nq) * np.sqrt(nk)) + np.float32(1e-6)
                layer += float(np.float32(dot / np.float32(den)))
            acc += layer / Hkv
            nl += 1
        out[b] = acc / nl if nl else 0.0
    return out


def test_scorer_matches_independent_restatement(oracle):
    rng = np.random.default_rng(7)
    L, B, Hkv, D, Hq = 3, 40, 2, 32, 6
    E = Hkv * D
    sums = (rng.standard_normal((L, B, E)) * 50).astype(np.float32)
    cnt = rng.integers(1, 129, size=(L, B)).astype(np.uint32)
    cnt[1, 3] = 0                       # a layer without statistics
    has = np.ones(B, np.uint8)
    has[7] = 0                          # a block without data
    q = rng.standard_normal((L, Hq * D)).astype(np.float32)
    qc = np.array([1, 0, 3], np.uint32)  # layer 1 has no query
    got, terms = oracle.score(sums, cnt, has, q, qc, Hkv, Hq, D, want_terms=True)
    want = _score_numpy(sums, cnt, has, q, qc, Hkv, Hq, D)
    assert got.tobytes() == want.tobytes()
    assert got[7] == 0.0 and np.all(terms[1] == 0.0)
    mt = oracle.score(sums, cnt, has, q, qc, Hkv, Hq, D, n_threads=4)
    assert mt.tobytes() == got.tobytes()


def test_scorer_matches_reference_golden(oracle):
    """Scores of the reference's own score_retrieval, recorded by
    tests/golden/make_golden.py, equal the oracle's bit for bit."""
    g = np.load(os.path.join(GOLD, "score_golden.npz"))
    for i in range(int(g["n_cases"])):
        L, B, Hkv, Hq, D, T = (int(x) for x in g[f"shape{i}"])
        sums, cnt = g[f"sums{i}"], g[f"cnt{i}"]
        has = (cnt > 0).any(axis=0).astype(np.uint8)
        got = oracle.score(sums, cnt, has, g[f"q{i}"], g[f"qc{i}"], Hkv, Hq, D)
        assert got.tobytes() == g[f"scores{i}"].tobytes(), i


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(HERE), "oracle", "_ref",
                                                    "libkvmem_ref.so")),
                    reason="reference library not built here")
def test_scorer_live_vs_reference_function(oracle):
    """The oracle's scorer against llama_memory_kvmem::score_retrieval itself
    (llama-memory-kvmem.cpp:2869-2916) on seeded shapes: GQA groups with and
    without a remainder, head sizes 32-256, partial and missing statistics,
    layers without query, every layer without query."""
    import sys
    sys.path.insert(0, GOLD)
    from make_golden import score_case
    rng = np.random.default_rng(31)
    for it in range(40):
        L = int(rng.integers(1, 5))
        B = int(rng.integers(5, 90))
        Hkv = int(rng.choice([1, 2, 4, 8]))
        Hq = Hkv * int(rng.integers(1, 7)) + (int(rng.integers(0, Hkv)) if it % 3 == 0 else 0)
        D = int(rng.choice([32, 64, 80, 128, 256]))
        T = int(rng.choice([16, 32, 128]))
        qc = rng.integers(0, 4, L)
        if it == 7:
            qc[:] = 0
        sums, cnt, q, qcount = score_case(rng, L, B, Hkv, Hq, D, T, qc)
        has = (cnt > 0).any(axis=0).astype(np.uint8)
        want = oracle.ref_score(sums, cnt, q, qcount, Hkv, Hq, D, T)
        got = oracle.score(sums, cnt, has, q, qcount, Hkv, Hq, D)
        assert got.tobytes() == want.tobytes(), (it, L, B, Hkv, Hq, D, T)
        if it == 7:
            assert not want.any()
