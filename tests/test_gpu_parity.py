"""GPU parity of libkvm against the CPU oracle, through the C ABI.

Bit-exact bars: quantized window bytes, selected block ids, KvMemPlan
fields, slot layout.  Scores: the device restates the reference arithmetic
operation for operation, so they are compared bit for bit as well (the
north-star tolerance of 1e-4 relative is asserted separately as the floor).
"""
import os

import numpy as np
import pytest

from kvm_testlib import OracleModel, Shape, make_query, make_rig

pytestmark = pytest.mark.gpu


def _cuda():
    import torch
    return torch


# ----------------------------------------------------------- quantizers ---

@pytest.mark.parametrize("type_id", [8, 2, 6, 1])
def test_quantize_rows_bitexact(kvm_lib, oracle, type_id):
    torch = _cuda()
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "quant_golden.npz"))
    rng = np.random.default_rng(type_id)
    rows = np.concatenate([
        g["rows_f16"].view(np.float16),
        oracle.synth_f16(rng, (37, 256), 256),           # row count not a tile multiple
    ])
    n, E = rows.shape
    src = torch.from_numpy(rows).cuda()
    rb = kvm_lib.row_bytes(type_id, E)
    dst = torch.zeros(n * rb, dtype=torch.uint8, device="cuda")
    kvm_lib.quantize_rows(type_id, src.data_ptr(), n, E, dst.data_ptr())
    got = dst.cpu().numpy().reshape(n, rb)
    want = oracle.quantize_rows_f16(type_id, rows)
    assert np.array_equal(got, want)
    if type_id != 1:
        # against the third-party golden bytes too (same -0.0 caveat as the oracle test)
        name = {8: "q8_0", 2: "q4_0", 6: "q5_0"}[type_id]
        gold = g[name]
        k = gold.shape[0]
        blk = g["rows_f16"].view(np.float16).astype(np.float32).reshape(k, -1, 32)
        neg0 = np.all(blk == 0, axis=2) & np.signbit(blk[:, :, 0])
        bs = {8: 34, 2: 18, 6: 22}[type_id]
        differ = np.any(got[:k].reshape(k, -1, bs) != gold.reshape(k, -1, bs), axis=2)
        assert not np.any(differ & ~neg0)


def test_quantize_rows_wide_and_narrow(kvm_lib, oracle):
    torch = _cuda()
    rng = np.random.default_rng(9)
    for E in (32, 96, 1024, 4096):
        rows = oracle.synth_f16(rng, (19, E), E)
        src = torch.from_numpy(rows).cuda()
        for t in (8, 2, 6):
            rb = kvm_lib.row_bytes(t, E)
            dst = torch.zeros(19 * rb, dtype=torch.uint8, device="cuda")
            kvm_lib.quantize_rows(t, src.data_ptr(), 19, E, dst.data_ptr())
            assert np.array_equal(dst.cpu().numpy().reshape(19, rb),
                                  oracle.quantize_rows_f16(t, rows)), (E, t)


@pytest.mark.parametrize("type_id", [8, 2, 6])
def test_quantize_rows_many(kvm_lib, oracle, type_id):
    """8M values: a contracted multiply-add in the code computation changes a
    q4_0 / q5_0 code a few times per million values."""
    torch = _cuda()
    rng = np.random.default_rng(40 + type_id)
    n, E = 8192, 1024
    rows = oracle.synth_f16(rng, (n, E), E)
    src = torch.from_numpy(rows).cuda()
    rb = kvm_lib.row_bytes(type_id, E)
    dst = torch.zeros(n * rb, dtype=torch.uint8, device="cuda")
    kvm_lib.quantize_rows(type_id, src.data_ptr(), n, E, dst.data_ptr())
    assert np.array_equal(dst.cpu().numpy().reshape(n, rb), oracle.quantize_rows_f16(type_id, rows))


def _edge_rows():
    """Blocks at the quantizers' boundaries: zeros and -0, +a/-a magnitude
    ties (q4/q5 keep the first), F16 max and subnormals, and scales where
    x*id + off lands exactly on integers and half-integers."""
    f = np.float16
    E = 256
    rows = []
    rows.append(np.zeros(E, f))
    rows.append(np.full(E, -0.0, f))
    r = np.zeros(E, np.float32)
    for blk in range(E // 32):                   # tie at varying positions, either sign first
        r[blk * 32 + (blk * 5) % 32] = 3.0 if blk % 2 else -3.0
        r[blk * 32 + (blk * 11 + 7) % 32] = -3.0 if blk % 2 else 3.0
        r[blk * 32 + (blk * 3 + 1) % 32] = 1.5
    rows.append(r.astype(f))
    rows.append(np.tile(np.array([65504.0, -65504.0, 1.0, -0.5], f), E // 4))
    rows.append((np.arange(E) % 17 - 8).astype(f) * f(2.0 ** -24))          # subnormal F16
    rows.append((np.arange(E) % 32 - 16).astype(np.float32).astype(f) * f(0.5))  # vmax -8: id 1
    rows.append((np.arange(E) % 32 - 15.5).astype(f))                            # half-integers
    rows.append(np.where(np.arange(E) % 32 == 0, -16.0, (np.arange(E) % 33) - 16.0).astype(f))
    # x*id rounds to exactly -7.5 (q4_0: x0 + 8.5 = 1.0); a multiply-add fused
    # without the product's rounding gives 0.99999976 and code 0 instead of 1
    blk = np.zeros(32, np.float32)
    blk[21], blk[26], blk[0] = -2.578125, -2.75, -2.263671875
    rows.append(np.tile(blk, E // 32).astype(f))
    # non-finite inputs: the reference's NaN-blind max scans, d = inf / 127
    # (or vmax = +-inf) with id = 0, and code 0 wherever x * id is NaN
    base = ((np.arange(E) % 29) - 14).astype(np.float32) * 0.25
    r = base.copy()
    r[(np.arange(E // 32) * 32 + (np.arange(E // 32) * 7) % 32)] = np.where(np.arange(E // 32) % 2, np.inf, -np.inf)
    rows.append(r.astype(f))
    r = base.copy()
    r[np.arange(E) % 32 == 3] = np.nan
    r[np.arange(E) % 64 == 40] = np.nan
    rows.append(r.astype(f))
    rows.append(np.full(E, np.nan, f))                                    # all-NaN blocks: d = 0
    r = np.full(E, np.nan, np.float32)
    r[np.arange(E) % 32 == 5] = -np.inf
    r[np.arange(E) % 64 == 9] = 2.0
    rows.append(r.astype(f))
    return np.stack(rows)


@pytest.mark.parametrize("type_id", [8, 2, 6])
def test_quantize_rows_edge_values(kvm_lib, oracle, type_id):
    torch = _cuda()
    rows = _edge_rows()
    n, E = rows.shape
    src = torch.from_numpy(rows).cuda()
    rb = kvm_lib.row_bytes(type_id, E)
    dst = torch.zeros(n * rb, dtype=torch.uint8, device="cuda")
    kvm_lib.quantize_rows(type_id, src.data_ptr(), n, E, dst.data_ptr())
    assert np.array_equal(dst.cpu().numpy().reshape(n, rb), oracle.quantize_rows_f16(type_id, rows))


# --------------------------------------------------------------- scorer ---

@pytest.mark.parametrize("Hkv,D,Hq", [(4, 64, 12), (2, 80, 6), (1, 1024, 2)])
def test_score_bitexact_uploaded_summaries(kvm_lib, oracle, Hkv, D, Hq):
    """Head sizes below, off and at the top of the channel batch (64, 80, 1024)."""
    torch = _cuda()
    rng = np.random.default_rng(21 + D)
    L, B = 3, 300
    E = Hkv * D
    cfg = kvm_lib.default_config(n_layer=L, n_head_kv=Hkv, head_dim=D, n_head_q=Hq,
                                 max_blocks=512, block_tokens=128, select_budget=128 * 32,
                                 gen_reserve=128 * 8)
    s = kvm_lib.Session(cfg, 0)
    s.register_append(B * 128 - 77)
    sums = (rng.standard_normal((L, B, E)) * 40).astype(np.float32)
    cnt = np.full((L, B), 128, np.uint32)
    cnt[:, -1] = 128 - 77
    cnt[2, 5] = 0                                    # no statistics in one layer
    for l in range(L):
        s.upload_summaries(l, 0, sums[l], cnt[l])
    q = rng.standard_normal((L, Hq * D)).astype(np.float32)
    qc = np.array([1, 2, 0], np.uint32)
    s.set_query(torch.from_numpy(q).cuda(), qc)
    s.score()
    got = s.scores()
    has = np.ones(B, np.uint8)
    want = oracle.score(sums, cnt, has, q, qc, Hkv, Hq, D)
    assert got.tobytes() == want.tobytes()
    rel = np.abs(got - want) / np.maximum(np.abs(want), 1e-30)
    assert rel.max() <= 1e-4


def test_score_matches_reference_golden(kvm_lib):
    """Device scores equal, bit for bit, the scores that the reference
    adapter's own score_retrieval (llama-memory-kvmem.cpp:2869-2916, compiled
    from its file by oracle/Makefile) produced for the same summaries and
    query sums (tests/golden/score_golden.npz)."""
    torch = _cuda()
    g = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "score_golden.npz"))
    for i in range(int(g["n_cases"])):
        L, B, Hkv, Hq, D, T = (int(x) for x in g[f"shape{i}"])
        sums, cnt = g[f"sums{i}"], g[f"cnt{i}"]
        cfg = kvm_lib.default_config(n_layer=L, n_head_kv=Hkv, head_dim=D, n_head_q=Hq,
                                     max_blocks=128, block_tokens=T, select_budget=T * 8,
                                     gen_reserve=T * 4)
        s = kvm_lib.Session(cfg, 0)
        s.register_append(B * T)
        for l in range(L):
            s.upload_summaries(l, 0, sums[l], cnt[l])
        s.set_query(torch.from_numpy(g[f"q{i}"]).cuda(), g[f"qc{i}"])
        s.score()
        assert s.scores().tobytes() == g[f"scores{i}"].tobytes(), i
        s.close()


def test_score_from_summarize_kernel(kvm_lib, oracle):
    shape = Shape(n_layer=2, n_blocks=70, block_tokens=32, partial_tokens=9)
    rig = make_rig(shape, seed=3)
    om = OracleModel(rig)
    q, qc = make_query(shape, np.random.default_rng(4))
    rig.sess.set_query(q, qc)
    rig.sess.score()
    assert rig.sess.scores().tobytes() == om.score(q, qc).tobytes()


# ------------------------------------------------------------- selection ---

@pytest.mark.parametrize("seed", range(6))
def test_select_matches_oracle(kvm_lib, oracle, seed):
    rng = np.random.default_rng(100 + seed)
    n = int(rng.integers(1, 3000))
    budget = int(rng.integers(1, 400))
    sink, recent = int(rng.integers(0, 4)), int(rng.integers(0, 4))
    if sink + recent > budget:
        sink = recent = 0
    cfg = kvm_lib.default_config(block_tokens=128, select_budget=budget * 128,
                                 gen_reserve=128, sink_blocks=sink, recent_blocks=recent,
                                 max_blocks=4096)
    s = kvm_lib.Session(cfg, 0)
    s.register_append(n * 128)
    ocfg = oracle.make_cfg(128, budget, sink, recent)
    for trial in range(5):
        scores = rng.standard_normal(n)
        if trial == 1:
            scores = np.round(scores * 3) / 3            # many exact ties
        if trial == 2:
            scores[:] = 0.0
            scores[rng.integers(0, n, n // 3)] = -0.0    # +0 / -0 compare equal
        if trial == 3:
            scores = np.abs(scores) * 1e-300             # subnormal / tiny
        mand = rng.integers(0, n + 5, size=int(rng.integers(0, 40))).astype(np.uint32)
        s.set_scores(scores)
        s.select(mand)
        got = s.plan()["selected"]
        want = oracle.pick_topk(ocfg, scores, mand)
        assert np.array_equal(got, want), (trial, n, budget)


def _select_vs_oracle(kvm_lib, oracle, n, budget, scores_list, sink=0, recent=0, mand=()):
    cfg = kvm_lib.default_config(block_tokens=128, select_budget=budget * 128,
                                 gen_reserve=128, sink_blocks=sink, recent_blocks=recent,
                                 max_blocks=max(n, 256))
    s = kvm_lib.Session(cfg, 0)
    try:
        s.register_append(n * 128)
        ocfg = oracle.make_cfg(128, budget, sink, recent)
        for i, scores in enumerate(scores_list):
            s.set_scores(scores)
            s.select(np.asarray(mand, np.uint32))
            got = s.plan()["selected"]
            want = oracle.pick_topk(ocfg, scores, np.asarray(mand, np.uint32))
            assert np.array_equal(got, want), (n, budget, i)
    finally:
        s.close()


def test_select_around_the_sign_halves(kvm_lib, oracle):
    """The selection's first digit is the key's sign half: scores >= 0 (+0 and
    -0 alike) above the negative ones.  The count of non-negative candidates
    is set to none, need - 1, need, need + 1 and all, so the threshold falls on
    each side of the split and on its edge, with zeros at the boundary."""
    rng = np.random.default_rng(31)
    n, budget = 1500, 200
    need = budget                                       # no pins: every slot is filled by score
    cases = []
    for c1 in (0, need - 1, need, need + 1, n):
        mag = np.abs(rng.standard_normal(n)) + 1e-3
        sign = np.full(n, -1.0)
        sign[rng.permutation(n)[:c1]] = 1.0
        scores = sign * mag
        cases.append(scores)
        z = scores.copy()                               # the smallest non-negative are zeros
        pos = np.flatnonzero(z >= 0)
        if pos.size:
            z[pos[: max(1, pos.size // 4)]] = np.where(rng.random(max(1, pos.size // 4)) < 0.5, 0.0, -0.0)
        cases.append(z)
        cases.append(np.round(scores * 2) / 2)          # ties across both halves
    _select_vs_oracle(kvm_lib, oracle, n, budget, cases)


@pytest.mark.parametrize("n", [8193, 20000])
def test_select_more_blocks_than_cached_keys(kvm_lib, oracle, n):
    """Above 8192 blocks a thread owns more than its 8 register-cached keys and
    reads them again on every pass."""
    rng = np.random.default_rng(n)
    s0 = rng.standard_normal(n)
    cases = [s0, np.round(s0 * 4) / 4, np.abs(s0) * 1e-300, -np.abs(s0)]
    _select_vs_oracle(kvm_lib, oracle, n, 300, cases, sink=1, recent=0, mand=[n - 1, 5])


def test_select_empty_and_all_fit(kvm_lib, oracle):
    cfg = kvm_lib.default_config(block_tokens=128, select_budget=128 * 100, max_blocks=256)
    s = kvm_lib.Session(cfg, 0)
    s.set_scores(np.zeros(0))
    s.select([])
    s.diff()
    assert s.plan()["selected"].size == 0
    s.register_append(3 * 128)
    s.set_scores(np.array([3.0, 1.0, 2.0]))
    s.select([])
    s.diff()
    assert s.plan()["selected"].tolist() == [0, 1, 2]


# --------------------------------------------------------- diff + layout ---

@pytest.mark.parametrize("imm,osi", [(False, True), (True, True), (False, False)])
def test_diff_sequence_matches_oracle(kvm_lib, oracle, imm, osi):
    _diff_sequence(kvm_lib, oracle, imm, osi, 200, 40, 7 + imm + 2 * osi)


@pytest.mark.parametrize("imm,osi", [(False, True), (True, True)])
def test_diff_sequence_many_blocks(kvm_lib, oracle, imm, osi):
    """9000 blocks: each thread of the one-CTA select + diff owns 9 ids, more
    than the selection's 8 register-cached keys."""
    _diff_sequence(kvm_lib, oracle, imm, osi, 9000, 300, 17 + imm)


def _diff_sequence(kvm_lib, oracle, imm, osi, n, budget, seed):
    rng = np.random.default_rng(seed)
    bt = 32
    cfg = kvm_lib.default_config(block_tokens=bt, select_budget=budget * bt, gen_reserve=8 * bt,
                                 sink_blocks=1, recent_blocks=1, max_blocks=max(256, n),
                                 immutable_source_k=int(imm), optimize_stage_in=int(osi),
                                 immutable_refresh_remaps=2, immutable_refresh_abs_delta_tokens=bt * 30)
    s = kvm_lib.Session(cfg, 0)
    s.register_append(n * bt - 5)
    ocfg = oracle.make_cfg(bt, budget, 1, 1, osi, imm, 2, bt * 30, 262144)
    blocks = oracle.Blocks.appended(n * bt - 5, bt, tier=oracle.TIER_CPU)
    prev = None
    for step in range(8):
        scores = rng.standard_normal(n)
        if prev is not None and step % 2:
            scores[prev] += 1.0                          # overlap with the previous selection
        mand = rng.integers(0, n, size=3).astype(np.uint32)
        s.set_scores(scores)
        s.select(mand)
        s.diff()
        got = s.plan()
        sel = oracle.pick_topk(ocfg, scores, mand)
        before = blocks.gpu_slot.copy()
        if not osi:
            before[:] = -1
        plan = oracle.set_selection(ocfg, blocks, sel)
        slot_after, moves, cold = oracle.layout(sel, before)
        blocks.gpu_slot[:] = slot_after
        blocks.tier[(slot_after < 0) & (blocks.tier == oracle.TIER_GPU)] = oracle.TIER_CPU
        blocks.tier[sel] = oracle.TIER_GPU
        assert np.array_equal(got["selected"], sel)
        assert np.array_equal(got["stage_in"], plan.stage_in)
        assert np.array_equal(got["stage_out"], plan.stage_out)
        for f in ("rm_block_id", "rm_n_tokens", "rm_from_base", "rm_to_base",
                  "rm_working_k_resident", "rm_skip", "rm_raw_refresh"):
            assert np.array_equal(got[f], getattr(plan, f)), f
        assert (got["total_window_tokens"], got["selection_overlap_blocks"],
                got["gpu_reused_blocks"], got["retained_position_stable"],
                got["retained_position_moved"]) == plan.counters()
        assert np.array_equal(np.stack([got["mv_block"], got["mv_from"], got["mv_to"]], 1)
                              .astype(np.int64), moves.astype(np.int64))
        assert np.array_equal(np.stack([got["cold_block"], got["cold_to"]], 1).astype(np.int64),
                              cold.astype(np.int64))
        prev = sel


# ------------------------------------------------------ full reselection ---

def _check_window(rig, om):
    mk, mv = om.window_valid_mask()
    gk = rig.win_k.cpu().numpy()
    gv = rig.win_v.cpu().numpy()
    assert np.array_equal(gk[:, mk], om.win_k[:, mk])
    assert np.array_equal(gv[:, mv], om.win_v[:, mv])


@pytest.mark.parametrize("tk,tv", [(8, 8), (8, 2), (6, 6), (1, 1)])
def test_step_window_bytes(kvm_lib, oracle, tk, tv):
    shape = Shape(n_layer=2, n_blocks=64, block_tokens=32, budget_blocks=12, gen_blocks=4,
                  type_k=tk, type_v=tv, partial_tokens=20)
    rig = make_rig(shape, seed=11)
    om = OracleModel(rig)
    rng = np.random.default_rng(12)
    q, qc = make_query(shape, rng)
    for step in range(4):
        if step:
            q2, _ = make_query(shape, rng)
            q = (0.8 * q + 0.6 * q2).astype(np.float32)  # overlapping selections
        rig.sess.set_query(q, qc)
        rig.sess.step(rig.src, rig.k_bases(), rig.v_bases(), mandatory=[shape.n_blocks - 1])
        _, sel, plan, moves, cold = om.step(q, qc, [shape.n_blocks - 1])
        got = rig.sess.plan()
        assert np.array_equal(got["selected"], sel)
        assert np.array_equal(np.stack([got["mv_block"], got["mv_from"], got["mv_to"]], 1)
                              .astype(np.int64), moves.astype(np.int64))
        _check_window(rig, om)
        if step:
            assert moves.shape[0] > 0 or cold.shape[0] < sel.size


def test_step_unaligned_rows(kvm_lib, oracle):
    """n_embd 96: q8_0 rows of 102 bytes are not 16-byte multiples, so the
    moves take the SIMT column kernel and the stage-in its word-store path."""
    shape = Shape(n_layer=2, n_blocks=64, block_tokens=32, n_head_kv=1, head_dim=96, n_head_q=3,
                  budget_blocks=12, gen_blocks=4, partial_tokens=11)
    rig = make_rig(shape, seed=23)
    om = OracleModel(rig)
    rng = np.random.default_rng(24)
    q, qc = make_query(shape, rng)
    n_moves = 0
    for step in range(4):
        if step:
            q2, _ = make_query(shape, rng)
            q = (0.8 * q + 0.6 * q2).astype(np.float32)
        rig.sess.set_query(q, qc)
        rig.sess.step(rig.src, rig.k_bases(), rig.v_bases(), mandatory=[shape.n_blocks - 1])
        _, sel, plan, moves, cold = om.step(q, qc, [shape.n_blocks - 1])
        got = rig.sess.plan()
        assert np.array_equal(got["selected"], sel)
        n_moves += moves.shape[0]
        _check_window(rig, om)
    assert n_moves > 0


def test_step_after_scrambled_slots(kvm_lib, oracle):
    """A layout that is not chronological (kvm_set_block_gpu_slot reversing the
    resident blocks' slots, the window bytes permuted to match): the next
    step's moves are not monotone, so the streaming permute must take its
    order-free column path; the window must still match the oracle."""
    torch = _cuda()
    shape = Shape(n_layer=2, n_blocks=64, block_tokens=32, budget_blocks=12, gen_blocks=4,
                  partial_tokens=20)
    rig = make_rig(shape, seed=17)
    om = OracleModel(rig)
    rng = np.random.default_rng(18)
    q, qc = make_query(shape, rng)
    rig.sess.set_query(q, qc)
    rig.sess.step(rig.src, rig.k_bases(), rig.v_bases())
    om.step(q, qc)
    _check_window(rig, om)
    # reverse the slots of the resident blocks, on the device and in the oracle
    res = np.nonzero(om.blocks.gpu_slot >= 0)[0]
    old = om.blocks.gpu_slot[res].copy()
    new = old[::-1].copy()
    L, T = shape.n_layer, shape.block_tokens
    for win_t, win_np, rb in ((rig.win_k, om.win_k, om.rbk), (rig.win_v, om.win_v, om.rbv)):
        span = T * rb
        dev = win_t.view(L, -1, span)
        snap_d = dev.clone()
        host = win_np.reshape(L, -1, span)
        snap_h = host.copy()
        for o, n in zip(old, new):
            dev[:, n] = snap_d[:, o]
            host[:, n] = snap_h[:, o]
    for b, n in zip(res, new):
        rig.sess.set_block_gpu_slot(int(b), int(n))
        om.blocks.gpu_slot[b] = n
    torch.cuda.synchronize()
    for step in range(2):
        q2, _ = make_query(shape, rng)
        q = (0.85 * q + 0.5 * q2).astype(np.float32)
        rig.sess.set_query(q, qc)
        rig.sess.step(rig.src, rig.k_bases(), rig.v_bases())
        _, sel, plan, moves, cold = om.step(q, qc)
        got = rig.sess.plan()
        assert np.array_equal(got["selected"], sel)
        assert np.array_equal(np.stack([got["mv_block"], got["mv_from"], got["mv_to"]], 1)
                              .astype(np.int64), moves.astype(np.int64))
        if step == 0:
            assert moves.shape[0] > 1 and np.any(np.diff(moves[:, 1]) < 0)   # not monotone
        _check_window(rig, om)
    rig.sess.wait()                     # raises on a device error status


def test_step_host_source(kvm_lib, oracle):
    torch = _cuda()
    shape = Shape(n_layer=2, n_blocks=48, block_tokens=32, budget_blocks=10, gen_blocks=2)
    rig = make_rig(shape, seed=5)
    om = OracleModel(rig)
    L, B, T, E = shape.n_layer, shape.n_blocks, shape.block_tokens, shape.n_embd
    hk = torch.from_numpy(rig.k_np).pin_memory()
    hv = torch.from_numpy(rig.v_np).pin_memory()
    src = kvm_lib.make_source(hk.data_ptr(), hv.data_ptr(), B * T * E * 2, T * E * 2, E * 2,
                              location=kvm_lib.LOC_HOST)
    rng = np.random.default_rng(6)
    q, qc = make_query(shape, rng)
    for step in range(3):
        if step:
            q = (0.7 * q + 0.7 * make_query(shape, rng)[0]).astype(np.float32)
        rig.sess.set_query(q, qc)
        rig.sess.step(src, rig.k_bases(), rig.v_bases())
        om.step(q, qc)
        rig.sess.wait()
        _check_window(rig, om)


def test_resident_append_and_reset(kvm_lib, oracle):
    shape = Shape(n_layer=1, n_blocks=40, block_tokens=32, budget_blocks=8, gen_blocks=4)
    rig = make_rig(shape, seed=8)
    q, qc = make_query(shape, np.random.default_rng(1))
    rig.sess.set_query(q, qc)
    rig.sess.step(rig.src, rig.k_bases(), rig.v_bases())
    p = rig.sess.plan()
    assert p["selected"].size == 8
    # decode tokens written by the model take the first free window slots (8, 9)
    rig.sess.register_append(40, resident=True)
    assert rig.sess.block_count == 42
    # the next reselection sees them as resident: selected ones move, others drop
    rig.sess.set_scores(np.r_[np.zeros(40), 5.0, 4.0])
    rig.sess.select([])
    rig.sess.diff()
    p = rig.sess.plan()
    assert 40 in p["selected"] and 41 in p["selected"]
    mv = dict(zip(p["mv_block"].tolist(), zip(p["mv_from"].tolist(), p["mv_to"].tolist())))
    assert mv[40][0] == 8 and mv[41][0] == 9
    assert 40 not in p["cold_block"] and 41 not in p["cold_block"]
    rig.sess.reset_window()
    rig.sess.set_scores(np.zeros(42))
    rig.sess.select([])
    rig.sess.diff()
    p = rig.sess.plan()
    assert p["mv_block"].size == 0 and p["cold_block"].size == 8
