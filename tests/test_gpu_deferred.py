"""Deferred launches keep call order: kvm_select and kvm_reset_window only
record their work, the next kvm_diff runs both in one launch, and every
other call that depends on them launches them first on its own stream.
Each test builds an order where running the work late would change the
result, and checks the result against the oracle."""
import numpy as np
import pytest

from kvm_testlib import OracleModel, Shape, make_query, make_rig

pytestmark = pytest.mark.gpu


def _topk(oracle, shape, scores):
    cfg = oracle.make_cfg(shape.block_tokens, shape.budget_blocks, shape.sink_blocks,
                          shape.recent_blocks)
    return oracle.pick_topk(cfg, np.asarray(scores, np.float64))


def test_select_uses_the_scores_it_was_called_with(kvm_lib, oracle):
    """select(); set_scores(new); diff(): the selection is the one of the
    scores installed before kvm_select."""
    shape = Shape(n_layer=1, n_blocks=32, block_tokens=32, budget_blocks=6, gen_blocks=2)
    rig = make_rig(shape, seed=51)
    s = rig.sess
    rng = np.random.default_rng(52)
    a, b = rng.standard_normal(32), rng.standard_normal(32)
    s.set_scores(a)
    s.select([])
    s.set_scores(b)            # must not reach the pending selection
    s.diff()
    assert np.array_equal(s.plan()["selected"], _topk(oracle, shape, a))
    s.select([])               # now with b
    s.diff()
    assert np.array_equal(s.plan()["selected"], _topk(oracle, shape, b))


def test_plan_read_between_select_and_diff(kvm_lib, oracle):
    """kvm_get_plan after kvm_select alone sees that selection; the diff
    afterwards lays it out as usual."""
    shape = Shape(n_layer=2, n_blocks=24, block_tokens=32, budget_blocks=6, gen_blocks=2)
    rig = make_rig(shape, seed=53)
    om = OracleModel(rig)
    q, qc = make_query(shape, np.random.default_rng(54))
    s = rig.sess
    s.set_query(q, qc)
    s.score()
    s.select([])
    scores, sel, _, _, _ = om.step(q, qc)
    assert np.array_equal(s.plan()["selected"], sel)
    s.diff()
    s.stagein(rig.src, rig.k_bases(), rig.v_bases())
    p = s.plan()
    assert np.array_equal(p["selected"], sel)
    mk, mv = om.window_valid_mask()
    assert np.array_equal(rig.win_k.cpu().numpy()[:, mk], om.win_k[:, mk])
    assert np.array_equal(rig.win_v.cpu().numpy()[:, mv], om.win_v[:, mv])


def test_reset_before_resident_append(kvm_lib, oracle):
    """reset_window(); register_append(resident); select(); diff(): the reset
    happens before the append, so the appended block stays resident in the
    slot it was given (a move, not a cold stage-in)."""
    shape = Shape(n_layer=1, n_blocks=20, block_tokens=32, budget_blocks=6, gen_blocks=2)
    rig = make_rig(shape, seed=55)
    s = rig.sess
    q, qc = make_query(shape, np.random.default_rng(56))
    s.set_query(q, qc)
    s.step(rig.src, rig.k_bases(), rig.v_bases())
    s.plan()
    s.reset_window()
    s.register_append(32, resident=True)        # block 20, window slot 0 (all free)
    new = s.block_count - 1
    sc = np.zeros(s.block_count)
    sc[new] = 9.0
    sc[3] = 8.0
    s.set_scores(sc)
    s.select([])
    s.diff()
    p = s.plan()
    assert new in p["selected"]
    mv = dict(zip(p["mv_block"].tolist(), p["mv_from"].tolist()))
    assert mv.get(new) == 0, p
    assert new not in p["cold_block"]


def test_two_streams_ordered_by_a_wait(kvm_lib, oracle):
    """select() on stream A, B.wait_stream(A), set_scores() and diff() on B:
    the pending selection runs on B before the new scores land."""
    import torch
    shape = Shape(n_layer=1, n_blocks=32, block_tokens=32, budget_blocks=6, gen_blocks=2)
    rig = make_rig(shape, seed=57)
    s = rig.sess
    rng = np.random.default_rng(58)
    a, b = rng.standard_normal(32), rng.standard_normal(32)
    sa, sb = torch.cuda.Stream(), torch.cuda.Stream()
    da = torch.from_numpy(a).cuda()
    db = torch.from_numpy(b).cuda()
    torch.cuda.synchronize()
    s.set_scores(da, stream=sa)
    s.select([], stream=sa)
    sb.wait_stream(sa)
    s.set_scores(db, stream=sb)
    s.diff(stream=sb)
    torch.cuda.synchronize()
    assert np.array_equal(s.plan(stream=sb)["selected"], _topk(oracle, shape, a))
