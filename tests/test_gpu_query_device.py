"""kvm_set_query with a query in device memory: the query prep itself reads
it, in stream order at that call, and keeps the copy that kvm_query_add
accumulates on.  Scores must equal those of the same query passed from host
memory (the copy path) and the oracle's, bit for bit, also when the caller
rewrites its buffer right after the call, when a layer has no query, when
kvm_query_add follows, and beyond the prep's 64 inline layer counts."""
import numpy as np
import pytest

from kvm_testlib import OracleModel, Shape, make_query, make_rig

pytestmark = pytest.mark.gpu


def _torch():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    return torch


def _scores_host(s, q, qc):
    s.set_query(q, qc)
    s.score()
    return s.scores()


def test_device_query_equals_host_query_and_oracle(kvm_lib, oracle):
    torch = _torch()
    shape = Shape(n_layer=3, n_blocks=40, block_tokens=32, budget_blocks=8, gen_blocks=2)
    rig = make_rig(shape, seed=61)
    om = OracleModel(rig)
    q, qc = make_query(shape, np.random.default_rng(62), count=3)
    s = rig.sess
    host = _scores_host(s, q, qc)
    qd = torch.from_numpy(q).cuda()
    s.set_query(qd.data_ptr(), qc)
    s.score()
    dev = s.scores()
    assert np.array_equal(dev, host)
    assert np.array_equal(dev, om.score(q, qc))


def test_device_query_is_read_at_set_query(kvm_lib, oracle):
    """The caller rewrites its buffer on the same stream after kvm_set_query:
    the scores are still those of the values at the call."""
    torch = _torch()
    shape = Shape(n_layer=2, n_blocks=24, block_tokens=32, budget_blocks=6, gen_blocks=2)
    rig = make_rig(shape, seed=63)
    om = OracleModel(rig)
    q, qc = make_query(shape, np.random.default_rng(64))
    qd = torch.from_numpy(q).cuda()
    s = rig.sess
    s.set_query(qd.data_ptr(), qc)
    qd.mul_(-3.0)
    s.score()
    assert np.array_equal(s.scores(), om.score(q, qc))


def test_device_query_layer_without_query(kvm_lib, oracle):
    torch = _torch()
    shape = Shape(n_layer=4, n_blocks=36, block_tokens=32, budget_blocks=8, gen_blocks=2)
    rig = make_rig(shape, seed=65)
    om = OracleModel(rig)
    q, _ = make_query(shape, np.random.default_rng(66))
    qc = np.array([2, 0, 1, 0], np.uint32)
    s = rig.sess
    host = _scores_host(s, q, qc)
    s.set_query(torch.from_numpy(q).cuda().data_ptr(), qc)
    s.score()
    dev = s.scores()
    assert np.array_equal(dev, host)
    assert np.array_equal(dev, om.score(q, qc))


@pytest.mark.parametrize("counts", [(1, 1), (2, 0)])
def test_device_query_then_query_add(kvm_lib, oracle, counts):
    """kvm_query_add after a device kvm_set_query adds to the copied sum (also
    of a layer the set query left without tokens)."""
    torch = _torch()
    import kvm
    shape = Shape(n_layer=2, n_blocks=24, block_tokens=32, budget_blocks=6, gen_blocks=2)
    rig = make_rig(shape, seed=67)
    q, _ = make_query(shape, np.random.default_rng(68))
    qc = np.array(counts, np.uint32)
    rng = np.random.default_rng(69)
    extra = torch.from_numpy(rng.standard_normal((5, shape.n_head_q * shape.head_dim)).astype(np.float32)).cuda()
    rows = kvm.rows_of(extra, shape.n_head_q, shape.head_dim)
    s = rig.sess
    s.set_query(q, qc)
    s.query_add(1, 5, rows)
    s.score()
    host = s.scores()
    s.set_query(torch.from_numpy(q).cuda().data_ptr(), qc)
    s.query_add(1, 5, rows)
    s.score()
    assert np.array_equal(s.scores(), host)


def test_device_query_many_layers_takes_the_copy_path(kvm_lib, oracle):
    """More layers than the prep's inline counts: the query is copied."""
    torch = _torch()
    shape = Shape(n_layer=66, n_blocks=8, block_tokens=16, budget_blocks=4, gen_blocks=1)
    rig = make_rig(shape, seed=70)
    om = OracleModel(rig)
    q, qc = make_query(shape, np.random.default_rng(71))
    s = rig.sess
    s.set_query(torch.from_numpy(q).cuda().data_ptr(), qc)
    s.score()
    assert np.array_equal(s.scores(), om.score(q, qc))


def test_device_query_heads_not_a_multiple_of_kv_heads(kvm_lib, oracle):
    """n_head_q = 5 over 2 KV heads: the group size is 2 and head 4 is not
    summed, but it is part of the kept copy that kvm_query_add adds to."""
    torch = _torch()
    import kvm
    shape = Shape(n_layer=2, n_blocks=24, block_tokens=32, n_head_kv=2, n_head_q=5, budget_blocks=6,
                  gen_blocks=2)
    rig = make_rig(shape, seed=72)
    om = OracleModel(rig)
    q, qc = make_query(shape, np.random.default_rng(73))
    s = rig.sess
    host = _scores_host(s, q, qc)
    s.set_query(torch.from_numpy(q).cuda().data_ptr(), qc)
    s.score()
    dev = s.scores()
    assert np.array_equal(dev, host)
    assert np.array_equal(dev, om.score(q, qc))
    # the kept copies of both paths, head 4 included, are the same
    rng = np.random.default_rng(74)
    extra = torch.from_numpy(rng.standard_normal((3, shape.n_head_q * shape.head_dim)).astype(np.float32)).cuda()
    rows = kvm.rows_of(extra, shape.n_head_q, shape.head_dim)
    s.set_query(q, qc)
    s.query_add(0, 3, rows)
    s.score()
    host2 = s.scores()
    s.set_query(torch.from_numpy(q).cuda().data_ptr(), qc)
    s.query_add(0, 3, rows)
    s.score()
    assert np.array_equal(s.scores(), host2)
