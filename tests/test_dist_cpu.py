"""Multi-rank host logic on CPU (gloo, world sizes 2 and 4): the layer split of one
session over ranks, with the per-layer score terms from the CPU oracle.

allgather mode must reproduce the single-process scores bit for bit and the
same selection; allreduce mode must agree to 1e-12 relative and select the
same blocks."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

L, B, HKV, D, HQ = 6, 96, 2, 32, 6


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(seed=3):
    rng = np.random.default_rng(seed)
    E = HKV * D
    sums = (rng.standard_normal((L, B, E)) * 30).astype(np.float32)
    cnt = rng.integers(1, 129, size=(L, B)).astype(np.uint32)
    has = np.ones(B, np.uint8)
    has[5] = 0
    q = rng.standard_normal((L, HQ * D)).astype(np.float32)
    qc = np.array([1, 1, 0, 2, 1, 1], np.uint32)      # layer 2 has no query
    return sums, cnt, has, q, qc


def _worker(rank, world, port, mode, results):
    import sys
    for p in (os.path.join(ROOT, "kvmem-llama.cpp_b200"), os.path.join(ROOT, "oracle")):
        sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import oracle as O
        from kvm.dist import LayerSplit
        sums, cnt, has, q, qc = _inputs()
        split = LayerSplit(L, rank, world, mode)
        l0, l1 = split.l0, split.l1
        _, terms = O.score(sums[l0:l1], cnt[l0:l1], has, q[l0:l1], qc[l0:l1], HKV, HQ, D,
                           want_terms=True)
        if mode == "allgather":
            full = split.gather_terms(torch.from_numpy(terms)).numpy()
            acc = np.zeros(B)
            for row in full:                 # global layer order
                acc = acc + row
        else:
            part = np.zeros(B)
            for row in terms:
                part = part + row
            pt = torch.from_numpy(part)
            split.reduce_partial(pt)
            acc = pt.numpy()
        n_active = int((qc > 0).sum())
        scores = np.where(has > 0, acc / n_active, 0.0)
        sel = O.pick_topk(O.make_cfg(128, 20, 1, 0), scores)
        results[rank] = (scores.tobytes(), sel.tolist())
    finally:
        dist.destroy_process_group()


def _run(mode, world=2):
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), mode, results), nprocs=world,
                       start_method="spawn", join=True)
    return dict(results)


@pytest.mark.parametrize("mode,world", [("allgather", 2), ("allreduce", 2), ("allgather", 4)])
def test_layer_split_matches_single_process(oracle, mode, world):
    """World 4 splits the 6 layers 2, 2, 1, 1: the all-gather pads the short
    ranks' shares and drops the padding rows again."""
    sums, cnt, has, q, qc = _inputs()
    want = oracle.score(sums, cnt, has, q, qc, HKV, HQ, D)
    want_sel = oracle.pick_topk(oracle.make_cfg(128, 20, 1, 0), want)
    res = _run(mode, world)
    assert len(res) == world
    for rank in range(world):
        got = np.frombuffer(res[rank][0], dtype=np.float64)
        if mode == "allgather":
            assert got.tobytes() == want.tobytes()
        else:
            assert np.allclose(got, want, rtol=1e-12, atol=0)
        assert res[rank][1] == want_sel.tolist()
    assert all(res[r][0] == res[0][0] for r in range(world))    # identical scores on every rank


def test_layer_ranges_cover_all_layers():
    import sys
    sys.path.insert(0, os.path.join(ROOT, "kvmem-llama.cpp_b200"))
    from kvm.dist import layer_range
    for n in (1, 5, 16, 17):
        for w in (1, 2, 3, 4, 8):
            r = [layer_range(n, k, w) for k in range(w)]
            assert r[0][0] == 0 and r[-1][1] == n
            assert all(r[k][1] == r[k + 1][0] for k in range(w - 1))
            assert max(b - a for a, b in r) - min(b - a for a, b in r) <= 1
