"""Layer-split scoring on the GPU.

One GPU: two sessions holding half the layers each emulate two ranks; their
terms, combined in layer order (kvm_reduce_terms), must give bit-identical
scores and the same selection as one session holding every layer.
Two GPUs: the same over NCCL through torchrun (skipped with fewer devices)."""
import json
import os
import socket
import subprocess
import sys
import tempfile

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _session(kvm, n_layer, B, T=32):
    cfg = kvm.default_config(n_layer=n_layer, n_head_kv=4, head_dim=64, n_head_q=12,
                             max_blocks=1024, block_tokens=T, select_budget=T * 64,
                             gen_reserve=T * 8, sink_blocks=1)
    s = kvm.Session(cfg, 0)
    s.register_append(B * T - 5)
    return s


def test_layer_split_emulated_on_one_gpu(kvm_lib, oracle):
    import torch
    rng = np.random.default_rng(5)
    L, B, E = 6, 900, 256
    sums = (rng.standard_normal((L, B, E)) * 25).astype(np.float32)
    cnt = np.full((L, B), 32, np.uint32)
    cnt[:, -1] = 27
    q = rng.standard_normal((L, 12 * 64)).astype(np.float32)
    qc = np.array([1, 1, 0, 1, 2, 1], np.uint32)
    full = _session(kvm_lib, L, B)
    for l in range(L):
        full.upload_summaries(l, 0, sums[l], cnt[l])
    full.set_query(q, qc)
    full.score()
    want = full.scores()
    full.select([])
    want_sel = full.plan()["selected"]
    parts = []
    for l0, l1 in ((0, 3), (3, 6)):
        s = _session(kvm_lib, l1 - l0, B)
        for i, l in enumerate(range(l0, l1)):
            s.upload_summaries(i, 0, sums[l], cnt[l])
        s.set_query(np.ascontiguousarray(q[l0:l1]), qc[l0:l1])
        t = torch.zeros((l1 - l0, 1024), dtype=torch.float64, device="cuda")
        s.score_terms(0, l1 - l0, t.data_ptr(), 1024)
        parts.append((s, t))
    terms = torch.cat([t[:, :B] for _, t in parts]).contiguous()
    acc = torch.zeros(1024, dtype=torch.float64, device="cuda")
    s0 = parts[0][0]
    s0.reduce_terms(terms.data_ptr(), L, B, acc.data_ptr())
    s0.set_scores_from_sum(acc.data_ptr(), int((qc > 0).sum()))
    assert s0.scores().tobytes() == want.tobytes()
    s0.select([])
    assert np.array_equal(s0.plan()["selected"], want_sel)
    assert want.tobytes() == oracle.score(sums, cnt, np.ones(B, np.uint8), q, qc, 4, 12, 64).tobytes()


@pytest.mark.parametrize("mode", ["allgather", "allreduce"])
def test_layer_split_nccl_two_gpus(kvm_lib, mode):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        port = so.getsockname()[1]
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "verdict.json")
        env = dict(os.environ, NCCL_NVLS_ENABLE="0")
        subprocess.run(["timeout", "-k", "30", "300", sys.executable, "-m",
                        "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
                        "--master-addr", "127.0.0.1", "--master-port", str(port),
                        os.path.join(HERE, "dist_gpu_worker.py"), out, mode],
                       check=True, env=env)
        v = json.load(open(out))
    assert v["ok"] and v["world"] == 2
