"""Worker for tests/test_gpu_multi.py, launched by torchrun (one rank per GPU,
NCCL): a layer-split session scored on every rank, combined over NCCL, and
compared by rank 0 with a full single-GPU session.  Writes a JSON verdict."""
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "kvmem-llama.cpp_b200"))

import datetime  # noqa: E402

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import kvm  # noqa: E402
from kvm.dist import LayerSplit, layer_split_scores  # noqa: E402

L, B, HKV, D, HQ, T = 8, 700, 4, 64, 12, 32


def session(n_layer, dev):
    cfg = kvm.default_config(n_layer=n_layer, n_head_kv=HKV, head_dim=D, n_head_q=HQ,
                             max_blocks=1024, block_tokens=T, select_budget=T * 64,
                             gen_reserve=T * 8, sink_blocks=1)
    s = kvm.Session(cfg, dev)
    s.register_append(B * T)
    return s


def main():
    out, mode = sys.argv[1], sys.argv[2]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    rng = np.random.default_rng(11)
    E = HKV * D
    sums = (rng.standard_normal((L, B, E)) * 25).astype(np.float32)
    cnt = np.full((L, B), T, np.uint32)
    q = rng.standard_normal((L, HQ * D)).astype(np.float32)
    qc = np.ones(L, np.uint32)
    qc[3] = 0
    split = LayerSplit(L, rank, world, mode)
    s = session(split.n_local, local)
    for i, l in enumerate(range(split.l0, split.l1)):
        s.upload_summaries(i, 0, sums[l], cnt[l])
    s.set_query(np.ascontiguousarray(q[split.l0:split.l1]), qc[split.l0:split.l1])
    terms = torch.zeros((split.n_local, 1024), dtype=torch.float64, device="cuda")
    acc = torch.zeros(1024, dtype=torch.float64, device="cuda")
    layer_split_scores(s, split, terms, acc, int((qc > 0).sum()))
    s.select([])
    got = s.scores()
    sel = s.plan()["selected"]
    gathered = [None] * world
    dist.all_gather_object(gathered, (got.tobytes(), sel.tolist()))
    verdict = {"ok": True}
    if rank == 0:
        full = session(L, local)
        for l in range(L):
            full.upload_summaries(l, 0, sums[l], cnt[l])
        full.set_query(q, qc)
        full.score()
        want = full.scores()
        full.select([])
        want_sel = full.plan()["selected"].tolist()
        for sc, sl in gathered:
            g = np.frombuffer(sc, dtype=np.float64)
            if mode == "allgather":
                verdict["ok"] &= g.tobytes() == want.tobytes()
            else:
                verdict["ok"] &= bool(np.allclose(g, want, rtol=1e-12, atol=0))
            verdict["ok"] &= sl == want_sel
        verdict["world"] = world
        with open(out, "w") as f:
            json.dump(verdict, f)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
