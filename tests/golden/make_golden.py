"""Generate the golden fixtures in this directory.

Run in a container that has the reference tree (for oracle/_ref) and gguf-py:

    python tests/golden/make_golden.py

Outputs (all small, committed):
  quant_golden.npz   seeded F16 rows + the q8_0 / q4_0 / q5_0 bytes gguf-py 0.19.0
                     produces for them (third-party oracle of ggml's quantizers)
  store_golden.json  selection + KvMemPlan sequences produced by the reference's own
                     kvmem::KvMemStore (oracle/_ref/libkvmem_ref.so)
  meank_golden.npz   means produced by the reference's own kvmem::RawKvStore
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle as O  # noqa: E402


def quant_rows(rng):
    """Seeded F16 rows with the bench distribution plus edge-case rows."""
    E = 256
    x = O.synth_f16(rng, (96, E), E).astype(np.float32)
    edge = np.zeros((8, E), dtype=np.float32)
    edge[0] = 0.0                                   # all-zero blocks
    edge[1] = 0.5                                   # constant blocks (ties everywhere)
    edge[2, ::2] = 127.0 * 0.5 / 127.0              # .5 ties after scaling
    edge[2, 1::2] = -1.0
    edge[3] = rng.choice([-65504.0, 65504.0, 0.0], size=E)   # F16 extremes
    edge[4] = (rng.standard_normal(E) * 6e-8)       # F16 subnormals
    edge[5] = np.tile(np.array([3.0, -3.0] * 16, dtype=np.float32), E // 32)  # |max| tie, sign order
    edge[6] = np.tile(np.array([-3.0, 3.0] * 16, dtype=np.float32), E // 32)
    edge[7] = np.linspace(-8.5, 8.5, E)             # q4 boundary region
    rows = np.concatenate([x, edge]).astype(np.float16)
    return rows


def make_quant(rng):
    import gguf
    from gguf.constants import GGMLQuantizationType as T
    rows = quant_rows(rng)
    f = rows.astype(np.float32)
    out = {"rows_f16": rows.view(np.uint16), "gguf_version": np.array(gguf.__version__ if hasattr(gguf, "__version__") else "0.19.0")}
    for name, t in (("q8_0", T.Q8_0), ("q4_0", T.Q4_0), ("q5_0", T.Q5_0)):
        out[name] = gguf.quants.quantize(f, t).reshape(rows.shape[0], -1)
    np.savez_compressed(os.path.join(HERE, "quant_golden.npz"), **out)


def make_store(rng):
    cases = []
    for case in range(24):
        bt = int(rng.choice([32, 128]))
        nb = int(rng.integers(1, 160))
        ntok = nb * bt - int(rng.integers(0, bt))
        budget = int(rng.integers(1, 48))
        sink = int(rng.integers(0, 3))
        recent = int(rng.integers(0, 3))
        if sink + recent > budget:
            sink, recent = 0, 0
        imm = bool(case % 3 == 2)
        cfg = dict(block_tokens=bt, select_budget=budget * bt, sink_blocks=sink,
                   recent_blocks=recent, optimize_stage_in=bool(case % 5 != 4),
                   immutable_source_k=imm, immutable_refresh_remaps=2 if imm else 8,
                   immutable_refresh_abs_delta_tokens=(bt * 16 if imm else 262144),
                   immutable_max_baked_position=262144)
        R = O.RefStore(**cfg)
        R.register_append(ntok)
        n = R.block_count()
        steps = []
        for step in range(5):
            scores = rng.standard_normal(n)
            if step % 2 == 1:
                scores = np.round(scores * 2) / 2       # many exact ties
            mand = rng.integers(0, n + 2, size=int(rng.integers(0, 4))).astype(np.uint32)
            R.set_retrieval_scores(scores)
            sel = R.pick_topk_blocks(mand)
            plan = R.set_selection(sel)
            for b in plan.stage_out:
                R.set_block_tier(int(b), O.TIER_CPU, int(b), -1)
            for b in plan.stage_in:
                R.set_block_tier(int(b), O.TIER_GPU, -1, -1)
            steps.append(dict(
                scores=scores.tolist(), mandatory=mand.tolist(), selected=sel.tolist(),
                stage_in=plan.stage_in.tolist(), stage_out=plan.stage_out.tolist(),
                rm_block_id=plan.rm_block_id.tolist(), rm_from_base=plan.rm_from_base.tolist(),
                rm_to_base=plan.rm_to_base.tolist(), rm_skip=plan.rm_skip.tolist(),
                rm_raw_refresh=plan.rm_raw_refresh.tolist(),
                rm_working_k_resident=plan.rm_working_k_resident.tolist(),
                counters=list(plan.counters())))
        cases.append(dict(cfg=cfg, n_tokens=ntok, steps=steps))
    with open(os.path.join(HERE, "store_golden.json"), "w") as f:
        json.dump(dict(source="kvmem::KvMemStore compiled from CrKcel/kvmem-llama.cpp kvmem/",
                       cases=cases), f, separators=(",", ":"))


def make_meank(rng):
    E, L, bt = 64, 2, 32
    count = 2 * bt + 7
    vals = np.array([1e7, .125, -1e7, .3, -7.1, .001, 9.7], dtype=np.float32)
    k = np.empty((count, E), dtype=np.float32)
    for t in range(count):
        for d in range(E):
            k[t, d] = vals[(t + d) % 7]
    k2 = rng.standard_normal((count, E)).astype(np.float32)
    raw = O.RefRaw(L, E, bt)
    raw.write_layer_mean_k(0, k, 0)
    raw.write_layer_mean_k(0, k2, 1)
    nb = (count + bt - 1) // bt
    means = np.stack([np.stack([raw.mean_k(b, il) for b in range(nb)]) for il in range(L)])
    np.savez_compressed(os.path.join(HERE, "meank_golden.npz"), k0=k, k1=k2, means=means,
                        block_tokens=bt)


if __name__ == "__main__":
    O.build(ref=True)
    if not O.have_ref():
        sys.exit("oracle/_ref/libkvmem_ref.so missing: needs the reference tree")
    rng = np.random.default_rng(20261201)
    make_quant(rng)
    make_store(rng)
    make_meank(rng)
    print("golden fixtures written to", HERE)
