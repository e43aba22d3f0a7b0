"""Generate the golden fixtures in this directory.

Run in a container that has the reference tree (for oracle/_ref) and gguf-py:

    python tests/golden/make_golden.py

Outputs (all small, committed):
  quant_golden.npz   seeded F16 rows + the q8_0 / q4_0 / q5_0 bytes gguf-py 0.19.0
                     produces for them (third-party oracle of ggml's quantizers)
  store_golden.json  selection + KvMemPlan sequences produced by the reference's own
                     kvmem::KvMemStore (oracle/_ref/libkvmem_ref.so)
  meank_golden.npz   means produced by the reference's own kvmem::RawKvStore
  meank_seq_golden.npz  a prefill + decode sequence on kvmem::RawKvStore: uneven
                     write_layer_mean_k batches across block edges (prefill
                     harvest), then decode sums flushed with write_layer_mean_sum
                     from mid-block and block-start positions; the means after it

  groups_golden.json  pick_semantic_groups selections of the reference's own
                     kvmem::KvMemStore for seeded random spans, scores, pins
  rope_golden.npz    F32 rows rotated by the reference's own kvmem::rope_neox_apply
                     (full and partial rotary dims, small and 256K-range positions)
  score_golden.npz   block scores from the reference adapter's own
                     llama_memory_kvmem::score_retrieval (oracle/ref_score.cpp) for
                     seeded summaries and queries: GQA 6:1, query heads not a multiple
                     of the KV heads, layers without query or statistics, partial
                     blocks, zero and large sums

`python tests/golden/make_golden.py meank_seq` regenerates only the named fixtures.
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


def meank_seq_ops(rng, L, E, bt):
    """The operation list of meank_seq_golden: ("k", il, pos0, rows) for
    write_layer_mean_k and ("s", il, pos0, n, sum) for write_layer_mean_sum."""
    ops = []
    prefill = 2 * bt + 9                    # ends mid-block
    for il in range(L):
        k = rng.standard_normal((prefill, E)).astype(np.float32) * 4
        k[:, rng.choice(E, 3, replace=False)] *= 20
        pos = 0
        for n in (5, bt - 5 + 3, 17, prefill):   # uneven batches across block edges
            n = min(n, prefill - pos)
            if n <= 0:
                break
            ops.append(("k", il, pos, k[pos:pos + n]))
            pos += n
    # decode: sums of the tokens after the prefill, flushed when the block fills,
    # then one full block from its start, then a partial block
    pos = prefill
    for n in (bt - prefill % bt, bt, 7):
        for il in range(L):
            rows = rng.standard_normal((n, E)).astype(np.float32)
            ops.append(("s", il, pos, n, O.add_rows(np.zeros(E, np.float32), rows)))
        pos += n
    return ops, pos


def make_meank_seq(rng):
    L, E, bt = 2, 64, 16
    ops, end = meank_seq_ops(rng, L, E, bt)
    raw = O.RefRaw(L, E, bt)
    for op in ops:
        if op[0] == "k":
            raw.write_layer_mean_k(op[2], op[3], op[1])
        else:
            raw.write_layer_mean_sum(op[2], op[3], op[1], op[4])
    nb = (end + bt - 1) // bt
    means = np.stack([np.stack([raw.mean_k(b, il) for b in range(nb)]) for il in range(L)])
    arrays = dict(means=means, block_tokens=bt, n_layer=L, n_embd=E, n_ops=len(ops))
    for i, op in enumerate(ops):
        if op[0] == "k":
            arrays[f"op{i}"] = np.array([0, op[1], op[2], op[3].shape[0]], np.int64)
            arrays[f"rows{i}"] = op[3]
        else:
            arrays[f"op{i}"] = np.array([1, op[1], op[2], op[3]], np.int64)
            arrays[f"rows{i}"] = op[4][None, :]
    np.savez_compressed(os.path.join(HERE, "meank_seq_golden.npz"), **arrays)


ROPE_CASES = (   # n_head, head_dim, n_rot, pos0, freq_base, freq_scale
    (2, 128, 128, 0, 1e6, 1.0),
    (4, 256, 256, 131000, 1e6, 1.0),
    (2, 128, 64, 262100, 1e4, 0.25),
)


def make_rope(rng):
    arrays = {}
    for i, (H, D, n_rot, pos0, base, scale) in enumerate(ROPE_CASES):
        x = rng.standard_normal((4, H * D)).astype(np.float32) * 3
        arrays[f"x{i}"] = x
        arrays[f"out{i}"] = O.ref_rope_neox(x, H, D, n_rot, pos0, base, scale)
        arrays[f"case{i}"] = np.array([H, D, n_rot, pos0, base, scale], np.float64)
    np.savez_compressed(os.path.join(HERE, "rope_golden.npz"), n_cases=len(ROPE_CASES), **arrays)


def groups_case(rng):
    """One seeded pick_semantic_groups case (config, spans, scores, pins)."""
    T = int(rng.choice([16, 32, 64, 128]))
    n = int(rng.integers(1, 160))
    cfg = dict(block_tokens=T, budget_blocks=int(rng.integers(0, n + 5)),
               sink_blocks=int(rng.integers(0, 4)), recent_blocks=int(rng.integers(0, 4)))
    total = n * T - int(rng.integers(0, T))
    G = int(rng.integers(0, 48))
    b0 = rng.integers(0, total + 3 * T, G)
    spans = np.stack([b0, b0 + rng.integers(-5, 6 * T, G)], 1).clip(0).astype(np.uint32)
    if rng.integers(0, 3) == 0:
        scores = rng.choice([0.0, -0.0, 1.0, 2.0], G)          # ties, signed zeros
    else:
        scores = rng.standard_normal(G)
    mand = rng.integers(0, n + 3, int(rng.integers(0, 5))).astype(np.uint32)
    return cfg, total, spans, scores, mand


def make_groups(rng):
    cases = []
    for _ in range(80):
        cfg, total, spans, scores, mand = groups_case(rng)
        rs = O.RefStore(block_tokens=cfg["block_tokens"],
                        select_budget=cfg["budget_blocks"] * cfg["block_tokens"],
                        sink_blocks=cfg["sink_blocks"], recent_blocks=cfg["recent_blocks"])
        rs.register_append(total)
        sel = rs.pick_semantic_groups(spans, scores, mand)
        cases.append(dict(cfg=cfg, total_tokens=total, spans=spans.tolist(),
                          scores=[float(x) for x in scores], signbits=[bool(np.signbit(x)) for x in scores],
                          mandatory=mand.tolist(), selected=sel.tolist()))
    with open(os.path.join(HERE, "groups_golden.json"), "w") as f:
        json.dump(dict(source="kvmem::KvMemStore::pick_semantic_groups compiled from CrKcel/kvmem-llama.cpp kvmem/",
                       cases=cases), f, separators=(",", ":"))


SCORE_CASES = (   # n_layer, n_blocks, n_head_kv, n_head_q, head_dim, block_tokens, q_count
    (3, 40, 4, 24, 64, 128, (1, 2, 0)),
    (2, 33, 2, 5, 80, 32, (1, 3)),
    (1, 20, 1, 1, 256, 16, (1,)),
)


def score_case(rng, L, B, Hkv, Hq, D, T, qc):
    """Summaries, counts and query sums of one scorer case."""
    E = Hkv * D
    # K sums as F16 values (what a block sum of F16 rows looks like in scale)
    sums = (rng.standard_normal((L, B, E)) * 40).astype(np.float16).astype(np.float32)
    cnt = rng.integers(1, T + 1, (L, B)).astype(np.uint32)
    cnt[:, 0] = T
    cnt[:, 1] = 0                    # a block without statistics in any layer
    cnt[0, 2] = 0                    # statistics missing in one layer only
    sums[cnt == 0] = 0.0
    sums[:, 3] = 0.0                 # statistics present, all-zero sums
    sums[0, 4] *= 1000.0             # large sums
    q = rng.standard_normal((L, Hq * D)).astype(np.float16).astype(np.float32)
    return sums, cnt, q, np.array(qc, np.uint32)


def make_score(rng):
    arrays = {}
    for i, (L, B, Hkv, Hq, D, T, qc) in enumerate(SCORE_CASES):
        sums, cnt, q, qcount = score_case(rng, L, B, Hkv, Hq, D, T, qc)
        arrays[f"sums{i}"] = sums
        arrays[f"cnt{i}"] = cnt
        arrays[f"q{i}"] = q
        arrays[f"qc{i}"] = qcount
        arrays[f"shape{i}"] = np.array([L, B, Hkv, Hq, D, T], np.uint32)
        arrays[f"scores{i}"] = O.ref_score(sums, cnt, q, qcount, Hkv, Hq, D, T)
    np.savez_compressed(os.path.join(HERE, "score_golden.npz"), n_cases=len(SCORE_CASES), **arrays)


if __name__ == "__main__":
    O.build(ref=True)
    if not O.have_ref():
        sys.exit("oracle/_ref/libkvmem_ref.so missing: needs the reference tree")
    only = set(sys.argv[1:])
    if not only or only & {"quant", "store", "meank"}:
        rng = np.random.default_rng(20261201)
        make_quant(rng)
        make_store(rng)
        make_meank(rng)
    if not only or "meank_seq" in only:
        make_meank_seq(np.random.default_rng(20261202))
    if not only or "rope" in only:
        make_rope(np.random.default_rng(20261203))
    if not only or "groups" in only:
        make_groups(np.random.default_rng(20261204))
    if not only or "score" in only:
        make_score(np.random.default_rng(20261205))
    print("golden fixtures written to", HERE)
