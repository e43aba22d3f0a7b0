"""Parity at BASELINE.json's full sizes (configs 1-4), through the C ABI.

config 1 (1 layer, 2048 blocks): everything against the CPU oracle -- every
score, the selection, every window byte of the 256 staged blocks.

configs 2-4 (16 layers, up to 8192 blocks) through size-independent properties:
  * summaries: sampled (layer, block) sums equal the oracle's ordered F16 token sum;
  * scores: all of them bit-exact against the oracle run on the read-back summaries;
  * selection and chronological layout (moves / cold lists): exact;
  * window: sampled slots -- moved ones included -- hold exactly the oracle's
    quantization of their block's F16 rows.
Config 4 runs 40 incremental steps with overlapping selections (no reset).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

T, HKV, D, HQ = 128, 4, 256, 24
E = HKV * D


def _history(torch, L, B, seed, dev):
    """Seeded N(0,1) F16 [L, B, T, E] with 1% of the channels of each layer x20."""
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(2):
        h = torch.empty((L, B, T, E), dtype=torch.float16, device=dev)
        for l in range(L):
            ch = torch.from_numpy(rng.choice(E, size=E // 100, replace=False)).to(dev)
            x = torch.randn((B, T, E), generator=g, device=dev, dtype=torch.float32)
            x[:, :, ch] *= 20.0
            h[l].copy_(x.to(torch.float16))
            del x
        out.append(h)
    return out


class Full:
    def __init__(self, kvm, torch, L, B, type_k, type_v, gen_reserve=16384, seed=0):
        self.torch, self.kvm = torch, kvm
        self.L, self.B = L, B
        dev = torch.device("cuda", 0)
        self.hk, self.hv = _history(torch, L, B, seed, dev)
        cfg = kvm.default_config(block_tokens=T, select_budget=32768, gen_reserve=gen_reserve,
                                 sink_blocks=1, n_layer=L, n_head_kv=HKV, head_dim=D,
                                 n_head_q=HQ, max_blocks=B, type_k=type_k, type_v=type_v)
        self.s = kvm.Session(cfg, 0)
        self.src = kvm.make_source(self.hk.data_ptr(), self.hv.data_ptr(), B * T * E * 2,
                                   T * E * 2, E * 2)
        self.s.register_append(B * T)
        self.s.summarize(self.src)
        self.tk, self.tv = type_k, type_v
        self.rbk, self.rbv = kvm.row_bytes(type_k, E), kvm.row_bytes(type_v, E)
        self.wk = torch.zeros((L, self.s.n_slots * T * self.rbk), dtype=torch.uint8, device=dev)
        self.wv = torch.zeros((L, self.s.n_slots * T * self.rbv), dtype=torch.uint8, device=dev)
        self.sums = None

    def close(self):
        self.s.close()
        del self.hk, self.hv, self.wk, self.wv
        self.torch.cuda.empty_cache()

    def read_summaries(self, oracle, rng, n_check=8):
        sums = np.empty((self.L, self.B, E), np.float32)
        cnt = np.empty((self.L, self.B), np.uint32)
        for l in range(self.L):
            sums[l], cnt[l] = self.s.download_summaries(l)
        assert np.all(cnt == T)
        for _ in range(n_check):
            l, b = int(rng.integers(self.L)), int(rng.integers(self.B))
            want = oracle.block_sum_f16(self.hk[l, b].cpu().numpy())
            assert sums[l, b].tobytes() == want.tobytes(), (l, b)
        self.sums, self.cnt = sums, cnt
        return sums

    def step(self, q, qc, reset=True):
        if reset:
            self.s.reset_window()
        self.s.set_query(q, qc)
        self.s.step(self.src, [self.wk[l].data_ptr() for l in range(self.L)],
                    [self.wv[l].data_ptr() for l in range(self.L)])
        return self.s.plan()

    def check_slots(self, oracle, sel, slots, rng, layers_per_slot=2):
        for i in slots:
            b = int(sel[i])
            for l in rng.choice(self.L, size=min(layers_per_slot, self.L), replace=False):
                l = int(l)
                k = oracle.quantize_rows_f16(self.tk, self.hk[l, b].cpu().numpy(), n_threads=8)
                v = oracle.quantize_rows_f16(self.tv, self.hv[l, b].cpu().numpy(), n_threads=8)
                gk = self.wk[l, i * T * self.rbk:(i + 1) * T * self.rbk].cpu().numpy()
                gv = self.wv[l, i * T * self.rbv:(i + 1) * T * self.rbv].cpu().numpy()
                assert np.array_equal(gk, k.ravel()), ("K", l, i, b)
                assert np.array_equal(gv, v.ravel()), ("V", l, i, b)


def _query(rng, L):
    import oracle as O
    return O.synth_f16(rng, (L, HQ * D), D).astype(np.float32)


def test_config1_everything_vs_oracle(kvm_lib, oracle):
    import torch
    f = Full(kvm_lib, torch, 1, 2048, 8, 8, seed=1)
    try:
        rng = np.random.default_rng(2)
        sums = f.read_summaries(oracle, rng)
        q = _query(rng, 1)
        qc = np.ones(1, np.uint32)
        p = f.step(q, qc)
        scores = oracle.score(sums, f.cnt, np.ones(2048, np.uint8), q, qc, HKV, HQ, D, n_threads=8)
        assert f.s.scores().tobytes() == scores.tobytes()
        sel = oracle.pick_topk(oracle.make_cfg(T, 256, 1, 0), scores)
        assert np.array_equal(p["selected"], sel) and sel.size == 256
        assert np.array_equal(p["cold_to"], np.arange(256)) and p["mv_block"].size == 0
        f.check_slots(oracle, sel, range(256), rng, layers_per_slot=1)
    finally:
        f.close()


@pytest.mark.parametrize("tk,tv,gen", [(8, 8, 16384), (8, 2, 16384), (6, 6, 12288)])
def test_config2_3_sixteen_layers(kvm_lib, oracle, tk, tv, gen):
    import torch
    f = Full(kvm_lib, torch, 16, 2048, tk, tv, gen_reserve=gen, seed=3)
    try:
        rng = np.random.default_rng(4)
        sums = f.read_summaries(oracle, rng)
        q = _query(rng, 16)
        qc = np.ones(16, np.uint32)
        p = f.step(q, qc)
        scores = oracle.score(sums, f.cnt, np.ones(2048, np.uint8), q, qc, HKV, HQ, D, n_threads=16)
        assert f.s.scores().tobytes() == scores.tobytes()
        sel = oracle.pick_topk(oracle.make_cfg(T, 256, 1, 0), scores)
        assert np.array_equal(p["selected"], sel)
        assert f.s.n_slots == (32768 + gen) // T
        f.check_slots(oracle, sel, rng.choice(256, size=24, replace=False), rng)
    finally:
        f.close()


def test_config4_incremental_40_steps(kvm_lib, oracle):
    import torch
    B, L = 8192, 16
    f = Full(kvm_lib, torch, L, B, 8, 8, seed=5)
    try:
        rng = np.random.default_rng(6)
        sums = f.read_summaries(oracle, rng)
        qc = np.ones(L, np.uint32)
        cfg = oracle.make_cfg(T, 256, 1, 0)
        slots = np.full(B, -1, np.int32)
        q = _query(rng, L)
        alpha = 0.94
        overlaps, moved_total = [], 0
        prev = None
        for step in range(40):
            if step:
                noise = _query(rng, L)
                q = (alpha * q + np.sqrt(1 - alpha * alpha) * noise).astype(np.float16).astype(np.float32)
            p = f.step(q, qc, reset=False)
            scores = oracle.score(sums, f.cnt, np.ones(B, np.uint8), q, qc, HKV, HQ, D, n_threads=16)
            assert f.s.scores().tobytes() == scores.tobytes(), step
            sel = oracle.pick_topk(cfg, scores)
            assert np.array_equal(p["selected"], sel), step
            slot_after, moves, cold = oracle.layout(sel, slots)
            got_mv = np.stack([p["mv_block"], p["mv_from"], p["mv_to"]], 1).astype(np.int64)
            assert np.array_equal(got_mv, moves.astype(np.int64)), step
            got_cold = np.stack([p["cold_block"], p["cold_to"]], 1).astype(np.int64)
            assert np.array_equal(got_cold, cold.astype(np.int64)), step
            slots = slot_after
            if prev is not None:
                overlaps.append(len(np.intersect1d(prev, sel)) / sel.size)
            moved_total += moves.shape[0]
            sample = list(rng.choice(256, size=6, replace=False))
            sample += [int(t) for t in moves[:4, 2]] + [int(t) for t in cold[:2, 1]]
            f.check_slots(oracle, sel, sample, rng, layers_per_slot=1)
            prev = sel
        mean_overlap = float(np.mean(overlaps))
        print(f"config 4: mean selection overlap {mean_overlap:.3f}, moved blocks {moved_total}")
        assert 0.3 < mean_overlap < 0.98 and moved_total > 0
    finally:
        f.close()
