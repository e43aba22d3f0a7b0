"""Helpers shared by the GPU parity tests and __graft_entry__.smoke().

Builds a synthetic session (seeded F16 K/V history in HBM, summaries produced
by libkvm's summarize kernel, seeded query) and computes what the reference
would produce for the same inputs with the CPU oracle: scores, selection,
plan, chronological layout and the quantized window bytes.
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field

import numpy as np

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load_meank_seq():
    """The meank_seq_golden operation list -- ("k", il, pos0, rows) for
    write_layer_mean_k and ("s", il, pos0, n, sum) for write_layer_mean_sum --
    and the npz holding the reference RawKvStore's means after it."""
    g = np.load(os.path.join(GOLD, "meank_seq_golden.npz"))
    ops = []
    for i in range(int(g["n_ops"])):
        kind, il, pos0, n = (int(x) for x in g[f"op{i}"])
        rows = g[f"rows{i}"]
        ops.append(("k", il, pos0, rows) if kind == 0 else ("s", il, pos0, n, rows[0]))
    return ops, g


@dataclass
class Shape:
    n_layer: int = 2
    n_blocks: int = 64
    block_tokens: int = 32
    n_head_kv: int = 2
    head_dim: int = 128
    n_head_q: int = 6
    budget_blocks: int = 12
    gen_blocks: int = 4
    sink_blocks: int = 1
    recent_blocks: int = 0
    type_k: int = 8
    type_v: int = 8
    partial_tokens: int = 0        # >0: last block holds this many tokens

    @property
    def n_embd(self):
        return self.n_head_kv * self.head_dim

    @property
    def n_tokens(self):
        full = self.n_blocks * self.block_tokens
        return full - (self.block_tokens - self.partial_tokens if self.partial_tokens else 0)


@dataclass
class Rig:
    shape: Shape
    sess: object
    k_hist: object                 # torch float16 [L, B, T, E] on device
    v_hist: object
    win_k: object                  # torch uint8 [L, slots*T*rb_k]
    win_v: object
    src: object
    n_tok: np.ndarray = field(default=None)

    def k_bases(self):
        return [self.win_k[l].data_ptr() for l in range(self.shape.n_layer)]

    def v_bases(self):
        return [self.win_v[l].data_ptr() for l in range(self.shape.n_layer)]


def make_rig(shape: Shape, seed: int = 0, device: int = 0, outlier_channels=None, **cfg_extra):
    import torch
    import kvm
    import oracle as O
    rng = np.random.default_rng(seed)
    L, B, T, E = shape.n_layer, shape.n_blocks, shape.block_tokens, shape.n_embd
    cfg = kvm.default_config(
        block_tokens=T, select_budget=shape.budget_blocks * T, gen_reserve=shape.gen_blocks * T,
        sink_blocks=shape.sink_blocks, recent_blocks=shape.recent_blocks, n_layer=L,
        n_head_kv=shape.n_head_kv, head_dim=shape.head_dim, n_head_q=shape.n_head_q,
        max_blocks=B + 8, type_k=shape.type_k, type_v=shape.type_v, **cfg_extra)
    sess = kvm.Session(cfg, device)
    dev = torch.device("cuda", device)
    k = O.synth_f16(rng, (L, B, T, E), E, outlier_channels=outlier_channels)
    v = O.synth_f16(rng, (L, B, T, E), E, outlier_channels=outlier_channels)
    k_t = torch.from_numpy(k).to(dev)
    v_t = torch.from_numpy(v).to(dev)
    rbk, rbv = kvm.row_bytes(shape.type_k, E), kvm.row_bytes(shape.type_v, E)
    slots = sess.n_slots
    win_k = torch.zeros((L, slots * T * rbk), dtype=torch.uint8, device=dev)
    win_v = torch.zeros((L, slots * T * rbv), dtype=torch.uint8, device=dev)
    src = kvm.make_source(k_t.data_ptr(), v_t.data_ptr(), B * T * E * 2, T * E * 2, E * 2)
    sess.register_append(shape.n_tokens)
    sess.summarize(src)
    rig = Rig(shape, sess, k_t, v_t, win_k, win_v, src)
    rig.k_np, rig.v_np = k, v
    nt = np.full(B, T, np.uint32)
    if shape.partial_tokens:
        nt[-1] = shape.partial_tokens
    rig.n_tok = nt
    return rig


def make_query(shape: Shape, rng, count=1):
    import oracle as O
    q = O.synth_f16(rng, (shape.n_layer, shape.n_head_q * shape.head_dim), shape.head_dim)
    return q.astype(np.float32), np.full(shape.n_layer, count, np.uint32)


class OracleModel:
    """CPU oracle of one session: block table + window bytes."""

    def __init__(self, rig: Rig):
        import oracle as O
        self.O = O
        s = rig.shape
        self.s = s
        self.cfg = O.make_cfg(s.block_tokens, s.budget_blocks, s.sink_blocks, s.recent_blocks)
        self.blocks = O.Blocks.appended(s.n_tokens, s.block_tokens, tier=O.TIER_CPU)
        L, B, T, E = s.n_layer, s.n_blocks, s.block_tokens, s.n_embd
        # summaries from F16 K (ordered F32 token sums)
        self.sums = np.zeros((L, B, E), np.float32)
        self.cnt = np.zeros((L, B), np.uint32)
        for l in range(L):
            for b in range(B):
                nt = int(rig.n_tok[b])
                self.sums[l, b] = O.block_sum_f16(rig.k_np[l, b, :nt])
                self.cnt[l, b] = nt
        self.has = np.ones(B, np.uint8)
        self.k_np, self.v_np, self.n_tok = rig.k_np, rig.v_np, rig.n_tok
        self.rbk = O.row_bytes(s.type_k, E)
        self.rbv = O.row_bytes(s.type_v, E)
        self.slots = s.budget_blocks + s.gen_blocks
        self.win_k = np.zeros((L, self.slots * T * self.rbk), np.uint8)
        self.win_v = np.zeros((L, self.slots * T * self.rbv), np.uint8)

    def score(self, q, qc):
        s = self.s
        return self.O.score(self.sums, self.cnt, self.has, q, qc, s.n_head_kv, s.n_head_q,
                            s.head_dim)

    def step(self, q, qc, mandatory=()):
        O, s = self.O, self.s
        scores = self.score(q, qc)
        sel = O.pick_topk(self.cfg, scores, mandatory)
        before = self.blocks.gpu_slot.copy()
        plan = O.set_selection(self.cfg, self.blocks, sel)
        slot_after, moves, cold = O.layout(sel, before)
        self.blocks.gpu_slot[:] = slot_after
        dropped = (slot_after < 0)
        self.blocks.tier[dropped & (self.blocks.tier == O.TIER_GPU)] = O.TIER_CPU
        self.blocks.tier[sel] = O.TIER_GPU
        self.apply_window(moves, cold)
        return scores, sel, plan, moves, cold

    def apply_window(self, moves, cold):
        O, s = self.O, self.s
        T = s.block_tokens
        for win, rb in ((self.win_k, self.rbk), (self.win_v, self.rbv)):
            snap = win.copy()
            span = T * rb
            for blk, frm, to in moves:
                nb = int(self.n_tok[blk]) * rb
                win[:, to * span:to * span + nb] = snap[:, frm * span:frm * span + nb]
        for blk, to in cold:
            nt = int(self.n_tok[blk])
            for l in range(s.n_layer):
                qk = O.quantize_rows_f16(s.type_k, self.k_np[l, blk, :nt], n_threads=4)
                qv = O.quantize_rows_f16(s.type_v, self.v_np[l, blk, :nt], n_threads=4)
                self.win_k[l, to * T * self.rbk:to * T * self.rbk + qk.size] = qk.ravel()
                self.win_v[l, to * T * self.rbv:to * T * self.rbv + qv.size] = qv.ravel()

    def window_valid_mask(self):
        """Bytes of window slots that hold a selected block's rows."""
        s = self.s
        T = s.block_tokens
        mk = np.zeros(self.win_k.shape[1], bool)
        mv = np.zeros(self.win_v.shape[1], bool)
        for b in np.nonzero(self.blocks.gpu_slot >= 0)[0]:
            slot = int(self.blocks.gpu_slot[b])
            nt = int(self.n_tok[b])
            mk[slot * T * self.rbk:slot * T * self.rbk + nt * self.rbk] = True
            mv[slot * T * self.rbv:slot * T * self.rbv + nt * self.rbv] = True
        return mk, mv
