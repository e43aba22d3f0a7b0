"""kvm_stagein_packed: the reference's stage-in of already-quantized rows
(write_block_to_gpu -> kvmem_stagein_enqueue_v / flush) against the oracle
window model, from device and pinned-host sources, through incremental steps
with moves, and the round trip kvm_stageout -> kvm_stagein_packed."""
import numpy as np
import pytest

from kvm_testlib import OracleModel, Shape, make_query, make_rig

pytestmark = pytest.mark.gpu


def _packed_history(oracle, rig):
    """Every block's rows quantized by the oracle, in the stage-out item layout
    (block b at item b): [B][L][K rows T*rbk | V rows T*rbv]."""
    s = rig.shape
    L, B, T, E = s.n_layer, s.n_blocks, s.block_tokens, s.n_embd
    rbk, rbv = oracle.row_bytes(s.type_k, E), oracle.row_bytes(s.type_v, E)
    out = np.zeros((B, L, T * (rbk + rbv)), np.uint8)
    for b in range(B):
        nt = int(rig.n_tok[b])
        for l in range(L):
            qk = oracle.quantize_rows_f16(s.type_k, rig.k_np[l, b, :nt]).ravel()
            qv = oracle.quantize_rows_f16(s.type_v, rig.v_np[l, b, :nt]).ravel()
            out[b, l, :qk.size] = qk
            out[b, l, T * rbk:T * rbk + qv.size] = qv
    return out.reshape(-1)


def _check_window(rig, model):
    mk, mv = model.window_valid_mask()
    wk, wv = rig.win_k.cpu().numpy(), rig.win_v.cpu().numpy()
    assert np.array_equal(wk[:, mk], model.win_k[:, mk])
    assert np.array_equal(wv[:, mv], model.win_v[:, mv])


@pytest.mark.parametrize("where", ["device", "host"])
def test_packed_stagein_incremental_steps(kvm_lib, oracle, where):
    import torch
    shape = Shape(n_layer=2, n_blocks=48, block_tokens=32, n_head_kv=2, head_dim=128, n_head_q=6,
                  budget_blocks=12, gen_blocks=4, type_k=8, type_v=2, partial_tokens=21)
    # a small staging ring (4 slots of 3 blocks) so the host path wraps it
    item = 2 * 32 * (272 + 144)
    rig = make_rig(shape, seed=31, staging_bytes=4 * 3 * item)
    model = OracleModel(rig)
    try:
        packed = _packed_history(oracle, rig)
        buf = torch.from_numpy(packed)
        buf = buf.cuda() if where == "device" else buf.pin_memory()
        src = rig.sess.stageout_source(buf, kvm_lib.LOC_DEVICE if where == "device" else kvm_lib.LOC_HOST)
        rng = np.random.default_rng(32)
        q, qc = make_query(shape, rng)
        for step in range(4):
            if step:
                q = (0.9 * q + 0.45 * make_query(shape, rng)[0]).astype(np.float16).astype(np.float32)
            rig.sess.set_query(q, qc)
            rig.sess.score()
            rig.sess.select()
            rig.sess.diff()
            rig.sess.stagein_packed(src, rig.k_bases(), rig.v_bases())
            p = rig.sess.plan()
            _, sel, _, moves, cold = model.step(q, qc)
            assert np.array_equal(p["selected"], sel), step
            assert p["mv_block"].size == moves.shape[0] and p["cold_block"].size == cold.shape[0]
            _check_window(rig, model)
    finally:
        rig.sess.close()


def test_stageout_then_packed_stagein_round_trip(kvm_lib, oracle):
    """Blocks quantized by the F16 stage-in, harvested with kvm_stageout,
    staged back from those packed rows into an emptied window: same bytes."""
    import torch
    shape = Shape(n_layer=3, n_blocks=40, block_tokens=32, n_head_kv=2, head_dim=128, n_head_q=6,
                  budget_blocks=10, gen_blocks=2, type_k=6, type_v=8)
    rig = make_rig(shape, seed=41)
    try:
        rng = np.random.default_rng(42)
        q, qc = make_query(shape, rng)
        rig.sess.set_query(q, qc)
        rig.sess.step(rig.src, rig.k_bases(), rig.v_bases())
        sel = rig.sess.plan()["selected"]
        before_k, before_v = rig.win_k.clone(), rig.win_v.clone()
        ids = np.arange(shape.n_blocks, dtype=np.uint32)   # item b = block b
        item = rig.sess.stageout_item_bytes
        harvest = torch.zeros(shape.n_blocks * item, dtype=torch.uint8).pin_memory()
        res = rig.sess.stageout(ids, rig.k_bases(), rig.v_bases(), harvest, want_resident=True)
        assert res.sum() == sel.size
        rig.win_k.zero_()
        rig.win_v.zero_()
        rig.sess.reset_window()
        rig.sess.score()
        rig.sess.select()
        rig.sess.diff()
        rig.sess.stagein_packed(rig.sess.stageout_source(harvest, kvm_lib.LOC_HOST), rig.k_bases(),
                                rig.v_bases())
        rig.sess.wait()
        assert np.array_equal(rig.sess.plan()["selected"], sel)
        assert torch.equal(rig.win_k, before_k) and torch.equal(rig.win_v, before_v)
    finally:
        rig.sess.close()


def test_packed_stagein_needs_a_plan(kvm_lib):
    import torch
    shape = Shape(n_layer=1, n_blocks=8, block_tokens=16, n_head_kv=2, head_dim=64, n_head_q=4,
                  budget_blocks=4, gen_blocks=1)
    rig = make_rig(shape, seed=1)
    try:
        buf = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
        with pytest.raises(kvm_lib.KvmError):
            rig.sess.stagein_packed(rig.sess.stageout_source(buf), rig.k_bases(), rig.v_bases())
    finally:
        rig.sess.close()
