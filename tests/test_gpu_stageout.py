"""Stage-out (harvest) of packed window rows through kvm_stageout: every
resident block's K and V rows of every layer, bit for bit equal to its window
slot and to the oracle's quantization of its F16 rows; non-resident and
out-of-range ids flagged and skipped.  Device, pinned-host and pageable-host
destinations; the HBM ring wrapping over many chunks; the byte-copy path for
rows that are not 16-byte multiples; a partial trailing block."""
import numpy as np
import pytest

from kvm_testlib import Shape, make_query, make_rig

pytestmark = pytest.mark.gpu


def _run_step(rig, seed):
    rng = np.random.default_rng(seed)
    q, qc = make_query(rig.shape, rng)
    rig.sess.set_query(q, qc)
    rig.sess.step(rig.src, rig.k_bases(), rig.v_bases())
    return rig.sess.plan()["selected"]


def _check_items(rig, oracle, ids, out, resident, sel):
    s = rig.shape
    L, T, E = s.n_layer, s.block_tokens, s.n_embd
    rbk, rbv = oracle.row_bytes(s.type_k, E), oracle.row_bytes(s.type_v, E)
    item = L * T * (rbk + rbv)
    assert rig.sess.stageout_item_bytes == item
    slot_of = {int(b): i for i, b in enumerate(sel)}
    wk, wv = rig.win_k.cpu().numpy(), rig.win_v.cpu().numpy()
    for j, b in enumerate(ids):
        b = int(b)
        want_res = b in slot_of
        assert resident[j] == (1 if want_res else 0), (j, b)
        if not want_res:
            continue
        slot = slot_of[b]
        nt = int(rig.n_tok[b])
        for l in range(L):
            base = j * item + l * T * (rbk + rbv)
            gk = out[base:base + nt * rbk]
            gv = out[base + T * rbk:base + T * rbk + nt * rbv]
            assert np.array_equal(gk, wk[l, slot * T * rbk:slot * T * rbk + nt * rbk]), ("K", j, l)
            assert np.array_equal(gv, wv[l, slot * T * rbv:slot * T * rbv + nt * rbv]), ("V", j, l)
            if l == 0:
                qk = oracle.quantize_rows_f16(s.type_k, rig.k_np[l, b, :nt]).ravel()
                assert np.array_equal(gk, qk), ("K oracle", j)


@pytest.mark.parametrize("dest", ["device", "pinned", "pageable"])
def test_stageout_resident_blocks(kvm_lib, oracle, dest):
    import torch
    shape = Shape(n_layer=3, n_blocks=40, block_tokens=32, n_head_kv=2, head_dim=128, n_head_q=6,
                  budget_blocks=12, gen_blocks=4, type_k=8, type_v=2, partial_tokens=19)
    rig = make_rig(shape, seed=11)
    try:
        sel = _run_step(rig, 12)
        # every selected block, two unselected ones, an id past block_count, repeats
        ids = list(sel[::-1]) + [int(np.setdiff1d(np.arange(40), sel)[0]), 39, 1000, int(sel[2])]
        n = len(ids)
        item = rig.sess.stageout_item_bytes
        if dest == "device":
            buf = torch.zeros(n * item, dtype=torch.uint8, device="cuda")
        elif dest == "pinned":
            buf = torch.zeros(n * item, dtype=torch.uint8).pin_memory()
        else:
            buf = np.zeros(n * item, np.uint8)
        res = rig.sess.stageout(ids, rig.k_bases(), rig.v_bases(), buf, want_resident=True)
        out = buf.cpu().numpy() if hasattr(buf, "cpu") else buf
        _check_items(rig, oracle, ids, out, res, sel)
    finally:
        rig.sess.close()


def test_stageout_ring_wraps_over_many_chunks(kvm_lib, oracle):
    """A staging ring of 4 slots x 2 blocks: 24 blocks take 12 chunks and wrap
    three times."""
    import torch
    shape = Shape(n_layer=2, n_blocks=48, block_tokens=32, n_head_kv=2, head_dim=64, n_head_q=4,
                  budget_blocks=24, gen_blocks=2, type_k=8, type_v=8)
    item = 2 * 32 * 2 * 136
    rig = make_rig(shape, seed=13, staging_bytes=4 * 2 * item)
    try:
        sel = _run_step(rig, 14)
        ids = list(sel)
        buf = torch.zeros(len(ids) * item, dtype=torch.uint8).pin_memory()
        res = rig.sess.stageout(ids, rig.k_bases(), rig.v_bases(), buf, want_resident=True)
        _check_items(rig, oracle, ids, buf.numpy(), res, sel)
        # the same window staged out twice in a row on one stream gives the same bytes
        buf2 = torch.zeros_like(buf)
        rig.sess.stageout(ids, rig.k_bases(), rig.v_bases(), buf2)
        rig.sess.wait()
        assert torch.equal(buf, buf2)
    finally:
        rig.sess.close()


def test_stageout_unaligned_rows_byte_path(kvm_lib, oracle):
    # E = 96: q8_0 rows of 102 bytes are not 16-byte multiples
    import torch
    shape = Shape(n_layer=2, n_blocks=20, block_tokens=16, n_head_kv=3, head_dim=32, n_head_q=6,
                  budget_blocks=6, gen_blocks=2, type_k=8, type_v=6)
    rig = make_rig(shape, seed=15)
    try:
        sel = _run_step(rig, 16)
        ids = list(sel) + [int(np.setdiff1d(np.arange(20), sel)[0])]
        for dev in (True, False):
            item = rig.sess.stageout_item_bytes
            buf = torch.zeros(len(ids) * item, dtype=torch.uint8, device="cuda" if dev else "cpu")
            if not dev:
                buf = buf.pin_memory()
            res = rig.sess.stageout(ids, rig.k_bases(), rig.v_bases(), buf, want_resident=True)
            _check_items(rig, oracle, ids, buf.cpu().numpy(), res, sel)
    finally:
        rig.sess.close()


def test_stageout_argument_checks(kvm_lib):
    import torch
    shape = Shape(n_layer=1, n_blocks=8, block_tokens=16, n_head_kv=2, head_dim=64, n_head_q=4,
                  budget_blocks=4, gen_blocks=1)
    rig = make_rig(shape, seed=1)
    try:
        buf = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
        with pytest.raises(kvm_lib.KvmError):
            rig.sess.stageout(np.zeros(100, np.uint32), rig.k_bases(), rig.v_bases(), buf)  # > max_blocks
        rig.sess.stageout([], rig.k_bases(), rig.v_bases(), buf)                            # no-op
    finally:
        rig.sess.close()
