"""The failure path on the GPU without a fault: a stage-in whose first tile
is never loaded (kvm_test_inject) lets that CTA's bounded mbarrier waits run
out; the launch drains its other copies and returns, kvm_wait reports
KVM_EDEVICE with the wait-timeout flag and clears it, and the same session
then runs a correct step."""
import numpy as np
import pytest

from kvm_testlib import OracleModel, Shape, make_query, make_rig

pytestmark = pytest.mark.gpu


def test_stagein_wait_timeout_reported_then_recovers(kvm_lib, oracle):
    shape = Shape(n_layer=2, n_blocks=48, block_tokens=32, budget_blocks=10, gen_blocks=2)
    rig = make_rig(shape, seed=31)
    rng = np.random.default_rng(32)
    q, qc = make_query(shape, rng)
    s = rig.sess
    s.set_query(q, qc)
    s.test_inject(kvm_lib.TEST_SKIP_TILE_LOAD)
    s.step(rig.src, rig.k_bases(), rig.v_bases())
    with pytest.raises(kvm_lib.KvmError) as err:
        s.wait()
    assert err.value.status == kvm_lib.KVM_EDEVICE
    assert "wait-timeout" in str(err.value)
    s.wait()                                    # the flags were cleared
    # the hook was one-shot: a cold step on the same session is correct again
    s.reset_window()
    om = OracleModel(rig)
    s.set_query(q, qc)
    s.step(rig.src, rig.k_bases(), rig.v_bases())
    _, sel, _, _, _ = om.step(q, qc)
    assert np.array_equal(s.plan()["selected"], sel)
    mk, mv = om.window_valid_mask()
    assert np.array_equal(rig.win_k.cpu().numpy()[:, mk], om.win_k[:, mk])
    assert np.array_equal(rig.win_v.cpu().numpy()[:, mv], om.win_v[:, mv])
    s.wait()


def test_test_inject_rejects_unknown_flags(kvm_lib):
    shape = Shape(n_layer=1, n_blocks=8, block_tokens=32, budget_blocks=4, gen_blocks=1)
    rig = make_rig(shape, seed=1)
    with pytest.raises(kvm_lib.KvmError):
        rig.sess.test_inject(0x80)


def test_odd_window_base_rejected_before_launch(kvm_lib, oracle):
    """A window layer base that is not 2-byte aligned would reach 2-byte
    device stores; kvm_stagein returns KVM_EINVAL before anything launches,
    and the same plan then stages into the aligned window bit-exactly."""
    shape = Shape(n_layer=2, n_blocks=24, block_tokens=32, budget_blocks=6, gen_blocks=2)
    rig = make_rig(shape, seed=41)
    om = OracleModel(rig)
    q, qc = make_query(shape, np.random.default_rng(42))
    s = rig.sess
    s.set_query(q, qc)
    s.score()
    s.select()
    s.diff()
    kb = rig.k_bases()
    bad = list(kb)
    bad[1] = bad[1] + 1
    launches = s.kernel_launches
    with pytest.raises(kvm_lib.KvmError) as err:
        s.stagein(rig.src, bad, rig.v_bases())
    assert err.value.status == kvm_lib.KVM_EINVAL
    assert "2-byte aligned" in str(err.value)
    assert s.kernel_launches == launches
    s.stagein(rig.src, kb, rig.v_bases())
    _, sel, _, _, _ = om.step(q, qc)
    assert np.array_equal(s.plan()["selected"], sel)
    mk, mv = om.window_valid_mask()
    assert np.array_equal(rig.win_k.cpu().numpy()[:, mk], om.win_k[:, mk])
    assert np.array_equal(rig.win_v.cpu().numpy()[:, mv], om.win_v[:, mv])
