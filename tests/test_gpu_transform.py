"""Stage-in transform mode (kvm_set_transform) against the oracle: the
attn_rot Walsh-Hadamard transform before quantization bit for bit, for every
head size and window type; NeoX RoPE at the original positions within the
last-bit differences of CUDA's sincosf and the host's cosf / sinf."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

L = 2


class TRig:
    def __init__(self, kvm, torch, oracle, H, D, T, B, tk, tv, seed, host=False, budget_blocks=8):
        self.kvm, self.torch, self.O = kvm, torch, oracle
        self.H, self.D, self.T, self.B, self.tk, self.tv = H, D, T, B, tk, tv
        E = self.E = H * D
        rng = np.random.default_rng(seed)
        self.hk_np = oracle.synth_f16(rng, (L, B, T, E), E)
        self.hv_np = oracle.synth_f16(rng, (L, B, T, E), E)
        if host:
            self.hk = torch.from_numpy(self.hk_np).pin_memory()
            self.hv = torch.from_numpy(self.hv_np).pin_memory()
        else:
            self.hk = torch.from_numpy(self.hk_np).cuda()
            self.hv = torch.from_numpy(self.hv_np).cuda()
        cfg = kvm.default_config(block_tokens=T, select_budget=budget_blocks * T, gen_reserve=2 * T,
                                 sink_blocks=1,
                                 n_layer=L, n_head_kv=H, head_dim=D, n_head_q=2 * H,
                                 max_blocks=B + 4, type_k=tk, type_v=tv)
        self.s = kvm.Session(cfg, 0)
        self.s.register_append(B * T)
        loc = kvm.LOC_HOST if host else kvm.LOC_DEVICE
        self.src = kvm.make_source(self.hk.data_ptr(), self.hv.data_ptr(), B * T * E * 2, T * E * 2,
                                   E * 2, location=loc)
        sums = np.stack([[oracle.block_sum_f16(self.hk_np[l, b]) for b in range(B)] for l in range(L)])
        for l in range(L):
            self.s.upload_summaries(l, 0, sums[l], np.full(B, T, np.uint32))
        self.rbk, self.rbv = kvm.row_bytes(tk, E), kvm.row_bytes(tv, E)
        n = self.s.n_slots
        self.wk = torch.zeros((L, n * T * self.rbk), dtype=torch.uint8, device="cuda")
        self.wv = torch.zeros((L, n * T * self.rbv), dtype=torch.uint8, device="cuda")
        q = oracle.synth_f16(rng, (L, 2 * H * D), D).astype(np.float32)
        self.s.set_query(q, np.ones(L, np.uint32))

    def step(self):
        self.s.reset_window()
        self.s.step(self.src, [self.wk[l].data_ptr() for l in range(L)],
                    [self.wv[l].data_ptr() for l in range(L)])
        p = self.s.plan()
        assert np.array_equal(p["cold_to"], np.arange(p["selected"].size))
        return p["selected"]

    def window(self, kv, l, slot):
        w, rb = (self.wv, self.rbv) if kv else (self.wk, self.rbk)
        return w[l, slot * self.T * rb:(slot + 1) * self.T * rb].cpu().numpy().reshape(self.T, rb)

    def close(self):
        self.s.close()


def _deq_q8(b):
    blk = b.reshape(b.shape[0], -1, 34)
    d = blk[:, :, :2].copy().view(np.float16).astype(np.float32)
    q = blk[:, :, 2:].view(np.int8).astype(np.float32)
    return (d * q).reshape(b.shape[0], -1), np.repeat(d[:, :, 0], 32, axis=1)


CASES = [  # H, D, T, B, type_k, type_v
    (2, 128, 32, 24, 8, 8),
    (4, 64, 16, 24, 2, 6),
    (2, 256, 32, 20, 6, 8),
    (2, 192, 32, 20, 8, 2),
    (1, 512, 16, 20, 8, 8),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"H{c[0]}D{c[1]}k{c[4]}v{c[5]}")
def test_attn_rot_stagein_bit_exact(kvm_lib, oracle, case):
    import torch
    H, D, T, B, tk, tv = case
    r = TRig(kvm_lib, torch, oracle, H, D, T, B, tk, tv, seed=D + tk)
    try:
        rot_k, rot_v = kvm_lib.attn_rot_nrot(tk, D, True), kvm_lib.attn_rot_nrot(tv, D, False)
        assert rot_k and rot_v == 64
        r.s.set_transform(rot_k=rot_k, rot_v=rot_v)
        sel = r.step()
        for slot in range(sel.size):
            b = int(sel[slot])
            for l in range(L):
                k = oracle.transform_quantize_rows(tk, r.hk_np[l, b], H, D, nrot=rot_k)
                v = oracle.transform_quantize_rows(tv, r.hv_np[l, b], H, D, nrot=rot_v)
                assert np.array_equal(r.window(0, l, slot), k), ("K", slot, l)
                assert np.array_equal(r.window(1, l, slot), v), ("V", slot, l)
        # switching the transform off gives the plain quantizer again
        r.s.clear_transform()
        sel = r.step()
        b = int(sel[1])
        assert np.array_equal(r.window(0, 0, 1), oracle.quantize_rows_f16(tk, r.hk_np[0, b]))
    finally:
        r.close()


@pytest.mark.parametrize("tk,tv", [(8, 2), (6, 6)])
def test_attn_rot_many_values(kvm_lib, oracle, tk, tv):
    """About 25M values through the attn_rot stage-in: a product rounded
    together with the following add (a contracted multiply-add) changes a
    q4_0 / q5_0 code a few times per million values, so this size catches it."""
    import torch
    H, D, T, B = 4, 256, 128, 56
    r = TRig(kvm_lib, torch, oracle, H, D, T, B, tk, tv, seed=31 + tk, budget_blocks=48)
    try:
        rot_k, rot_v = kvm_lib.attn_rot_nrot(tk, D, True), kvm_lib.attn_rot_nrot(tv, D, False)
        r.s.set_transform(rot_k=rot_k, rot_v=rot_v)
        sel = r.step()
        assert sel.size >= 40
        for l in range(L):
            got_k = r.wk[l, :sel.size * T * r.rbk].cpu().numpy().reshape(sel.size, T, r.rbk)
            got_v = r.wv[l, :sel.size * T * r.rbv].cpu().numpy().reshape(sel.size, T, r.rbv)
            for slot in range(sel.size):
                b = int(sel[slot])
                k = oracle.transform_quantize_rows(tk, r.hk_np[l, b], H, D, nrot=rot_k)
                v = oracle.transform_quantize_rows(tv, r.hv_np[l, b], H, D, nrot=rot_v)
                assert np.array_equal(got_k[slot], k), ("K", slot, l)
                assert np.array_equal(got_v[slot], v), ("V", slot, l)
    finally:
        r.close()


def test_attn_rot_stagein_from_host_source(kvm_lib, oracle):
    import torch
    H, D, T, B = 2, 128, 32, 24
    r = TRig(kvm_lib, torch, oracle, H, D, T, B, 8, 2, seed=77, host=True)
    try:
        r.s.set_transform(rot_k=128, rot_v=64)
        sel = r.step()
        for slot in (0, 3, sel.size - 1):
            b = int(sel[slot])
            k = oracle.transform_quantize_rows(8, r.hk_np[1, b], H, D, nrot=128)
            v = oracle.transform_quantize_rows(2, r.hv_np[1, b], H, D, nrot=64)
            assert np.array_equal(r.window(0, 1, slot), k)
            assert np.array_equal(r.window(1, 1, slot), v)
    finally:
        r.close()


@pytest.mark.parametrize("n_rope,base,rot", [(128, 1e6, 128), (64, 1e4, 0)])
def test_rope_then_rot_stagein(kvm_lib, oracle, n_rope, base, rot):
    """K = quantize(Hadamard(RoPE(k, block_id*T + t))), q8_0: every value within
    half a quantization step of the oracle's pre-quantization value -- plus the
    grid shift of the F16-rounded scale (127 * |d - f16(d)| <= 127 * 2^-11 d)
    and the sincosf last-bit slack -- and nearly all bytes identical."""
    import torch
    H, D, T, B = 2, 128, 128, 24
    r = TRig(kvm_lib, torch, oracle, H, D, T, B, 8, 8, seed=5)
    try:
        r.s.set_transform(rot_k=rot, rot_v=64, rope_n_rot=n_rope, rope_freq_base=base)
        th = oracle.rope_theta(n_rope, base)
        sel = r.step()
        same = total = 0
        for slot in range(sel.size):
            b = int(sel[slot])
            l = slot % L
            want, pre = oracle.transform_quantize_rows(8, r.hk_np[l, b], H, D, nrot=rot, n_rope=n_rope,
                                                       pos0=b * T, theta=th, pre_quant=True)
            got = r.window(0, l, slot)
            deq, d = _deq_q8(got)
            bound = 0.5 * d + 127.0 * 2.0 ** -11 * d + 1e-5 * np.abs(pre) + 1e-6
            assert np.all(np.abs(deq - pre) <= bound), slot
            same += int(np.count_nonzero(got == want))
            total += got.size
            # V has no RoPE: bit-exact Hadamard
            v = oracle.transform_quantize_rows(8, r.hv_np[l, b], H, D, nrot=64)
            assert np.array_equal(r.window(1, l, slot), v)
        assert same / total > 0.995, same / total
    finally:
        r.close()


def test_rope_only_f16_window(kvm_lib, oracle):
    import torch
    H, D, T, B = 2, 64, 32, 24
    r = TRig(kvm_lib, torch, oracle, H, D, T, B, 1, 1, seed=8)
    try:
        r.s.set_transform(rope_n_rot=64, rope_freq_base=1e6)
        th = oracle.rope_theta(64, 1e6)
        sel = r.step()
        for slot in (0, 5, sel.size - 1):
            b = int(sel[slot])
            want = oracle.rope_neox_rows(r.hk_np[0, b].astype(np.float32), H, D, 64, b * T, th)
            got = r.window(0, 0, slot).view(np.float16).astype(np.float32)
            assert np.allclose(got, want, rtol=2 ** -10, atol=1e-6), slot
            # V untouched: plain F16 copy
            assert np.array_equal(r.window(1, 0, slot).view(np.float16), r.hv_np[0, b])
    finally:
        r.close()


def test_set_transform_checks(kvm_lib, oracle):
    import torch
    r = TRig(kvm_lib, torch, oracle, 2, 64, 16, 12, 1, 8, seed=1)
    try:
        with pytest.raises(kvm_lib.KvmError):
            r.s.set_transform(rot_k=64)               # K window is F16: no attn_rot
        with pytest.raises(kvm_lib.KvmError):
            r.s.set_transform(rot_v=128)              # does not divide head_dim 64
        with pytest.raises(kvm_lib.KvmError):
            r.s.set_transform(rot_v=96)
        with pytest.raises(kvm_lib.KvmError):
            r.s.set_transform(rope_n_rot=32)          # RoPE dims in multiples of 64
        r.s.set_transform(rot_v=64)
        r.s.clear_transform()
    finally:
        r.close()
