"""Device producers of the scorer's statistics (kvm_write_mean_k,
kvm_meank_add/flush, kvm_summarize, kvm_query_add) against the reference's own
kvmem::RawKvStore (a committed golden sequence) and the oracle restatement,
bit for bit: F32 / F16 / BF16 captures, contiguous and strided ggml views,
writes that start mid-block, decode flushes, masked query tokens."""
import numpy as np
import pytest

from kvm_testlib import load_meank_seq

pytestmark = pytest.mark.gpu


def _session(kvm, L, H, D, HQ, T, max_blocks):
    cfg = kvm.default_config(block_tokens=T, select_budget=4 * T, gen_reserve=T, sink_blocks=1,
                             n_layer=L, n_head_kv=H, head_dim=D, n_head_q=HQ,
                             max_blocks=max_blocks, type_k=8, type_v=8)
    return kvm.Session(cfg, 0)


def _sums(sess, L, nb):
    out = [sess.download_summaries(l, 0, nb) for l in range(L)]
    return np.stack([o[0] for o in out]), np.stack([o[1] for o in out])


def test_meank_sequence_matches_reference_golden(kvm_lib, oracle):
    """Replays the reference RawKvStore sequence: uneven prefill writes across
    block edges, decode sums flushed mid-block and at block starts."""
    import torch
    ops, g = load_meank_seq()
    L, E, T = int(g["n_layer"]), int(g["n_embd"]), int(g["block_tokens"])
    H, D = 2, E // 2
    nb = g["means"].shape[1]
    s = _session(kvm_lib, L, H, D, 2 * H, T, nb + 3)
    try:
        for op in ops:
            if op[0] == "k":
                rows = torch.from_numpy(op[3]).cuda()
                s.write_mean_k(op[1], op[2], rows.shape[0], kvm_lib.rows_of(rows, H, D))
            else:
                acc = torch.from_numpy(op[4][None, :].copy()).cuda()   # 0 + sum == sum
                s.meank_add(op[1], 0, 1, kvm_lib.rows_of(acc, H, D))
                s.meank_flush(op[2], op[3], layer0=op[1], n_layers=1)
        sums, cnt = _sums(s, L, nb)
        for il in range(L):
            for b in range(nb):
                got = oracle.mean_k(sums[il, b], int(cnt[il, b])) if cnt[il, b] else np.zeros(E, np.float32)
                assert got.tobytes() == g["means"][il, b].tobytes(), (il, b)
    finally:
        s.close()


def _views(torch, x, H, D):
    """The same [n, H*D] F32 values as captured tensors of every layout:
    contiguous, head-major storage permuted to [n, H, D], and a channel-strided
    view (every other element of a wider buffer)."""
    n = x.shape[0]
    out = {"contig": x.view(n, H, D)}
    hm = x.view(n, H, D).permute(1, 0, 2).contiguous()           # storage [H, n, D]
    out["head_major"] = hm.permute(1, 0, 2)
    wide = torch.zeros((n, H, 2 * D), dtype=x.dtype, device=x.device)
    wide[:, :, ::2] = x.view(n, H, D)
    out["dim_strided"] = wide[:, :, ::2]
    return out


@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
def test_write_mean_k_types_and_layouts(kvm_lib, oracle, dtype):
    import torch
    L, H, D, T = 2, 4, 64, 32
    E = H * D
    n_tok = 3 * T + 19
    nb = (n_tok + T - 1) // T
    rng = np.random.default_rng(7)
    tdt = getattr(torch, dtype)
    for layout in ("contig", "head_major", "dim_strided"):
        s = _session(kvm_lib, L, H, D, 2 * H, T, nb + 2)
        ms = oracle.MeanStore(L, nb + 2, E, T)
        try:
            for il in range(L):
                x = torch.from_numpy(rng.standard_normal((n_tok, E)).astype(np.float32) * 8).cuda()
                x = x.to(tdt)
                xf = x.float().cpu().numpy()
                v = _views(torch, x, H, D)[layout]
                pos = 0
                for n in (T - 3, 5, T + 7, n_tok):         # batches that cross block edges
                    n = min(n, n_tok - pos)
                    if n <= 0:
                        break
                    s.write_mean_k(il, pos, n, kvm_lib.rows_of(v[pos:pos + n], H, D))
                    ms.write_layer_mean_k(pos, xf[pos:pos + n], il)
                    pos += n
            sums, cnt = _sums(s, L, nb)
            assert np.array_equal(cnt, ms.mean_tok[:, :nb]), layout
            assert sums.tobytes() == ms.sums[:, :nb].tobytes(), layout
        finally:
            s.close()


def test_decode_meank_accumulate_and_flush(kvm_lib, oracle):
    """Prefill harvest, then decode tokens one and three at a time into the
    per-layer accumulators, flushed when the block fills (decode_mean_commit)."""
    import torch
    L, H, D, T = 2, 2, 64, 32
    E = H * D
    prefill, total = 45, 45 + 2 * T + 11
    nb = (total + T - 1) // T
    rng = np.random.default_rng(9)
    s = _session(kvm_lib, L, H, D, 2 * H, T, nb + 1)
    ms = oracle.MeanStore(L, nb + 1, E, T)
    try:
        k = torch.from_numpy(rng.standard_normal((L, total, E)).astype(np.float32)).cuda().half()
        kf = k.float().cpu().numpy()
        for il in range(L):
            s.write_mean_k(il, 0, prefill, kvm_lib.rows_of(k[il, :prefill], H, D))
            ms.write_layer_mean_k(0, kf[il, :prefill], il)
        pos, run0, run_n = prefill, prefill, 0
        while pos < total:
            n = min(1 if pos % 2 else 3, total - pos, T - pos % T)
            for il in range(L):
                # the ubatch holds 4 tokens; the committed ones start at index 1
                ub = torch.zeros((4, E), dtype=torch.float16, device="cuda")
                ub[1:1 + n] = k[il, pos:pos + n]
                s.meank_add(il, 1, n, kvm_lib.rows_of(ub, H, D))
            run_n += n
            pos += n
            if (run0 % T) + run_n >= T or pos == total:
                s.meank_flush(run0, run_n)
                for il in range(L):
                    ms.write_layer_mean_sum(run0, run_n, il,
                                            oracle.add_rows(np.zeros(E, np.float32),
                                                            kf[il, run0:run0 + run_n]))
                run0, run_n = pos, 0
        sums, cnt = _sums(s, L, nb)
        assert np.array_equal(cnt, ms.mean_tok[:, :nb])
        assert sums.tobytes() == ms.sums[:, :nb].tobytes()
    finally:
        s.close()


@pytest.mark.parametrize("pad", [0, 2])
def test_summarize_vector_and_scalar_paths(kvm_lib, oracle, pad):
    """kvm_summarize on an aligned source (16-byte lanes) and on rows padded by
    one F16 (scalar lanes); partial last block."""
    import torch
    L, H, D, T, B = 2, 4, 64, 32, 21
    E = H * D
    rng = np.random.default_rng(3 + pad)
    s = _session(kvm_lib, L, H, D, 2 * H, T, B + 3)
    try:
        row = E + pad
        h = torch.from_numpy(oracle.synth_f16(rng, (L, B, T, row), row)).cuda()
        s.register_append(B * T - 5)
        src = kvm_lib.make_source(h.data_ptr(), h.data_ptr(), B * T * row * 2, T * row * 2, row * 2)
        s.summarize(src)
        sums, cnt = _sums(s, L, B)
        hn = h.cpu().numpy()
        for l in range(L):
            for b in range(B):
                nt = T if b < B - 1 else T - 5
                assert cnt[l, b] == nt
                want = oracle.block_sum_f16(np.ascontiguousarray(hn[l, b, :nt, :E]))
                assert sums[l, b].tobytes() == want.tobytes(), (l, b)
    finally:
        s.close()


def test_query_accumulation_scores_match_oracle(kvm_lib, oracle):
    """query_reset + masked query_add per layer (BF16 and F32 captures), then
    the scores of summaries produced on the device -- bit-exact against the
    oracle scorer run on the oracle's accumulated q_sum / q_count.  Layer 2
    gets no query and must not vote."""
    import torch
    L, H, D, HQ, T, B = 3, 2, 64, 6, 16, 40
    E = H * D
    rng = np.random.default_rng(21)
    s = _session(kvm_lib, L, H, D, HQ, T, B + 2)
    try:
        k = torch.from_numpy(oracle.synth_f16(rng, (L, B * T, E), E)).cuda()
        s.register_append(B * T)
        ms = oracle.MeanStore(L, B, E, T)
        for il in range(L):
            s.write_mean_k(il, 0, B * T, kvm_lib.rows_of(k[il], H, D))
            ms.write_layer_mean_k(0, k[il].float().cpu().numpy(), il)
        q_sum = np.zeros((L, HQ * D), np.float32)
        q_cnt = np.zeros(L, np.uint32)
        s.query_reset()
        for il in range(2):
            for dt, n in ((torch.bfloat16, 5), (torch.float32, 3)):
                q = torch.from_numpy(oracle.synth_f16(rng, (n, HQ * D), HQ * D).astype(np.float32))
                q = q.cuda().to(dt)
                keep = rng.integers(0, 2, n).astype(np.uint8)
                keep[0] = 1
                s.query_add(il, n, kvm_lib.rows_of(q.view(n, HQ, D), HQ, D), keep=keep)
                qf = q.float().cpu().numpy()
                q_sum[il] = oracle.add_rows(q_sum[il], qf[keep.astype(bool)])
                q_cnt[il] += int(keep.sum())
        s.score()
        got = s.scores()
        want = oracle.score(ms.sums, ms.mean_tok, np.ones(B, np.uint8), q_sum, q_cnt, H, HQ, D)
        assert got.tobytes() == want.tobytes()
        # a reset query leaves every block at 0 (no layer votes)
        s.query_reset()
        s.score()
        assert not np.any(s.scores())
    finally:
        s.close()


def test_producer_argument_checks(kvm_lib):
    import torch
    s = _session(kvm_lib, 1, 2, 64, 4, 16, 4)
    try:
        x = torch.zeros((4, 128), dtype=torch.float16, device="cuda")
        with pytest.raises(kvm_lib.KvmError):
            s.write_mean_k(0, 60, 8, kvm_lib.rows_of(x, 2, 64))      # beyond max_blocks
        with pytest.raises(kvm_lib.KvmError):
            s.write_mean_k(1, 0, 4, kvm_lib.rows_of(x, 2, 64))       # layer out of range
        with pytest.raises(kvm_lib.KvmError):
            s.meank_add(0, 0, 4, kvm_lib.rows_of(x, 4, 64))          # wrong width
        with pytest.raises(kvm_lib.KvmError):
            s.query_add(0, 4, kvm_lib.rows_of(x, 2, 64))             # Q width is 4*64
        bad = kvm_lib.rows_of(x, 2, 64)
        bad.type = 8                                                 # q8_0 is no capture type
        with pytest.raises(kvm_lib.KvmError):
            s.meank_add(0, 0, 1, bad)
    finally:
        s.close()
