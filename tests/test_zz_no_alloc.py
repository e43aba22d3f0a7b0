"""kvm_quantize_rows_noalloc: the quantize entry point for callers that cannot
call cudaMalloc (a caching allocator owns all free HBM, or a latency-critical
loop cannot take the device-wide synchronisation of cudaMalloc/cudaFree).
It must write exactly the bytes of kvm_quantize_rows.  Two calls in a row
check that the shared fixed work array carries nothing from one call into the
next; a call of exactly 16384 row tiles fills the whole array.  Named so
pytest collects it last; it calls the C ABI directly."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _run(kvm, fn, type_id, src, n, E, torch):
    rb = kvm.row_bytes(type_id, E)
    dst = torch.full((n * rb,), 0xA5, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    st = fn(stream, type_id, src.data_ptr(), n, E, dst.data_ptr())
    assert st == kvm.KVM_OK, kvm.lib().kvm_last_error(None)
    torch.cuda.synchronize()
    return dst.cpu().numpy()


@pytest.mark.parametrize("type_id", [8, 2, 6])
def test_noalloc_matches_allocating_entry_point(kvm_lib, oracle, type_id):
    import torch
    L = kvm_lib.lib()
    rng = np.random.default_rng(40 + type_id)
    # first a large call, then a smaller one with another width: the second
    # must not see any of the first call's work list
    for n, E in ((2000, 1024), (37, 256)):
        rows = oracle.synth_f16(rng, (n, E), E)
        src = torch.from_numpy(rows).cuda()
        want = _run(kvm_lib, L.kvm_quantize_rows, type_id, src, n, E, torch)
        got = _run(kvm_lib, L.kvm_quantize_rows_noalloc, type_id, src, n, E, torch)
        assert np.array_equal(got, want), (n, E)
        assert np.array_equal(got.reshape(n, -1), oracle.quantize_rows_f16(type_id, rows))


def test_noalloc_rejects_oversized_calls(kvm_lib):
    import torch
    L = kvm_lib.lib()
    E = 8192                                   # one row per tile
    src = torch.zeros((16, E), dtype=torch.float16, device="cuda")
    dst = torch.zeros(16, dtype=torch.uint8, device="cuda")
    st = L.kvm_quantize_rows_noalloc(0, kvm_lib.TYPE_Q8_0, src.data_ptr(), 16385, E,
                                     dst.data_ptr())
    assert st == kvm_lib.KVM_EINVAL
    assert b"16384 row tiles" in L.kvm_last_error(None)


def test_noalloc_full_array(kvm_lib, oracle):
    """Exactly the array's 16384 row tiles (n_embd 8192: one row a tile), then
    a small call: both equal kvm_quantize_rows byte for byte."""
    import torch
    L = kvm_lib.lib()
    rng = np.random.default_rng(77)
    for n, E in ((16384, 8192), (5, 1024)):
        rows = oracle.synth_f16(rng, (n, E), E)
        src = torch.from_numpy(rows).cuda()
        want = _run(kvm_lib, L.kvm_quantize_rows, kvm_lib.TYPE_Q8_0, src, n, E, torch)
        got = _run(kvm_lib, L.kvm_quantize_rows_noalloc, kvm_lib.TYPE_Q8_0, src, n, E, torch)
        assert np.array_equal(got, want), (n, E)
        del src
    torch.cuda.empty_cache()
