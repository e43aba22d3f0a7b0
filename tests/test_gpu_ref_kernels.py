"""The CPU oracle against the reference's own stage-in device kernels.

fwht_kernel<N>, quant_q8_0, quant_q4_0 and rope_neox_kernel of
src/adapter/llama-kvmem-stagein.cu are compiled unchanged from that file, with
nvcc's default floating point as the reference builds it, by oracle/Makefile
into oracle/_ref/libstagein_ref.so (oracle/ref_stagein.cu holds the launch
wrappers).  Since the device transform path equals the oracle bit for bit
(tests/test_gpu_transform.py), these comparisons pin it to the reference's
GPU code as well:

  * the Walsh-Hadamard transform: bit-exact for every size the reference
    launches (64, 128, 256, 512);
  * q8_0: bit-exact;
  * q4_0: nvcc contracts the kernel's `x*id + 8.5f` into one fused
    multiply-add, so on a few blocks per ten thousand its codes differ from
    ggml's quantize_row_q4_0_ref, which rounds the product first.  This
    library follows ggml (the bytes llama.cpp's CPU path writes; gguf-py
    fixtures pin them); the test checks that every block on which the two
    disagree is exactly the fused computation;
  * NeoX RoPE: the kernel's sincosf and contracted rotation agree with the
    oracle's host sin/cos within 1e-6 of the row's largest magnitude.
"""
import ctypes as C
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(os.path.dirname(HERE), "oracle", "_ref", "libstagein_ref.so")
needs_ref = pytest.mark.skipif(not os.path.exists(LIB),
                               reason="reference stage-in kernels not built (oracle/Makefile ref)")


def _lib():
    L = C.CDLL(LIB)
    L.ref_cuda_fwht.argtypes = [C.c_void_p, C.c_int64, C.c_int, C.c_void_p]
    L.ref_cuda_quantize.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p]
    L.ref_cuda_rope_neox.argtypes = [C.c_void_p, C.c_int64, C.c_int, C.c_int, C.c_int, C.c_int32,
                                     C.c_void_p, C.c_void_p]
    return L


def _rows(oracle, rng, n, e):
    return oracle.synth_f16(rng, (n, e), e).astype(np.float32)


def _ref_fwht(L, torch, x, nrot):
    d = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    assert L.ref_cuda_fwht(d.data_ptr(), x.size // nrot, nrot, None) == 0
    torch.cuda.synchronize()
    return d.cpu().numpy()


def _ref_quant(L, torch, type_id, x):
    bs = {8: 34, 2: 18}[type_id]
    nb = x.size // 32
    dx = torch.from_numpy(np.ascontiguousarray(x, np.float32).ravel()).cuda()
    dy = torch.zeros(nb * bs, dtype=torch.uint8, device="cuda")
    assert L.ref_cuda_quantize(type_id, dx.data_ptr(), dy.data_ptr(), nb, None) == 0
    torch.cuda.synchronize()
    return dy.cpu().numpy().reshape(nb, bs)


@needs_ref
@pytest.mark.parametrize("nrot", [64, 128, 256, 512])
def test_fwht_equals_reference_kernel(oracle, nrot):
    import torch
    x = _rows(oracle, np.random.default_rng(nrot), 2048, nrot)
    got = _ref_fwht(_lib(), torch, x, nrot)
    assert got.tobytes() == oracle.fwht_rows(x, nrot).tobytes()


@needs_ref
def test_q8_0_equals_reference_kernel(oracle):
    import torch
    L = _lib()
    rng = np.random.default_rng(80)
    for x in (_rows(oracle, rng, 1024, 1024), oracle.fwht_rows(_rows(oracle, rng, 1024, 1024), 256)):
        got = _ref_quant(L, torch, 8, x)
        assert np.array_equal(got, oracle.quantize(8, x.ravel()).reshape(got.shape))


def _q4_0_fused(blk):
    """quant_q4_0 of one block with x*id + 8.5f as one fused multiply-add
    (the exact product plus 8.5, rounded once to float)."""
    a = np.abs(blk)
    vmax = blk[int(np.argmax(a))] if a.max() > 0 else np.float32(0)   # first largest magnitude
    d = np.float32(vmax * np.float32(-0.125))
    idv = np.float32(np.float32(1.0) / d) if d != 0 else np.float32(0)
    t = (blk.astype(np.float64) * np.float64(idv) + 8.5).astype(np.float32)
    q = np.minimum(15, np.trunc(t).astype(np.int64))
    nib = ((q[:16] & 15) | ((q[16:] & 15) << 4)).astype(np.uint8)
    return np.concatenate([np.array([d], np.float32).astype(np.float16).view(np.uint8), nib])


@needs_ref
def test_q4_0_reference_kernel_differs_only_by_its_fused_multiply_add(oracle):
    import torch
    L = _lib()
    rng = np.random.default_rng(40)
    n_diff = 0
    n_blocks = 0
    for x in (_rows(oracle, rng, 1024, 1024), oracle.fwht_rows(_rows(oracle, rng, 1024, 1024), 256)):
        got = _ref_quant(L, torch, 2, x)
        want = oracle.quantize(2, x.ravel()).reshape(got.shape)
        bad = np.flatnonzero(np.any(got != want, axis=1))
        blocks = x.reshape(-1, 32)
        for b in bad:
            assert np.array_equal(got[b], _q4_0_fused(blocks[b])), b
        n_diff += bad.size
        n_blocks += got.shape[0]
    assert n_diff <= n_blocks // 1000


@needs_ref
@pytest.mark.parametrize("pos0", [0, 131000])
def test_rope_reference_kernel_within_sincos_tolerance(oracle, pos0):
    import torch
    L = _lib()
    H, D, n_rot = 4, 256, 256
    theta = oracle.rope_theta(n_rot, 1e6)
    x = _rows(oracle, np.random.default_rng(pos0 + 1), 256, H * D)
    dx = torch.from_numpy(x.copy()).cuda()
    dth = torch.from_numpy(theta.copy()).cuda()
    assert L.ref_cuda_rope_neox(dx.data_ptr(), x.shape[0], H, D, n_rot, pos0, dth.data_ptr(), None) == 0
    torch.cuda.synchronize()
    got = dx.cpu().numpy()
    want = oracle.rope_neox_rows(x, H, D, n_rot, pos0, theta)
    tol = 1e-6 * np.abs(want).max(axis=1, keepdims=True)
    assert np.all(np.abs(got - want) <= tol)
