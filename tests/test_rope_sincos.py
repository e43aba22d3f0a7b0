"""The RoPE angle table's sin / cos (`rope_sincos`, csrc/kvm_stagein.cu),
emulated on the host operation by operation -- double-precision FMAs and
single-precision FMAs rounded exactly through fractions -- and held to
CUDA's documented bound for sinf / cosf: within 2 ulp of the true value.
The angles are those of the RoPE stage-in: float(pos) * theta_i rounded to
float, theta_i = base^(-2i/n_rot) (rope_neox_apply, kvmem/src/host/rope.cpp),
positions up to 2^21, plus angles next to multiples of pi/2 and zero.  The
GPU stage-in's RoPE output is checked against the host cosf / sinf in
tests/test_gpu_transform.py."""
import math
from fractions import Fraction

import numpy as np

P1 = float.fromhex("0x1.921fb54442d18p+0")
P2 = float.fromhex("0x1.1a62633145c07p-54")
TWO_OVER_PI = float.fromhex("0x1.45f306dc9c883p-1")


def _f32(fr):
    """Fraction -> nearest float32 (ties to even), without double rounding."""
    f = np.float32(float(fr))
    cands = (np.nextafter(f, np.float32(-np.inf)), f, np.nextafter(f, np.float32(np.inf)))
    return min(cands, key=lambda g: (abs(Fraction(float(g)) - fr), int(np.array(g).view(np.uint32)) & 1))


def _fmaf(a, b, c):
    return _f32(Fraction(float(a)) * Fraction(float(b)) + Fraction(float(c)))


def _fma(a, b, c):
    return float(Fraction(a) * Fraction(b) + Fraction(c))      # correctly rounded double


def rope_sincos(x):
    """The device function, step by step (x: float32)."""
    xd = float(x)
    k = float(np.rint(np.float64(xd) * np.float64(TWO_OVER_PI)))
    rd = _fma(-k, P2, _fma(-k, P1, xd))
    r = np.float32(rd)
    r2 = np.float32(r * r)
    c = {n: np.float32(1.0 / n) for n in (6, 120, 5040, 362880, 24, 720, 40320, 3628800)}
    ps = _fmaf(r2, c[362880], -c[5040])
    ps = _fmaf(ps, r2, c[120])
    ps = _fmaf(ps, r2, -c[6])
    s = _fmaf(ps, np.float32(r2 * r), r)
    pc = _fmaf(r2, -c[3628800], c[40320])
    pc = _fmaf(pc, r2, -c[720])
    pc = _fmaf(pc, r2, c[24])
    pc = _fmaf(pc, r2, np.float32(-0.5))
    co = _fmaf(pc, r2, np.float32(1.0))
    q = int(k) & 3
    s1, c1 = (co, s) if q & 1 else (s, co)
    return (-s1 if q & 2 else s1), (-c1 if (q + 1) & 2 else c1)


def _ulp_err(got, true):
    t = np.float32(true)
    ulp = float(np.spacing(np.abs(t))) if t != 0 else float(np.spacing(np.float32(0)))
    return abs(float(got) - true) / ulp


def _angles(n, seed):
    rng = np.random.default_rng(seed)
    out = [np.float32(0.0), np.float32(1e-30), np.float32(math.pi / 4), np.float32(math.pi / 2)]
    for k in (1, 2, 3, 7, 100, 1000, 12345, 98765, 333333, 1 << 20):
        x = np.float32(k * math.pi / 2)
        out += [np.nextafter(x, np.float32(0)), x, np.nextafter(x, np.float32(np.inf))]
    for base in (1e4, 1e6):
        th = np.power(np.float32(base), -2.0 * np.arange(128, dtype=np.float32) / np.float32(256)).astype(np.float32)
        pos = rng.integers(0, 1 << 21, n // 2).astype(np.float32)
        i = rng.integers(0, 128, n // 2)
        out += list((pos * th[i]).astype(np.float32))
    return out


def test_rope_sincos_within_two_ulp():
    worst = 0.0
    for x in _angles(1600, 7):
        s, c = rope_sincos(x)
        worst = max(worst, _ulp_err(s, math.sin(float(x))), _ulp_err(c, math.cos(float(x))))
    assert worst <= 2.0, worst


def test_rope_sincos_quadrants():
    for k in range(-8, 9):
        x = np.float32(k * math.pi / 2 + 0.3)
        s, c = rope_sincos(x)
        assert abs(float(s) - math.sin(float(x))) < 1e-6
        assert abs(float(c) - math.cos(float(x))) < 1e-6
