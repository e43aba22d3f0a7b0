"""The task decoders' division by a launch-constant d (FastDiv,
csrc/kvm_internal.cuh): floor(t * ceil(2^32 / d) / 2^32) == floor(t / d)
whenever t * d <= 2^32, the bound the stage-in and copy kernels check before
they take that path.  Exhaustive over small divisors near the bound,
random elsewhere, and the decoders' (item, layer, K|V, tile) split on launch
shapes of the benchmark configs."""
import numpy as np


def fast_div(t, d):
    m = ((1 << 32) + d - 1) // d
    return (t * m) >> 32


def test_fast_div_exact_within_bound():
    rng = np.random.default_rng(3)
    for d in list(range(1, 300)) + [511, 512, 513, 4095, 4096, 65535, 65536, 1 << 20, (1 << 31) + 11]:
        tmax = (1 << 32) // d                     # t * d <= 2^32
        ts = {0, 1, tmax, max(0, tmax - 1)}
        ts.update(int(x) for x in rng.integers(0, tmax + 1, 2000))
        # every t around multiples of d near the top of the range
        for k in (tmax // 2, tmax // 3):
            base = (k // d) * d if d < tmax else k
            ts.update(range(max(0, base - 3), min(tmax, base + 3) + 1))
        for t in ts:
            assert fast_div(t, d) == t // d, (t, d)


def test_fast_div_can_fail_past_bound():
    """The bound matters: d = 3 (m*d = 2^32 + 2) gives a wrong quotient for
    t = 2^31 (remainder 2, error term 1/3), where t * d > 2^32."""
    d = 3
    t = 1 << 31
    assert t % d == 2 and t * d > 1 << 32
    assert fast_div(t, d) != t // d
    assert all(fast_div(u, d) == u // d for u in range((1 << 32) // d - 100, (1 << 32) // d + 1))


def test_task_split_matches_division():
    for n_items, n_layer, n_kv, tiles in [(256, 16, 2, 16), (2048, 16, 2, 16), (8192, 16, 2, 16),
                                          (37, 3, 2, 5), (1, 1, 1, 1), (1000, 7, 1, 13)]:
        per_layer = n_kv * tiles
        per_item = n_layer * per_layer
        total = n_items * per_item
        assert total * per_item <= 1 << 32
        t = np.arange(total, dtype=np.uint64)

        def fd(x, d):
            return (x * np.uint64(((1 << 32) + d - 1) // d)) >> np.uint64(32)

        item = fd(t, per_item)
        r = t - item * np.uint64(per_item)
        layer = fd(r, per_layer)
        r2 = r - layer * np.uint64(per_layer)
        kv = fd(r2, tiles)
        tile = r2 - kv * np.uint64(tiles)
        assert np.array_equal(item, t // np.uint64(per_item))
        assert np.array_equal(layer, (t % np.uint64(per_item)) // np.uint64(per_layer))
        assert np.array_equal(kv, (t % np.uint64(per_layer)) // np.uint64(tiles))
        assert np.array_equal(tile, t % np.uint64(tiles))
