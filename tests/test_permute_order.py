"""The streaming permute's move order, modelled on the CPU.

permute_chain_kernel (csrc/kvm_stagein.cu) copies each (layer, K|V, piece)
stream's moves in this order: moves to a lower slot in list order (the diff
emits them by ascending new slot), then moves to a higher slot in reverse,
with loads running kChainStages - 1 moves ahead of the stores.  It does so
only when the move list is monotone (old and new slots both strictly
increasing), which the chronological layout guarantees; otherwise it takes
the order-free column path.  This test replays that exact event sequence on
slot contents for random chronological layouts from the oracle's `layout`
and checks that every load still sees the bytes the slot held before the
step and that the result equals snapshot semantics (new[to] = old[from])."""
import numpy as np
import pytest

STAGES = 4          # kChainStages


def _stream_order(moves):
    left = [m for m in moves if m[2] < m[1]]
    right = [m for m in moves if m[2] > m[1]][::-1]
    return left + right


def _monotone(moves):
    f, t = moves[:, 1], moves[:, 2]
    return bool(np.all(np.diff(f) > 0) and np.all(np.diff(t) > 0))


def _replay(moves, mem, stages=STAGES):
    """Loads and stores in the kernel's order; returns (memory, clean) where
    clean is False when a load saw a slot an earlier store had overwritten."""
    order = _stream_order([tuple(int(x) for x in m) for m in moves])
    orig = mem.copy()
    buf = {}
    clean = True

    def load(j):
        nonlocal clean
        _, frm, _ = order[j]
        if mem[frm] != orig[frm]:
            clean = False
        buf[j] = mem[frm]

    issued = 0
    while issued < min(stages - 1, len(order)):
        load(issued)
        issued += 1
    for i in range(len(order)):
        _, _, to = order[i]
        mem[to] = buf.pop(i)
        if issued < len(order):
            load(issued)
            issued += 1
    return mem, clean


def _random_step(rng, oracle, n_blocks, budget):
    prev = np.sort(rng.choice(n_blocks, size=budget, replace=False)).astype(np.uint32)
    slot_before = np.full(n_blocks, -1, np.int32)
    slot_before[prev] = np.arange(budget)            # chronological window
    keep = rng.random(budget) < rng.uniform(0.3, 0.95)
    fresh = rng.choice(np.setdiff1d(np.arange(n_blocks), prev), size=budget - int(keep.sum()),
                       replace=False)
    sel = np.sort(np.concatenate([prev[keep], fresh])).astype(np.uint32)
    return oracle.layout(sel, slot_before)


@pytest.mark.parametrize("seed", range(40))
def test_stream_order_reads_before_writes(oracle, seed):
    rng = np.random.default_rng(seed)
    n_blocks, budget = int(rng.integers(40, 400)), int(rng.integers(4, 40))
    _, moves, _ = _random_step(rng, oracle, n_blocks, budget)
    if moves.shape[0] == 0:
        return
    assert _monotone(moves)                          # what the kernel checks first
    slots = budget + 8
    mem = np.arange(slots) + 1000                    # slot s holds value 1000 + s
    want = mem.copy()
    for _, frm, to in moves:
        want[to] = mem[frm]                          # snapshot semantics
    for stages in (2, STAGES, 8):
        got, clean = _replay(moves, mem.copy(), stages)
        assert clean, (seed, stages)
        assert np.array_equal(got, want), (seed, stages)


def test_unordered_list_needs_the_column_path():
    """A swap of two slots is not monotone: streamed, its second load would
    see a slot the first store already overwrote, which is why such lists
    (kvm_set_block_gpu_slot can create them) take the column path."""
    moves = np.array([[7, 1, 0], [9, 0, 1]])
    assert not _monotone(moves)
    mem = np.array([100, 101, 102])
    got, clean = _replay(moves, mem.copy(), stages=1 + 1)
    assert not clean or not np.array_equal(got, [101, 100, 102])
