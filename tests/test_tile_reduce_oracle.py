"""The oracle's tile reductions (no counterpart in the reference) against
the order and semantics include/simtgo_b200.h states, restated a second
time here in plain Python (float32 by numpy scalars) for small cases, plus
known answers for the edge values: NaN, signed zeros, infinities, ties and
empty input. Parity unpinned: the reference has no reductions to compare
with; these pin the oracle to the library's own statement."""
import numpy as np
import pytest

import oracle_lib as O

F = np.float32
NAN_BITS = 0x7FC00000


def _bits(v):
    return int(np.array(v, np.float32).view(np.uint32))


def _py_sum(x):
    """The header's summation order, independently: blocks of 2048 padded
    with +0, lanes, butterflies, eight warps, then levels of the same."""
    def block(v):
        v = list(v) + [F(0)] * (2048 - len(v))
        lane = []
        for t in range(256):
            g0, g1 = v[4 * t:4 * t + 4], v[1024 + 4 * t:1024 + 4 * t + 4]
            lane.append(F(F(F(g0[0] + g0[1]) + F(g0[2] + g0[3]))
                          + F(F(g1[0] + g1[1]) + F(g1[2] + g1[3]))))
        w = []
        for k in range(8):
            a = lane[32 * k:32 * k + 32]
            for m in (16, 8, 4, 2, 1):
                a = [F(a[l] + a[l ^ m]) for l in range(32)]
            w.append(a[0])
        return F(F(F(w[0] + w[1]) + F(w[2] + w[3])) + F(F(w[4] + w[5]) + F(w[6] + w[7])))

    vals = [F(v) for v in x]
    if not vals:
        return block([])
    while True:
        vals = [block(vals[i:i + 2048]) for i in range(0, len(vals), 2048)]
        if len(vals) == 1:
            return vals[0]


@pytest.mark.parametrize("n", [0, 1, 3, 2047, 2048, 2049, 3 * 2048 + 5])
def test_sum_matches_the_stated_order(n):
    x = np.random.default_rng(n + 1).standard_normal(n).astype(np.float32) * 1e3
    v, _ = O.tile_reduce(x, "sum")
    assert _bits(v) == _bits(_py_sum(x))


def test_sum_order_is_the_tree_not_the_sequence():
    # Sequentially ((1e8 + 1) - 1e8) + 1 = 1; the tree pairs (1e8 + 1) and
    # (-1e8 + 1), each rounding the 1 away: 0.
    x = np.array([1e8, 1, -1e8, 1], np.float32)
    v, _ = O.tile_reduce(x, "sum")
    assert v == 0.0
    assert _py_sum(x) == 0.0


def test_sum_levels_above_one_block():
    # 2048 * 2048 + 1 values: three levels, the last over two partials.
    n = 2048 * 2048 + 1
    x = np.ones(n, np.float32)
    v, _ = O.tile_reduce(x, "sum")
    assert v == np.float32(n)  # every partial is exact here


def test_min_max_edges():
    nan = np.float32("nan")
    cases = [
        ([1.0, -2.0, 3.0], -2.0, 3.0),
        ([0.0, -0.0], -0.0, 0.0),
        ([-0.0, 0.0], -0.0, 0.0),
        ([np.inf, -np.inf], -np.inf, np.inf),
    ]
    for x, lo, hi in cases:
        x = np.array(x, np.float32)
        assert _bits(O.tile_reduce(x, "min")[0]) == _bits(lo), x
        assert _bits(O.tile_reduce(x, "max")[0]) == _bits(hi), x
    x = np.array([1.0, nan, -5.0], np.float32)
    assert _bits(O.tile_reduce(x, "min")[0]) == NAN_BITS
    assert _bits(O.tile_reduce(x, "max")[0]) == NAN_BITS
    e = np.zeros(0, np.float32)
    assert O.tile_reduce(e, "min")[0] == np.inf
    assert O.tile_reduce(e, "max")[0] == -np.inf
    assert _bits(O.tile_reduce(e, "sum")[0]) == 0


def test_argmax_edges():
    nan = np.float32("nan")
    # Ties: the first index; across blocks too.
    x = np.zeros(5000, np.float32)
    x[[7, 3000, 4999]] = 2.5
    assert O.tile_reduce(x, "argmax") == (np.float32(2.5), 7)
    # +0 above -0.
    assert O.tile_reduce(np.array([-0.0, 0.0, -0.0], np.float32), "argmax")[1] == 1
    # The first NaN wins.
    i, = [O.tile_reduce(np.array([1.0, 9.0, nan, 4.0, nan], np.float32), "argmax")[1]]
    assert i == 2
    # All -inf: index 0; empty: -1.
    assert O.tile_reduce(np.full(3, -np.inf, np.float32), "argmax")[1] == 0
    assert O.tile_reduce(np.zeros(0, np.float32), "argmax") == (np.float32(-np.inf), -1)
    # idx_base shifts the index.
    assert O.tile_reduce(np.array([0.0, 5.0], np.float32), "argmax", idx_base=100)[1] == 101


@pytest.mark.parametrize("kind", ["sum", "min", "max", "argmax"])
def test_sharded_partials_equal_the_whole(kind):
    # Shards of whole blocks: concatenating their first-level partials and
    # finishing the tree gives the whole signal's result bit for bit.
    n = 5 * 2048 + 77
    x = np.random.default_rng(3).standard_normal(n).astype(np.float32)
    x[1234] = 40.0
    whole = O.tile_reduce(x, kind)
    pv, pi = [], []
    for s0 in range(0, n, 2 * 2048):
        v, i = O.tile_reduce_partials(x[s0:s0 + 2 * 2048], kind, idx_base=s0)
        pv.append(v)
        pi.append(i)
    got = O.tile_reduce_levels(np.concatenate(pv), np.concatenate(pi), kind)
    assert _bits(got[0]) == _bits(whole[0])
    if kind == "argmax":
        assert got[1] == whole[1] == 1234


def test_shard_range_covers_in_whole_blocks():
    """The library's split for the sharded reduction (host code only)."""
    from simtgo_b200 import tile
    from simtgo_b200._lib import SimtgoError

    for n in (0, 1, 2047, 2048, 5000, 1 << 20, (1 << 28) + 3):
        for world in (1, 2, 3, 8):
            pos = 0
            for r in range(world):
                s0, ln = tile.ShardRange(n, world, r)
                assert s0 == pos and ln >= 0, (n, world, r)
                if s0 + ln < n:
                    assert s0 % 2048 == 0 and ln % 2048 == 0 and ln > 0
                pos += ln
            assert pos == n
    with pytest.raises(SimtgoError):
        tile.ShardRange(10, 2, 2)
