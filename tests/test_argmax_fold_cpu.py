"""The greedy pick's semantics on the host (no GPU): `greedy_last_max`, the
reference the device argmax tests compare with, against a literal
restatement of Rust's `Iterator::max_by` with
`partial_cmp(..).unwrap_or(Equal)` (run.rs:234-238, serve.rs:300): the fold
keeps its accumulator only when it compares Greater than the next element.
Also the vocabulary-sharded combine that the device runs for a
tensor-parallel LM head (per-shard pick, value and "held a NaN" bit, folded
in shard order, restarted at a shard with a NaN): over any split of a row it
must give the whole row's pick."""
import numpy as np
import pytest

from hypno_b200.serve import greedy_last_max


def partial_cmp_greater(a, b):
    """a.partial_cmp(b) == Some(Greater); NaN on either side gives None."""
    return not (np.isnan(a) or np.isnan(b)) and a > b


def rust_max_by(v):
    if len(v) == 0:
        return 0
    acc = 0
    for i in range(1, len(v)):
        if not partial_cmp_greater(v[acc], v[i]):   # Less, Equal or None -> take the next
            acc = i
    return acc


def shard_pick(v):
    """What k_argmax reports for one slice: (pick, value, held a NaN)."""
    nan = np.flatnonzero(np.isnan(v))
    last = int(nan[-1]) if nan.size else -1
    tail = v[last + 1:]
    if tail.size == 0:
        return last, v[last], True
    j = last + 1 + int(np.flatnonzero(tail == tail.max())[-1])
    return j, v[j], last >= 0


def sharded_pick(v, shards):
    """k_pick_pairs over the shards' (pick, value, NaN bit) in shard order."""
    n = len(v) // shards
    best, bi = 0.0, -1
    for r in range(shards):
        j, val, has_nan = shard_pick(v[r * n:(r + 1) * n])
        if has_nan or bi < 0 or not (best > val):
            best, bi = val, r * n + j
    return bi


def random_row(rng, n):
    v = rng.standard_normal(n).astype(np.float32)
    v = np.round(v, 1)                                    # many ties
    for special in (np.nan, np.inf, -np.inf, -0.0, 0.0):
        k = rng.integers(0, 3)
        v[rng.integers(0, n, k)] = special
    return v


@pytest.mark.parametrize("seed", range(40))
def test_host_fold_matches_rust_max_by(seed):
    rng = np.random.default_rng(seed)
    for n in (1, 2, 7, 64, 333):
        v = random_row(rng, n)
        assert greedy_last_max(v) == rust_max_by(v), (n, v)


@pytest.mark.parametrize("seed", range(40))
def test_sharded_combine_matches_whole_row(seed):
    rng = np.random.default_rng(1000 + seed)
    for shards in (2, 3, 4, 8):
        v = random_row(rng, shards * int(rng.integers(1, 40)))
        assert sharded_pick(v, shards) == rust_max_by(v), (shards, v)


def test_fold_edge_rows():
    nan = np.nan
    cases = [
        [nan, nan, nan],                  # all NaN: the last index
        [3.0, nan],                       # a NaN that ends the row is the pick
        [5.0, nan, 1.0, 1.0],             # after the NaN: the last of equal maxima
        [-0.0, 0.0, -0.0],                # signed zeros compare Equal
        [np.inf, 1.0, np.inf],            # +inf ties
        [-np.inf, -np.inf],
    ]
    for c in cases:
        v = np.array(c, np.float32)
        assert greedy_last_max(v) == rust_max_by(v), c
        for shards in (1, len(c)):
            if len(c) % shards == 0:
                assert sharded_pick(v, shards) == rust_max_by(v), (c, shards)
