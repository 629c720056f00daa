"""The device greedy pick (hc_argmax_dev: k_argmax, and with shards > 1 the
per-slice pairs plus k_pick_pairs of a tensor-parallel LM head) against the
host restatement of the reference's fold, `max_by(|a, b|
a.partial_cmp(b).unwrap_or(Equal))` (run.rs:234-238, serve.rs:300): the last
maximal index, and with NaNs the last maximal index after the last NaN, or
that NaN when it ends the row.  Integer index work: the ids must be equal."""
import ctypes

import numpy as np
import pytest

from hypno_b200._lib import call
from hypno_b200.serve import greedy_last_max

pytestmark = pytest.mark.gpu


def rows_for(V, rng):
    """Rows that exercise every branch of the fold."""
    rows = []
    base = rng.standard_normal(V).astype(np.float32)
    rows.append(base.copy())                                    # plain
    r = base.copy(); m = r.max(); r[[3, V // 2, V - 5]] = m      # ties: the last one wins
    rows.append(r)
    r = base.copy(); r[0] = np.nan                              # NaN first: ignored after it
    rows.append(r)
    r = base.copy(); r[int(np.argmax(r)) // 2] = np.nan          # NaN before the maximum
    rows.append(r)
    r = base.copy(); i = int(np.argmax(r)); r[min(V - 2, i + 1)] = np.nan  # NaN just after the maximum
    rows.append(r)
    r = base.copy(); r[V - 1] = np.nan                          # NaN ends the row: it is the pick
    rows.append(r)
    r = base.copy(); r[[1, V // 3, V - 7]] = np.nan             # several NaNs
    rows.append(r)
    rows.append(np.full(V, np.nan, np.float32))                 # all NaN: the last index
    r = base.copy(); r[V // 4] = np.inf; r[V // 2] = np.inf     # +inf ties
    rows.append(r)
    rows.append(np.full(V, -np.inf, np.float32))                # all -inf
    r = np.zeros(V, np.float32); r[V // 3] = -0.0; r[2] = -0.0  # signed zeros compare equal
    rows.append(r)
    r = base.copy(); r[V - 3] = np.nan; r[V - 1] = r.max() + 1   # NaN, then a new maximum
    rows.append(r)
    return np.stack(rows)


@pytest.mark.parametrize("V,pad,shards", [(128256, 0, 1), (128256, 0, 2), (128256, 0, 4), (1001, 7, 1),
                                          (1000, 12, 4), (64, 0, 2)])
def test_argmax_fold_vs_host(cuda_device, V, pad, shards):
    import torch
    rng = np.random.default_rng(V + pad + shards)
    L = rows_for(V, rng)
    B = L.shape[0]
    ld = V + pad
    host = np.zeros((B, ld), np.float32)
    host[:, :V] = L
    dl = torch.from_numpy(host).to(cuda_device)
    out = torch.zeros(B, dtype=torch.int32, device=cuda_device)
    pairs = torch.zeros(2 * shards * B, dtype=torch.float32, device=cuda_device)
    call("hc_argmax_dev", ctypes.c_void_p(dl.data_ptr()), ctypes.c_size_t(ld), B, V, shards,
         ctypes.c_void_p(pairs.data_ptr()), ctypes.c_void_p(out.data_ptr()), None)
    torch.cuda.synchronize()
    got = out.cpu().numpy().astype(np.int64)
    want = np.array([greedy_last_max(L[b]) for b in range(B)])
    assert np.array_equal(got, want), [(b, int(got[b]), int(want[b])) for b in range(B) if got[b] != want[b]]
