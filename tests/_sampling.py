"""Helpers of the sampling tests: the reference's XorShift64 draw and the
running sum of the kept weights in f64, to tell a pick at a token boundary
(within rounding of the draw) from a wrong pick."""
import numpy as np


def xorshift_next_f32(state):
    """XorShift64::next then next_f32 (run.rs:267-278): (new state, r)."""
    x = state
    x ^= (x << 13) & 0xFFFFFFFFFFFFFFFF
    x ^= x >> 7
    x ^= (x << 17) & 0xFFFFFFFFFFFFFFFF
    return x, np.float32((x >> 40) / 16777216.0)


def cdf_f64(logits, T, tp, tk):
    """The running sum of sample_token's kept weights over its total, in f64
    (None when the total is not positive)."""
    p = np.exp(logits.astype(np.float64) / T) if T > 0 else logits.astype(np.float64)
    if 0 < tk < p.size:
        thr = np.sort(p)[::-1][tk - 1]
        p = np.where(p < thr, 0.0, p)
    if tp < 1.0:
        s = p.sum()
        if s > 0:
            srt = np.sort(p)[::-1]
            c = np.cumsum(srt / s)
            hit = np.nonzero(c > tp)[0]
            thr = srt[hit[0]] if hit.size else np.inf
            p = np.where(p < thr, 0.0, p)
    s = p.sum()
    return (np.cumsum(p) / s) if s > 0 else None


def boundary_margin(logits, T, tp, tk, state_before, a, b):
    """Distance of the draw from the boundary between tokens a and b."""
    _, r = xorshift_next_f32(state_before)
    c = cdf_f64(np.asarray(logits, np.float32), T, tp, tk)
    return abs(float(c[min(a, b)]) - float(r)) if c is not None else 1.0
