"""Known-answer tests of the f32 -> f16 rounding used for Q4_0 scales.

The reference stores scales with `half` 2.7.1's `f16::from_f32`
(quant.rs:57), which implements IEEE 754 binary16 round-to-nearest-even
(the crate's software path and its F16C path agree).  That crate is not
vendored here, so the oracle's conversion is pinned against numpy's
independent IEEE implementation on ties, subnormals, overflow and every
representable f16."""
import numpy as np

from oracle import oracle as orc


def _np_f16_bits(x):
    return int(np.array([x], np.float32).astype(np.float16).view(np.uint16)[0])


def test_every_f16_round_trips():
    lib = orc.lib()
    for h in range(0x10000):
        if (h & 0x7C00) == 0x7C00 and (h & 0x3FF):
            continue  # NaN payloads
        f = lib.orc_f16_to_f32(h)
        assert np.float32(f) == np.array([h], np.uint16).view(np.float16).astype(np.float32)[0]
        assert lib.orc_f32_to_f16(f) == h


def test_rounding_against_numpy():
    rng = np.random.default_rng(0)
    bits = rng.integers(0, 2 ** 32, size=200_000, dtype=np.uint64).astype(np.uint32)
    xs = bits.view(np.float32)
    xs = xs[np.isfinite(xs)]
    lib = orc.lib()
    ref = xs.astype(np.float16).view(np.uint16)
    for x, r in zip(xs[:50_000], ref[:50_000]):
        assert lib.orc_f32_to_f16(float(x)) == int(r), hex(np.array([x], np.float32).view(np.uint32)[0])


def test_ties_subnormals_overflow():
    lib = orc.lib()
    cases = [
        1.0 + 2 ** -11,             # tie between 1.0 and 1+2^-10: to even (1.0)
        1.0 + 3 * 2 ** -11,         # tie: to even (1+2^-9)
        2 ** -24,                   # smallest subnormal
        2 ** -25,                   # half of it: tie to 0
        3 * 2 ** -26,               # rounds up to 2^-24
        65504.0, 65519.99, 65520.0, 1e6, -1e6,  # max normal / overflow to inf
        6.1035156e-05, 6.097555e-05,  # around the smallest normal
        0.0, -0.0, 0.02 / 7, 1.0 / 7,
    ]
    for c in cases:
        assert lib.orc_f32_to_f16(float(np.float32(c))) == _np_f16_bits(np.float32(c)), c
