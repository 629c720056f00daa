"""CPU-side checks of the backend library: it loads without a GPU, exports
every entry point include/hypno_cuda.h declares, its host-only pieces
(synthetic stream, .hypno writer) behave, and compute calls fail loudly
instead of falling back to the CPU when no device is present."""
import ctypes
import os
import re

import numpy as np
import pytest

from hypno_b200 import _lib, build, hypno_file as hf, synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def _declared():
    text = open(os.path.join(ROOT, "include", "hypno_cuda.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(hc_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_bound_entry_points():
    decl = _declared()
    assert set(decl) == set(_lib.SIGNATURES), set(decl) ^ set(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol(lib):
    raw = ctypes.CDLL(_lib.LIB_PATH)
    for name in _declared():
        assert hasattr(raw, name), name


def test_version_and_error_string(lib):
    assert lib.hc_version() >= 100
    assert isinstance(lib.hc_last_error(), bytes)


def test_synth_stream_deterministic_and_normal(lib):
    a = synth.normal_host(0, "w", 1 << 20, std=0.02)
    b = synth.normal_host(0, "w", 1 << 20, std=0.02)
    c = synth.normal_host(1, "w", 1 << 20, std=0.02)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    assert abs(a.mean()) < 1e-4 and abs(a.std() - 0.02) < 2e-4
    # offset addressing: element i of the stream does not depend on the chunking
    d = synth.normal_host(0, "w", 1000, std=0.02, offset=5000)
    assert np.array_equal(d, a[5000:6000])


def test_synth_matches_independent_numpy_restatement(lib):
    """The generator restated in numpy (integer steps + one f32 multiply)."""
    M = 0xFFFFFFFFFFFFFFFF

    def sm(z):
        z = (z + 0x9E3779B97F4A7C15) & M
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
        return z ^ (z >> 31)

    seed, stream = 7, synth.fnv1a64("model.norm.weight")
    key = sm(((seed * 0x100000001B3) & M) ^ sm((stream + 0x51ED270B2) & M))
    ref = []
    for i in range(64):
        s = 0
        for j in range(3):
            h = sm((key + 3 * i + j) & M)
            s += (h & 0xFFFF) + ((h >> 16) & 0xFFFF) + ((h >> 32) & 0xFFFF) + (h >> 48)
        ref.append(np.float32(s - 393210) * np.float32(np.float32(0.02) / np.float32(65536)))
    got = synth.normal_host(seed, "model.norm.weight", 64, std=0.02)
    assert np.array_equal(got, np.array(ref, np.float32))


def test_image_writer_layout():
    img = hf.write_image([("a", "1")], [("z", (40,), hf.DT_FP32, np.zeros(160, np.uint8)),
                                         ("b", (2, 32), hf.DT_Q4_0, np.ones(36, np.uint8))])
    man = hf.Manifest(img)
    names = list(man.tensors)
    assert names == ["b", "z"]  # BTreeMap order
    for n in names:
        assert man.tensors[n][2] % 64 == 0
    assert img.size % 64 == 0
    assert hf.rust_f64_display(1e-5) == "0.00001" and hf.rust_f64_display(500000.0) == "500000"


def test_compute_without_gpu_fails_loudly(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    x = np.ones(32, np.float32)
    with pytest.raises(_lib.HypnoCudaError) as e:
        from hypno_b200 import ops
        ops.silu_in_place(x)
    assert e.value.code == -2


def test_model_bytes_match_quoted_figures():
    # per-step Q4_0 weight bytes of the benchmark configs (0.5625 B per weight)
    assert synth.model_bytes(synth.CONFIGS["c1"]) == 75_644_928
    assert synth.model_bytes(synth.CONFIGS["c3"]) == 581_861_376
    assert synth.model_bytes(synth.CONFIGS["c4"]) == 4_221_370_368
