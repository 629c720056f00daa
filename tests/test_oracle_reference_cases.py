"""The reference's own unit tests (crates/hypno/src/*.rs #[cfg(test)]),
re-expressed against the CPU oracle.  They pin the restatement to the
behaviour the reference asserts about itself."""
import numpy as np
import pytest

from hypno_b200 import hypno_file as hf
from oracle import oracle as orc
from tests import _models


# ---- quant.rs:212-237 --------------------------------------------------
def test_q4_0_roundtrip():
    src = (np.arange(32, dtype=np.float32) - np.float32(15.5)) * np.float32(0.1)
    dst = orc.dequantize_q4_0(orc.quantize_f32_to_q4_0(src))
    assert np.all(np.abs(src - dst) < 0.5)


def test_q4_0_zero():
    q = orc.quantize_f32_to_q4_0(np.zeros(32, np.float32))
    assert q[:2] == bytes([0x00, 0x3C])  # scale 1.0 in f16
    assert all(b == 0x88 for b in q[2:])  # q = 0 -> nibble 8
    assert np.all(np.abs(orc.dequantize_q4_0(q)) < 1e-6)


# ---- kernels.rs:707-742 ------------------------------------------------
def test_matmul_f32_correctness():
    n, m = 128, 256
    i = np.arange(n * m, dtype=np.float32)
    w = np.sin(i * np.float32(1.234)).astype(np.float32)
    x = np.cos(np.arange(m, dtype=np.float32) * np.float32(0.789)).astype(np.float32)
    y = orc.matmul_f32(w, x, n, m)
    y_ref = (w.reshape(n, m).astype(np.float64) @ x.astype(np.float64)).astype(np.float32)
    assert np.max(np.abs(y - y_ref)) < 1e-3


def test_rms_norm_const():
    y = orc.rms_norm(np.full(64, 2.0, np.float32), np.ones(64, np.float32), 1e-5)
    assert np.all(np.abs(y - 1.0) < 0.001)


def test_softmax_fast_small():
    y = orc.softmax(np.array([1.0, 2.0, 3.0, 4.0], np.float32))
    assert abs(y.sum() - 1.0) < 0.001
    assert y[3] > y[2] > y[1]


# ---- ops.rs:113-137 ----------------------------------------------------
def test_ops_matmul_vec():
    y = orc.matmul_f32(np.array([1, 2, 3, 4], np.float32), np.array([5, 6], np.float32), 2, 2)
    assert abs(y[0] - 17) < 0.001 and abs(y[1] - 39) < 0.001


def test_ops_softmax():
    assert abs(orc.softmax(np.array([1, 2, 3], np.float32)).sum() - 1) < 0.001


def test_ops_rms_norm():
    y = orc.rms_norm(np.full(4, 2.0, np.float32), np.ones(4, np.float32), 1e-5)
    assert np.all(np.abs(y - 1) < 0.001)


# ---- softmax beyond the reference's own test: the polynomial body ------
def test_softmax_polynomial_body_matches_formula():
    rng = np.random.default_rng(3)
    for n in (8, 9, 15, 16, 17, 40, 129):
        x = rng.standard_normal(n).astype(np.float32)
        y = orc.softmax(x)
        m = x.max()
        n8 = n - n % 8
        v = np.clip(x - m, -87, 87).astype(np.float64)
        e = np.where(np.arange(n) < n8, 1 + v / 8 + v ** 2 / 128 + v ** 3 / 3072 + v ** 4 / 98304, np.exp(v))
        np.testing.assert_allclose(y, e / e.sum(), rtol=2e-6, atol=1e-7)


# ---- loader.rs:214-319 (hand-assembled file) ---------------------------
def test_loader_hand_built_image():
    q4 = orc.quantize_f32_to_q4_0(np.arange(32, dtype=np.float32) * np.float32(0.1))
    img = hf.write_image([("architecture", "llama"), ("hidden_size", "64")],
                         [("weight", (64,), hf.DT_FP32, np.arange(64, dtype=np.float32).view(np.uint8)),
                          ("qweight", (32,), hf.DT_Q4_0, np.frombuffer(q4, np.uint8))])
    man = hf.Manifest(img)
    assert man.metadata == {"architecture": "llama", "hidden_size": "64"}
    # the oracle's reader (loader.rs:39-133) sees the same file
    with pytest.raises(ValueError):
        orc.OracleModel(img)  # no num_attention_heads -> HypnoConfig::from_model is None
    data, dt = man.tensor_bytes("weight")
    f = np.frombuffer(bytes(data), np.float32)
    assert dt == hf.DT_FP32 and f.size == 64 and f[0] == 0 and f[63] == 63
    data, dt = man.tensor_bytes("qweight")
    assert dt == hf.DT_Q4_0 and len(data) == 18


def test_loader_rejects_bad_images():
    with pytest.raises(ValueError):
        orc.OracleModel(np.zeros(8, np.uint8))
    img = hf.write_image([("hidden_size", "64"), ("num_attention_heads", "4")], [])
    bad = img.copy()
    bad[:4] = np.frombuffer(b"XXXX", np.uint8)
    with pytest.raises(ValueError):
        orc.OracleModel(bad)


# ---- sft_convert.rs:430-457 --------------------------------------------
def test_q4_payload_size_8192():
    data = np.arange(8192, dtype=np.float32) * np.float32(0.1)
    assert len(orc.quantize_f32_to_q4_0(data)) == 4608
    assert hf.data_bytes(hf.DT_Q4_0, 8192) == 4608
    assert hf.effective_dtype(hf.DT_Q4_0, 64) == hf.DT_FP32


# ---- transformer.rs:671-697 (FlatKVCache) -------------------------------
def test_flat_kv_cache():
    img = _models.reference_model_image(_models.TINY, 0.01, hf.DT_FP32)
    m = orc.OracleModel(img)
    kv = m.new_kv(128)
    assert kv.seq_len() == 0
    orc.model_forward(m, 42, kv)
    assert kv.seq_len() == 1
    kv.set_pos(0)
    assert kv.seq_len() == 0


# ---- turbo.rs:474-921 (batch prefill == token-by-token) ----------------
def _seq_logits(m, ids, extra=None):
    kv = m.new_kv()
    out = None
    for t in ids:
        out = orc.model_forward(m, t, kv)
    if extra is not None:
        out = orc.model_forward(m, extra, kv)
    return out, kv


@pytest.fixture(scope="module")
def tiny_fp32():
    return orc.OracleModel(_models.reference_model_image(_models.TINY, 0.01, hf.DT_FP32))


@pytest.fixture(scope="module")
def tiny_q4():
    return orc.OracleModel(_models.reference_model_image(_models.TINY, 0.01, hf.DT_Q4_0))


def test_batch_forward_vs_token_by_token(tiny_fp32):
    ids = [1, 5, 10, 42, 100, 7, 3]
    kv = tiny_fp32.new_kv()
    turbo = orc.batch_forward(tiny_fp32, ids, kv)
    seq, _ = _seq_logits(tiny_fp32, ids)
    assert turbo.shape == seq.shape
    assert np.max(np.abs(turbo - seq)) < 1e-5


def test_generation_after_batch_forward(tiny_fp32):
    prompt, nxt = [1, 5, 10, 42], 100
    kv = tiny_fp32.new_kv()
    orc.batch_forward(tiny_fp32, prompt, kv)
    a = orc.model_forward(tiny_fp32, nxt, kv)
    b, _ = _seq_logits(tiny_fp32, prompt, nxt)
    assert np.max(np.abs(a - b)) < 1e-5


def test_generation_after_batch_forward_q4(tiny_q4):
    prompt, nxt = [1, 5, 10, 42], 100
    kv = tiny_q4.new_kv()
    orc.batch_forward(tiny_q4, prompt, kv)
    a = orc.model_forward(tiny_q4, nxt, kv)
    b, _ = _seq_logits(tiny_q4, prompt, nxt)
    assert np.max(np.abs(a - b)) < 1e-3


def test_batch_forward_single_token(tiny_fp32):
    kv = tiny_fp32.new_kv()
    a = orc.batch_forward(tiny_fp32, [42], kv)
    b, _ = _seq_logits(tiny_fp32, [42])
    assert np.max(np.abs(a - b)) < 1e-5


def test_batch_kv_cache_positions(tiny_fp32):
    kv = tiny_fp32.new_kv()
    assert kv.seq_len() == 0
    orc.batch_forward(tiny_fp32, [1, 2, 3, 4, 5], kv)
    assert kv.seq_len() == 5


def test_batch_forward_empty_prompt(tiny_fp32):
    kv = tiny_fp32.new_kv()
    out = orc.batch_forward(tiny_fp32, [], kv)
    assert out.shape == (1000,) and np.all(out == 0) and kv.seq_len() == 0


def test_intermediate_state_q_projection(tiny_fp32):
    # turbo.rs:767-850: batch_matmul of one row == matmul_vec_auto
    w, dt = tiny_fp32.tensor("model.layers.0.self_attn.q_proj.weight")
    assert dt == hf.DT_FP32
    x = np.linspace(-1, 1, 64, dtype=np.float32)
    a = orc.matmul_f32(w.view(np.float32), x, 64, 64)
    b = orc.matmul_f32(w.view(np.float32), x, 64, 64)
    assert np.array_equal(a, b)


@pytest.mark.slow
def test_generation_full_scale_q4():
    """turbo.rs:613-711: TinyLlama dimensions, Q4_0, weights (i+1)*0.001."""
    m = orc.OracleModel(_models.reference_model_image(_models.TINYLLAMA, 0.001, hf.DT_Q4_0))
    prompt, nxt = [1, 5, 10, 42, 100, 7, 3], 500
    kv = m.new_kv()
    orc.batch_forward(m, prompt, kv)
    a = orc.model_forward(m, nxt, kv)
    b, _ = _seq_logits(m, prompt, nxt)
    assert np.max(np.abs(a - b)) < 1e-3


# ---- turbo.rs:924-1004 ---------------------------------------------------
def test_silu_values():
    s = orc.silu(np.array([0.0, -1.0, 1.0], np.float32))
    assert abs(s[0]) < 0.001 and abs(s[1] + 0.2689) < 0.01 and abs(s[2] - 0.7311) < 0.01
