"""Op-level parity of the sm_100a backend against the CPU oracle, through
the C ABI (hypno_b200.ops -> include/hypno_cuda.h).

Bars: Q4_0 pack/unpack and RoPE bit-exact; matmul outputs within
max|gpu - ref| / max(1, max|ref|) <= 1e-3 (north_star tolerance); the
element-wise ops within a few f32 ulps."""
import hashlib

import numpy as np
import pytest

from hypno_b200 import ops, synth
from oracle import oracle as orc

pytestmark = pytest.mark.gpu
TOL = 1e-3


def rel_err(a, ref):
    return float(np.max(np.abs(a.astype(np.float64) - ref)) / max(1.0, float(np.max(np.abs(ref)))))


def _edge_blocks():
    rng = np.random.default_rng(11)
    blocks = [np.zeros(32, np.float32)]
    b = np.zeros(32, np.float32); b[5] = 7.0; b[6] = 3.5; b[7] = -3.5; b[8] = 0.5; b[9] = -0.5; blocks.append(b)
    blocks.append(np.full(32, -1e-30, np.float32))           # subnormal scale
    blocks.append(np.full(32, 1e5, np.float32))              # scale overflows f16
    blocks.append((np.arange(32, dtype=np.float32) - 15.5) * np.float32(0.1))
    b = rng.standard_normal(32).astype(np.float32); b[3] = np.nan; blocks.append(b)
    b = rng.standard_normal(32).astype(np.float32); b[0] = np.inf; blocks.append(b)
    # exact halfway points q + 0.5 of an exactly representable scale
    s = np.float32(1.0)
    b = (np.arange(32, dtype=np.float32) % 15 - 7 + 0.5).astype(np.float32) * s; b[0] = 7.0; blocks.append(b)
    return np.concatenate(blocks)


@pytest.mark.parametrize("kind", ["normal", "edge", "wide"])
def test_q4_pack_unpack_bit_exact(cuda_device, kind):
    rng = np.random.default_rng(1)
    if kind == "normal":
        x = (rng.standard_normal(32 * 4099) * 0.02).astype(np.float32)
    elif kind == "edge":
        x = _edge_blocks()
    else:
        x = (rng.standard_normal(32 * 1000) * np.exp(rng.uniform(-20, 8, 32 * 1000))).astype(np.float32)
    x = np.concatenate([x, rng.standard_normal(17).astype(np.float32)])  # ragged tail: floor(n/32) blocks
    q_gpu = ops.quantize_f32_to_q4_0(x)
    q_ref = orc.quantize_f32_to_q4_0(x)
    assert q_gpu == q_ref
    d_gpu = ops.dequantize_q4_0(q_gpu)
    d_ref = orc.dequantize_q4_0(q_ref)
    # 0 * inf scales give NaN on both sides; NaN payloads differ between the
    # GPU's canonical NaN and x86's default NaN, every other value is bit-equal
    nan = np.isnan(d_ref)
    assert np.array_equal(nan, np.isnan(d_gpu))
    assert np.array_equal(d_gpu[~nan].view(np.uint32), d_ref[~nan].view(np.uint32))


def test_q4_pack_byte_diagnostic(cuda_device):
    """Localises any pack mismatch: per block, which of the 18 bytes differ."""
    x = (np.random.default_rng(2).standard_normal(32 * 64) * 0.02).astype(np.float32)
    q_gpu = np.frombuffer(ops.quantize_f32_to_q4_0(x), np.uint8).reshape(64, 18)
    q_ref = np.frombuffer(orc.quantize_f32_to_q4_0(x), np.uint8).reshape(64, 18)
    bad = np.argwhere(q_gpu != q_ref)
    if bad.size:
        print("mismatching (block, byte):", bad[:40].tolist())
        print("gpu block0", q_gpu[0].tobytes().hex(), "ref block0", q_ref[0].tobytes().hex())
    assert bad.size == 0


def test_q4_empty_and_short(cuda_device):
    assert ops.quantize_f32_to_q4_0(np.zeros(31, np.float32)) == b""
    assert ops.dequantize_q4_0(b"\x00" * 17).size == 0


@pytest.mark.parametrize("n,m", [(64, 64), (100, 96), (7, 172), (172, 64), (576, 576), (1536, 576), (4096, 4096),
                                 (33, 14336)])
def test_matmul_q4_vs_oracle(cuda_device, n, m):
    w = orc.quantize_f32_to_q4_0(synth.normal_host(0, f"w{n}x{m}", n * m, 0.02))
    x = synth.normal_host(1, f"x{m}", m, 1.0)
    y = np.empty(n, np.float32)
    ops.matmul_vec_auto(y, w, ops.DTYPE_Q4_0, x, None, n, m)
    ref = orc.matmul_q4_0(w, x, n, m)
    assert rel_err(y, ref) <= 1e-5, rel_err(y, ref)


def test_matmul_bias_and_short_buffer(cuda_device):
    n, m = 40, 64
    w = orc.quantize_f32_to_q4_0(synth.normal_host(0, "wb", n * m, 0.02))
    x = synth.normal_host(1, "xb", m, 1.0)
    bias = synth.normal_host(2, "bb", n, 1.0)
    y = np.empty(n, np.float32)
    ops.matmul_vec_auto(y, w, ops.DTYPE_Q4_0, x, bias, n, m)
    assert rel_err(y, orc.matmul_q4_0(w, x, n, m, bias)) <= 1e-5
    short = w[: len(w) - 18 * 3]  # the reference skips missing trailing blocks (kernels.rs:294, 374)
    ops.matmul_vec_auto(y, short, ops.DTYPE_Q4_0, x, None, n, m)
    assert rel_err(y, orc.matmul_q4_0(short, x, n, m)) <= 1e-5


def test_matmul_fp32_fp16_weights(cuda_device):
    n, m = 96, 200
    w = synth.normal_host(0, "wf", n * m, 0.1)
    x = synth.normal_host(1, "xf", m, 1.0)
    y = np.empty(n, np.float32)
    ops.matmul_vec_auto(y, w.view(np.uint8), ops.DTYPE_FP32, x, None, n, m)
    assert rel_err(y, orc.matmul_f32(w, x, n, m)) <= 1e-5
    w16 = w.astype(np.float16)
    ops.matmul_vec_auto(y, w16.view(np.uint8), ops.DTYPE_FP16, x, None, n, m)
    assert rel_err(y, orc.matmul_f16(w16.view(np.uint16), x, n, m)) <= 1e-5


def test_q8_0_is_rejected(cuda_device):
    from hypno_b200._lib import HypnoCudaError
    y = np.empty(4, np.float32)
    with pytest.raises(HypnoCudaError):
        ops.matmul_vec_auto(y, np.zeros(34 * 4, np.uint8), ops.DTYPE_Q8_0, np.ones(32, np.float32), None, 4, 32)


@pytest.mark.parametrize("batch", [1, 2, 3, 8, 17, 64, 130])
def test_batch_matmul_vs_oracle(cuda_device, batch):
    n, m = 256, 512
    w = orc.quantize_f32_to_q4_0(synth.normal_host(0, "wbm", n * m, 0.02))
    X = synth.normal_host(1, "xbm", batch * m, 1.0)
    Y = np.empty(batch * n, np.float32)
    ops.batch_matmul(Y, w, ops.DTYPE_Q4_0, X, n, m, batch)
    ref = orc.batch_matmul_q4_0(w, X, n, m).reshape(-1)
    assert rel_err(Y, ref) <= TOL


def test_rmsnorm_vs_oracle(cuda_device):
    for n in (4, 63, 64, 576, 4096, 8192):
        x = synth.normal_host(3, f"r{n}", n, 1.0)
        w = synth.normal_host(4, f"rw{n}", n, 0.02)
        y = x.copy()
        ops.rms_norm_in_place(y, w, 1e-5)
        ref = orc.rms_norm(x, w, 1e-5)
        np.testing.assert_allclose(y, ref, rtol=2e-6, atol=1e-12)
    y = np.full(64, 2.0, np.float32)
    ops.rms_norm_in_place(y, np.ones(64, np.float32), 1e-5)
    assert np.all(np.abs(y - 1) < 1e-3)


def test_softmax_vs_oracle(cuda_device):
    rng = np.random.default_rng(5)
    for n in list(range(1, 42)) + [127, 128, 129, 1000, 4607]:
        x = (rng.standard_normal(n) * 3).astype(np.float32)
        y = x.copy()
        ops.softmax_in_place(y)
        ref = orc.softmax(x)
        np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-9)
    # clamp region (|x - max| > 87) and ties at the max
    x = np.array([0, -100, 50, 50, -200, 1, 2, 3, 4, 5], np.float32)
    y = x.copy()
    ops.softmax_in_place(y)
    np.testing.assert_allclose(y, orc.softmax(x), rtol=1e-5, atol=1e-9)


def test_silu_vs_oracle(cuda_device):
    x = np.linspace(-30, 30, 10001, dtype=np.float32)
    y = x.copy()
    ops.silu_in_place(y)
    np.testing.assert_allclose(y, orc.silu(x), rtol=1e-6, atol=1e-30)


@pytest.mark.parametrize("hd,pos,theta", [(16, 0, 1e4), (64, 7, 1e4), (64, 4607, 1e4), (128, 2303, 5e5),
                                          (128, 4607, 5e5)])
def test_rope_bit_exact(cuda_device, hd, pos, theta):
    q = synth.normal_host(5, "q", hd, 1.0)
    k = synth.normal_host(6, "k", hd, 1.0)
    qg, kg = q.copy(), k.copy()
    ops.rope(qg, kg, hd, pos, theta)
    qr, kr = orc.rope(q, k, hd, pos, theta)
    assert np.array_equal(qg.view(np.uint32), qr.view(np.uint32))
    assert np.array_equal(kg.view(np.uint32), kr.view(np.uint32))


def test_synth_device_equals_host(cuda_device):
    import torch
    from hypno_b200._lib import call
    n = (1 << 22) + 3
    buf = torch.empty(n, dtype=torch.float32, device=cuda_device)
    call("hc_synth_normal_dev", 3, synth.fnv1a64("t"), 11, n, 0.02, buf.data_ptr(), None)
    torch.cuda.synchronize()
    host = synth.normal_host(3, "t", n, 0.02, offset=11)
    assert np.array_equal(buf.cpu().numpy().view(np.uint32), host.view(np.uint32))


def test_streamed_image_file_equals_host_image(cuda_device, tmp_path):
    """synth.write_image_file (the c5 writer: one tensor at a time, generated
    and quantized on the device) writes the bytes of the host-built image, and
    a model opened from the file (memory-mapped) loads."""
    from hypno_b200 import engine
    cfg = dict(hidden=256, inter=512, heads=4, kv_heads=2, layers=2, vocab=512, theta=10000.0, max_pos=64,
               embed="q4", lm_head="tied")
    path = str(tmp_path / "m.hypno")
    synth.write_image_file(cfg, path, seed=7, device=cuda_device)
    want = synth.build_image(cfg, seed=7)
    got = np.fromfile(path, dtype=np.uint8)
    assert got.size == want.size and np.array_equal(got, want)
    m = engine.HypnoModel.open(path)
    assert m.config.num_hidden_layers == 2
    m.close()


# ---- the Q4_0 operator sweep ---------------------------------
@pytest.mark.parametrize("N,K", synth.SWEEP_NK)
def test_sweep_pack_and_matmul(cuda_device, N, K):
    """Pack bit-exact on the sweep tensors; Y = X W^T for every M of the
    sweep against the oracle on a subset of rows (full rows for M = 1)."""
    import torch
    from hypno_b200._lib import call
    import ctypes
    w32 = torch.empty(N * K, dtype=torch.float32, device=cuda_device)
    call("hc_synth_normal_dev", 0, synth.fnv1a64(f"sweep.W.{N}x{K}"), 0, N * K, 0.02, w32.data_ptr(), None)
    wq = torch.empty(N * K // 32 * 18, dtype=torch.uint8, device=cuda_device)
    call("hc_q4_0_quantize_dev", w32.data_ptr(), N * K, wq.data_ptr(), None)
    torch.cuda.synchronize()
    w_host = w32.cpu().numpy()
    del w32
    wq_host = wq.cpu().numpy()
    # bit-exact pack against the oracle on a 1/16 slice of blocks (the whole
    # tensor is hashed on the GPU side for the golden check)
    sl = slice(0, (N * K // 16) // 32 * 32)
    assert orc.quantize_f32_to_q4_0(w_host[sl]) == wq_host[: (sl.stop // 32) * 18].tobytes()
    h = ctypes.c_void_p()
    call("hc_q4_matrix_from_dev", wq.data_ptr(), wq.numel(), N, K, None, ctypes.byref(h))
    try:
        rows = np.unique(np.concatenate([np.arange(64), np.linspace(0, N - 1, 192).astype(np.int64)]))
        kb = K // 32
        sub = np.concatenate([wq_host[r * kb * 18:(r + 1) * kb * 18] for r in rows])
        for M in synth.SWEEP_M:
            X = torch.from_numpy(synth.normal_host(1, f"sweep.X.{M}x{K}", M * K, 1.0)).to(cuda_device)
            Y = torch.empty(M * N, dtype=torch.float32, device=cuda_device)
            call("hc_q4_matmul_dev", h, X.data_ptr(), M, Y.data_ptr(), None)
            torch.cuda.synchronize()
            Yh = Y.cpu().numpy().reshape(M, N)
            Xh = X.cpu().numpy().reshape(M, K)
            ms = range(M) if M <= 8 else [0, 1, M // 2, M - 1]
            for mi in ms:
                ref = orc.matmul_q4_0(sub, Xh[mi], rows.size, K)
                err = rel_err(Yh[mi, rows], ref)
                assert err <= TOL, (M, mi, err)
            if M == 1:
                full = orc.matmul_q4_0(wq_host, Xh[0], N, K)
                assert rel_err(Yh[0], full) <= 1e-5
    finally:
        call("hc_q4_matrix_free", h)
    digest = hashlib.sha256(wq_host.tobytes()).hexdigest()
    assert len(digest) == 64
