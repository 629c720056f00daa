"""The tcgen05 Q4_0 GEMM (hc_gemm_tc.cu) against the oracle's per-token
matvec on ragged token counts, row counts that are not multiples of the
128-row tile, every token-tile size (32 / 64 / 128) and several token tiles.

The GEMM multiplies exact two-term fp16 weights by fp16 hi + lo activations
with f32 accumulation, so its error is that of an f32 dot product in another
summation order: the bar is 1e-4 of max(1, max|ref|), ten times tighter than
the north_star tolerance (1e-3), which a single fp16 operand per product
(~3e-4 per product) would not leave room for; the observed error is printed."""
import ctypes

import numpy as np
import pytest

from hypno_b200 import synth
from hypno_b200._lib import call
from oracle import oracle as orc

pytestmark = pytest.mark.gpu
TOL_TC = 1e-4


def rel_err(a, ref):
    return float(np.max(np.abs(a.astype(np.float64) - ref)) / max(1.0, float(np.max(np.abs(ref)))))


# (38400, 512): 300 tiles of 4 stages over 148 SMs, so at <= 32 tokens the
# launcher takes the stream-K grid (runs of 8-9 stages crossing tiles)
@pytest.mark.parametrize("N,K", [(128, 128), (256, 512), (200, 256), (1152, 4096), (640, 14336), (38400, 512)])
@pytest.mark.parametrize("T", [2, 8, 31, 32, 33, 64, 100, 128, 129, 256, 300])
def test_tc_gemm_vs_oracle(cuda_device, N, K, T):
    import torch
    wq = orc.quantize_f32_to_q4_0(synth.normal_host(0, f"tc.W.{N}x{K}", N * K, 0.02))
    X = synth.normal_host(1, f"tc.X.{T}x{K}", T * K, 1.0)
    h = ctypes.c_void_p()
    wb = np.frombuffer(wq, np.uint8)
    call("hc_q4_matrix_upload", wb.ctypes.data, wb.size, N, K, ctypes.byref(h))
    try:
        Xd = torch.from_numpy(X).to(cuda_device)
        Yd = torch.full((T * N,), float("nan"), dtype=torch.float32, device=cuda_device)
        call("hc_q4_matmul_dev", h, Xd.data_ptr(), T, Yd.data_ptr(), None)
        torch.cuda.synchronize()
        Y = Yd.cpu().numpy().reshape(T, N)
    finally:
        call("hc_q4_matrix_free", h)
    assert np.all(np.isfinite(Y))
    worst = 0.0
    for t in sorted({0, 1, T // 2, T - 1}):
        ref = orc.matmul_q4_0(wq, X[t * K:(t + 1) * K], N, K)
        worst = max(worst, rel_err(Y[t], ref))
    print(f"N={N} K={K} T={T}: rel err {worst:.2e}")
    assert worst <= TOL_TC


def test_tc_gemm_residual_epilogue(cuda_device):
    """EPI_ADD through the model path: y = W x + residual, in place."""
    import torch
    from hypno_b200 import ops
    N, K, T = 384, 256, 40
    wq = orc.quantize_f32_to_q4_0(synth.normal_host(0, "tc.res.W", N * K, 0.02))
    X = synth.normal_host(1, "tc.res.X", T * K, 1.0)
    Y = np.empty(T * N, np.float32)
    ops.batch_matmul(Y, wq, ops.DTYPE_Q4_0, X, N, K, T)
    ref = orc.batch_matmul_q4_0(wq, X, N, K).reshape(-1)
    assert rel_err(Y, ref) <= TOL_TC
