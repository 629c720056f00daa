"""hc_q4_matmul_noalloc: the matmul for callers that cannot allocate device
memory while running (a serving process whose device memory all belongs to
its own pool, or code that may not call cudaMalloc mid-stream).  Checked
through the C ABI against hc_q4_matmul_dev on the same inputs, call after
call, with the same tolerance as the other matmul tests, and against the
oracle on sample rows.  The sizes cover the CUDA-core path (one token), the
tensor-core path, the largest token count the fixed scratch takes at this
width and the first one it refuses.  This file is collected last so a
failure here never hides the other tests' results."""
import ctypes

import numpy as np
import pytest

from hypno_b200 import synth
from hypno_b200._lib import HypnoCudaError, call
from oracle import oracle as orc

pytestmark = pytest.mark.gpu
TOL = 1e-3
SCRATCH_BYTES = 8 << 20   # the fixed array of the library's device image
FLAG_BYTES = 256          # its first bytes hold the pipeline abort flag


def rel_err(a, ref):
    return float(np.max(np.abs(a.astype(np.float64) - ref)) / max(1.0, float(np.max(np.abs(ref)))))


def test_noalloc_matmul_matches_existing_entry_point(cuda_device):
    import torch
    N, K = 1024, 4096
    max_t = (SCRATCH_BYTES - FLAG_BYTES) // (2 * K * 2)  # split fp16 rows: 2 x K halves per token
    assert max_t == 511
    wq = np.frombuffer(orc.quantize_f32_to_q4_0(synth.normal_host(0, "noalloc.W", N * K, 0.02)), np.uint8)
    h = ctypes.c_void_p()
    call("hc_q4_matrix_upload", wq.ctypes.data, wq.size, N, K, ctypes.byref(h))
    try:
        # calls in a row: tensor-core shapes, the one-token CUDA-core shape, the largest accepted size
        for call_no, T in enumerate((32, 200, 1, max_t)):
            Xh = synth.normal_host(call_no + 1, "noalloc.X", T * K, 1.0)
            X = torch.from_numpy(Xh).to(cuda_device)
            y_ref = torch.empty(T * N, dtype=torch.float32, device=cuda_device)
            y_new = torch.full((T * N,), float("nan"), dtype=torch.float32, device=cuda_device)
            call("hc_q4_matmul_dev", h, X.data_ptr(), T, y_ref.data_ptr(), None)
            torch.cuda.synchronize()
            free_before = torch.cuda.mem_get_info()[0]
            call("hc_q4_matmul_noalloc", h, X.data_ptr(), T, y_new.data_ptr(), None)
            torch.cuda.synchronize()
            if call_no >= 1:  # after the first call (which may load the module), no device memory is taken
                assert torch.cuda.mem_get_info()[0] == free_before
            a, b = y_new.cpu().numpy(), y_ref.cpu().numpy()
            assert np.all(np.isfinite(a))
            assert rel_err(a, b) <= TOL, (T, rel_err(a, b))
            for t in sorted({0, T // 2, T - 1}):  # and the oracle on sample rows
                ref = orc.matmul_q4_0(wq, Xh[t * K:(t + 1) * K], N, K)
                assert rel_err(a.reshape(T, N)[t], ref) <= TOL, (T, t)
        # beyond the fixed scratch: rejected with a clear error, nothing launched
        T_big = max_t + 1
        Xb = torch.zeros(T_big * K, dtype=torch.float32, device=cuda_device)
        yb = torch.zeros(T_big * N, dtype=torch.float32, device=cuda_device)
        with pytest.raises(HypnoCudaError) as e:
            call("hc_q4_matmul_noalloc", h, Xb.data_ptr(), T_big, yb.data_ptr(), None)
        assert e.value.code == -1 and "scratch" in str(e.value)
    finally:
        call("hc_q4_matrix_free", h)
