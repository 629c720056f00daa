"""Host-side mirror of hypno's op facade (crates/hypno/src/ops.rs) and of the
Q4_0 helpers of quant.rs, computed by the sm_100a backend.

Each function takes and returns numpy arrays on the host, like the
reference's slices, and calls the C ABI (include/hypno_cuda.h).  Shapes and
argument meaning follow the reference; errors raise HypnoCudaError.
"""
import numpy as np

from ._lib import DTYPE_FP16, DTYPE_FP32, DTYPE_Q4_0, DTYPE_Q8_0, call

__all__ = [
    "DTYPE_FP32", "DTYPE_FP16", "DTYPE_Q8_0", "DTYPE_Q4_0",
    "matmul_vec_auto", "matmul_vec_q4_0", "batch_matmul", "rms_norm_in_place", "rms_norm",
    "softmax_in_place", "softmax", "silu_in_place", "silu", "rope",
    "quantize_f32_to_q4_0", "dequantize_q4_0",
]


def _f32(a, name):
    if not (isinstance(a, np.ndarray) and a.dtype == np.float32 and a.flags.c_contiguous):
        raise TypeError(f"{name} must be a C-contiguous float32 numpy array")
    return a


def _bytes(w):
    if isinstance(w, (bytes, bytearray, memoryview)):
        w = np.frombuffer(w, dtype=np.uint8)
    if not isinstance(w, np.ndarray):
        raise TypeError("weights must be bytes or a numpy array")
    return np.ascontiguousarray(w).view(np.uint8).reshape(-1)


def matmul_vec_auto(y, w, dtype, x, bias, n, m):
    """ops::matmul_vec_auto (ops.rs:25-38): y[n] = W[n x m] . x[m] (+ bias),
    W given as its raw .hypno payload bytes of `dtype`."""
    _f32(y, "y"), _f32(x, "x")
    if y.size < n or x.size < m:
        raise ValueError("y/x shorter than n/m")
    wb = _bytes(w)
    b = None
    if bias is not None:
        b = _f32(bias, "bias")
        if b.size < n:
            raise ValueError("bias shorter than n")
    call("hc_matmul_vec_auto", y.ctypes.data, wb.ctypes.data, wb.size, int(dtype), x.ctypes.data,
         b.ctypes.data if b is not None else None, n, m)


def matmul_vec_q4_0(y, w_q, x, bias, n, m):
    """ops::matmul_vec_q4_0 (ops.rs:15-17)."""
    matmul_vec_auto(y, w_q, DTYPE_Q4_0, x, bias, n, m)


def batch_matmul(y, w, dtype, x, n, dim, batch):
    """turbo::batch_matmul (turbo.rs:306-343): Y[batch x n] = X[batch x dim] . W^T."""
    _f32(y, "y"), _f32(x, "x")
    if y.size < batch * n or x.size < batch * dim:
        raise ValueError("y/x too short")
    wb = _bytes(w)
    call("hc_batch_matmul", y.ctypes.data, wb.ctypes.data, wb.size, int(dtype), x.ctypes.data, n, dim, batch)


def rms_norm_in_place(x, weight, eps):
    """ops::rms_norm_in_place (ops.rs:59-61)."""
    _f32(x, "x"), _f32(weight, "weight")
    if weight.size < x.size:
        raise ValueError("weight shorter than x")
    call("hc_rms_norm_in_place", x.ctypes.data, weight.ctypes.data, x.size, float(eps))


def rms_norm(x, weight, eps):
    """ops::rms_norm (ops.rs:52-56)."""
    y = np.array(x, dtype=np.float32, copy=True)
    rms_norm_in_place(y, np.ascontiguousarray(weight, dtype=np.float32), eps)
    return y


def softmax_in_place(x):
    """ops::softmax_in_place (ops.rs:71-73)."""
    _f32(x, "x")
    call("hc_softmax_in_place", x.ctypes.data, x.size)


def softmax(x):
    """ops::softmax (ops.rs:64-68)."""
    y = np.array(x, dtype=np.float32, copy=True)
    softmax_in_place(y)
    return y


def silu_in_place(x):
    """ops::silu_in_place (ops.rs:81-83)."""
    _f32(x, "x")
    call("hc_silu_in_place", x.ctypes.data, x.size)


def silu(x):
    """ops::silu (ops.rs:76-78)."""
    y = np.array(x, dtype=np.float32, copy=True)
    silu_in_place(y)
    return y


def rope(q, k, head_dim, pos, theta):
    """ops::rope (ops.rs:86-99): rotates one head of q and k in place."""
    _f32(q, "q"), _f32(k, "k")
    if q.size < head_dim or k.size < head_dim:
        raise ValueError("q/k shorter than head_dim")
    call("hc_rope", q.ctypes.data, k.ctypes.data, head_dim, pos, float(theta))


def quantize_f32_to_q4_0(data):
    """quant::quantize_f32_to_q4_0 (quant.rs:108-117): floor(n/32) blocks of 18 bytes."""
    x = np.ascontiguousarray(data, dtype=np.float32).reshape(-1)
    nb = x.size // 32
    out = np.empty(nb * 18, dtype=np.uint8)
    if nb:
        call("hc_q4_0_quantize", x.ctypes.data, x.size, out.ctypes.data)
    return out.tobytes()


def dequantize_q4_0(q4_data):
    """quant::dequantize_q4_0 (quant.rs:120-132)."""
    qb = _bytes(q4_data)
    nb = qb.size // 18
    out = np.empty(nb * 32, dtype=np.float32)
    if nb:
        call("hc_q4_0_dequantize", qb.ctypes.data, qb.size, out.ctypes.data)
    return out
