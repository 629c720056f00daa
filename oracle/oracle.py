"""ctypes wrapper of the CPU oracle (liboracle.so, built from hypno_oracle.c).

TEST INFRASTRUCTURE ONLY: the parity checker and the timed CPU baseline.
Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
--impl reference legs use it; the GPU product never does.  Parity status:
pinned by the reference's own unit tests re-expressed in tests/ and by f16
known-answer tests; beyond those, parity with the (unbuildable) Rust
reference is "unpinned".
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

_lib = None


def build():
    """Builds liboracle.so with the committed Makefile (gcc, no GPU)."""
    env = dict(os.environ)
    env.pop("CC", None)
    r = subprocess.run(["make", "-C", HERE, "-s"], capture_output=True, text=True, env=env)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{r.stdout}\n{r.stderr}")
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        src = os.path.join(HERE, "hypno_oracle.c")
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P, SZ, F = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_float
        sig = {
            "orc_f32_to_f16": (ctypes.c_uint16, [F]),
            "orc_f16_to_f32": (F, [ctypes.c_uint16]),
            "orc_q4_0_quantize": (None, [P, SZ, P]),
            "orc_q4_0_dequantize": (None, [P, SZ, P]),
            "orc_q4_0_extract_row": (None, [P, SZ, SZ, P]),
            "orc_matmul_q4_0": (None, [P, P, SZ, P, P, SZ, SZ]),
            "orc_matmul_f32": (None, [P, P, P, P, SZ, SZ]),
            "orc_matmul_f16": (None, [P, P, P, P, SZ, SZ]),
            "orc_rms_norm": (None, [P, P, SZ, F]),
            "orc_softmax": (None, [P, SZ]),
            "orc_silu": (None, [P, SZ]),
            "orc_rope": (None, [P, P, SZ, SZ, F]),
            "orc_model_open": (P, [P, SZ, ctypes.POINTER(ctypes.c_int)]),
            "orc_model_free": (None, [P]),
            "orc_model_config": (None, [P, P, P]),
            "orc_meta": (ctypes.c_char_p, [P, ctypes.c_char_p]),
            "orc_tensor_data": (ctypes.c_int, [P, ctypes.c_char_p, ctypes.POINTER(P),
                                               ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint32)]),
            "orc_kv_new": (P, [SZ, SZ, SZ, SZ]),
            "orc_kv_free": (None, [P]),
            "orc_kv_pos": (SZ, [P]),
            "orc_kv_set_pos": (None, [P, SZ]),
            "orc_kv_k": (P, [P]),
            "orc_kv_v": (P, [P]),
            "orc_model_forward": (ctypes.c_int, [P, P, ctypes.c_uint32, P]),
            "orc_batch_forward": (ctypes.c_int, [P, P, P, SZ, P]),
            "orc_num_threads": (ctypes.c_int, []),
            "orc_set_num_threads": (None, [ctypes.c_int]),
            "orc_synth_normal": (None, [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, F, P]),
            "orc_xorshift_next": (ctypes.c_uint64, [P]),
            "orc_xorshift_next_f32": (F, [P]),
            "orc_sample_token": (ctypes.c_uint32, [P, SZ, F, F, SZ, P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def synth_normal(seed, stream, n, std, offset=0):
    """The benchmark's seeded synthetic stream on the CPU (the same floats as
    hc_synth_normal_host); test-harness input generation, not a reference
    algorithm."""
    out = np.empty(n, dtype=np.float32)
    if n:
        lib().orc_synth_normal(seed, stream, offset, n, float(std), out.ctypes.data)
    return out


def use_all_cores():
    """Sets the oracle's OpenMP thread count to the cores this process may run
    on (torchrun exports OMP_NUM_THREADS=1 to every rank); returns it."""
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:
        n = os.cpu_count() or 1
    lib().orc_set_num_threads(n)
    return n


def f32_to_f16(x):
    return lib().orc_f32_to_f16(float(x))


def f16_to_f32(h):
    return lib().orc_f16_to_f32(int(h))


def quantize_f32_to_q4_0(data):
    """quant.rs:108-117."""
    x = _f32(data).reshape(-1)
    out = np.empty(x.size // 32 * 18, dtype=np.uint8)
    lib().orc_q4_0_quantize(x.ctypes.data, x.size, out.ctypes.data)
    return out.tobytes()


def dequantize_q4_0(q):
    """quant.rs:120-132."""
    qb = np.frombuffer(bytes(q), dtype=np.uint8) if not isinstance(q, np.ndarray) else q.view(np.uint8).reshape(-1)
    out = np.empty(qb.size // 18 * 32, dtype=np.float32)
    lib().orc_q4_0_dequantize(qb.ctypes.data, qb.size, out.ctypes.data)
    return out


def matmul_q4_0(w, x, n, m, bias=None):
    """kernels::matmul_q4_0 (AVX2 path), y[n]."""
    wb = np.frombuffer(bytes(w), dtype=np.uint8) if not isinstance(w, np.ndarray) else w.view(np.uint8).reshape(-1)
    xx = _f32(x)
    y = np.empty(n, dtype=np.float32)
    b = _f32(bias) if bias is not None else None
    lib().orc_matmul_q4_0(y.ctypes.data, wb.ctypes.data, wb.size, xx.ctypes.data,
                          b.ctypes.data if b is not None else None, n, m)
    return y


def batch_matmul_q4_0(w, X, n, m):
    """turbo::batch_matmul for Q4_0: one matvec per row of X [T, m]."""
    X = _f32(X).reshape(-1, m)
    return np.stack([matmul_q4_0(w, X[t], n, m) for t in range(X.shape[0])]) if X.shape[0] else np.zeros((0, n), np.float32)


def matmul_f32(w, x, n, m, bias=None):
    ww, xx = _f32(w), _f32(x)
    y = np.empty(n, dtype=np.float32)
    b = _f32(bias) if bias is not None else None
    lib().orc_matmul_f32(y.ctypes.data, ww.ctypes.data, xx.ctypes.data, b.ctypes.data if b is not None else None, n, m)
    return y


def matmul_f16(w16, x, n, m):
    ww = np.ascontiguousarray(w16, dtype=np.uint16)
    xx = _f32(x)
    y = np.empty(n, dtype=np.float32)
    lib().orc_matmul_f16(y.ctypes.data, ww.ctypes.data, xx.ctypes.data, None, n, m)
    return y


def rms_norm(x, w, eps):
    y = _f32(x).copy()
    ww = _f32(w)
    lib().orc_rms_norm(y.ctypes.data, ww.ctypes.data, y.size, float(eps))
    return y


def softmax(x):
    y = _f32(x).copy()
    lib().orc_softmax(y.ctypes.data, y.size)
    return y


def silu(x):
    y = _f32(x).copy()
    lib().orc_silu(y.ctypes.data, y.size)
    return y


def rope(q, k, head_dim, pos, theta):
    qq, kk = _f32(q).copy(), _f32(k).copy()
    lib().orc_rope(qq.ctypes.data, kk.ctypes.data, head_dim, pos, float(theta))
    return qq, kk


class OracleModel:
    """HypnoModel::open over an in-memory image + the forward passes."""

    def __init__(self, image):
        self._img = np.ascontiguousarray(image).view(np.uint8).reshape(-1)
        err = ctypes.c_int()
        h = lib().orc_model_open(self._img.ctypes.data, self._img.size, ctypes.byref(err))
        if not h:
            raise ValueError(f"oracle: malformed .hypno image (code {err.value})")
        self._h = h
        u = (ctypes.c_uint64 * 10)()
        f = (ctypes.c_float * 2)()
        lib().orc_model_config(h, u, f)
        (self.hidden, self.inter, self.nh, self.nkv, self.layers, self.vocab, self.max_pos, self.head_dim,
         self.n_tensors, self.n_meta) = list(u)
        self.eps, self.theta = f[0], f[1]

    def meta(self, key):
        v = lib().orc_meta(self._h, key.encode())
        return v.decode() if v is not None else None

    def tensor(self, name):
        p = ctypes.c_void_p()
        ln = ctypes.c_uint64()
        dt = ctypes.c_uint32()
        if lib().orc_tensor_data(self._h, name.encode(), ctypes.byref(p), ctypes.byref(ln), ctypes.byref(dt)) != 0:
            return None
        off = p.value - self._img.ctypes.data
        return self._img[off: off + ln.value], dt.value

    def new_kv(self, max_pos=None):
        return OracleKV(self, max_pos or self.max_pos)

    def close(self):
        if getattr(self, "_h", None):
            lib().orc_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class OracleKV:
    def __init__(self, model, max_pos):
        self.model = model
        self.max_pos = max_pos
        self._h = lib().orc_kv_new(model.layers, model.nkv, max_pos, model.head_dim)

    def seq_len(self):
        return lib().orc_kv_pos(self._h)

    def set_pos(self, p):
        lib().orc_kv_set_pos(self._h, p)

    def arrays(self):
        m = self.model
        n = m.layers * m.nkv * self.max_pos * m.head_dim
        shape = (m.layers, m.nkv, self.max_pos, m.head_dim)
        K = np.ctypeslib.as_array(ctypes.cast(lib().orc_kv_k(self._h), ctypes.POINTER(ctypes.c_float)), (n,))
        V = np.ctypeslib.as_array(ctypes.cast(lib().orc_kv_v(self._h), ctypes.POINTER(ctypes.c_float)), (n,))
        return K.reshape(shape), V.reshape(shape)

    def __del__(self):
        try:
            lib().orc_kv_free(self._h)
        except Exception:
            pass


def model_forward(model, token, kv):
    logits = np.empty(model.vocab, dtype=np.float32)
    rc = lib().orc_model_forward(model._h, kv._h, int(token), logits.ctypes.data)
    if rc != 0:
        raise RuntimeError(f"oracle model_forward failed ({rc})")
    return logits


def batch_forward(model, ids, kv):
    a = np.ascontiguousarray(ids, dtype=np.uint32).reshape(-1)
    logits = np.empty(model.vocab, dtype=np.float32)
    rc = lib().orc_batch_forward(model._h, kv._h, a.ctypes.data if a.size else None, a.size, logits.ctypes.data)
    if rc != 0:
        raise RuntimeError(f"oracle batch_forward failed ({rc})")
    return logits


class XorShift64:
    """run.rs:267-278 (state = seed.max(1))."""

    def __init__(self, seed):
        self.state = ctypes.c_uint64(max(int(seed), 1))

    def next_f32(self):
        return lib().orc_xorshift_next_f32(ctypes.byref(self.state))


def sample_token(logits, temperature, top_p, top_k, rng):
    """run.rs:203-251 (f32 step by step, sequential sums in index order)."""
    l = _f32(logits)
    return int(lib().orc_sample_token(l.ctypes.data, l.size, float(temperature), float(top_p), int(top_k),
                                      ctypes.byref(rng.state)))


def greedy(logits):
    """Argmax with Rust's Iterator::max_by tie rule: the last maximal index."""
    l = np.asarray(logits)
    mx = l.max()
    return int(np.nonzero(l == mx)[0][-1])
