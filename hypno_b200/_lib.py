"""ctypes binding of libhypno_cuda.so (the C ABI declared in include/hypno_cuda.h).

The shared library is the product: there is no Python or CPU fallback.  If
the library is missing or cannot be loaded, every entry point raises.
"""
import ctypes
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libhypno_cuda.so")

HC_OK = 0
ERR_NAMES = {
    -1: "HC_ERR_INVALID",
    -2: "HC_ERR_CUDA",
    -3: "HC_ERR_UNSUPPORTED",
    -4: "HC_ERR_FORMAT",
    -5: "HC_ERR_OOM",
    -6: "HC_ERR_TIMEOUT",
    -7: "HC_ERR_STATE",
}

DTYPE_FP32, DTYPE_FP16, DTYPE_Q8_0, DTYPE_Q4_0 = 0, 1, 2, 3
KV_FP32, KV_FP16 = 0, 1


class HypnoCudaError(RuntimeError):
    """A negative status returned by the C ABI, with hc_last_error()'s text."""

    def __init__(self, code, message):
        self.code = code
        super().__init__(f"{ERR_NAMES.get(code, code)}: {message}")


class HcConfig(ctypes.Structure):
    _fields_ = [
        ("hidden_size", ctypes.c_uint64),
        ("intermediate_size", ctypes.c_uint64),
        ("num_attention_heads", ctypes.c_uint64),
        ("num_key_value_heads", ctypes.c_uint64),
        ("num_hidden_layers", ctypes.c_uint64),
        ("vocab_size", ctypes.c_uint64),
        ("max_position_embeddings", ctypes.c_uint64),
        ("head_dim", ctypes.c_uint64),
        ("rms_norm_eps", ctypes.c_float),
        ("rope_theta", ctypes.c_float),
        ("embed_dtype", ctypes.c_uint32),
        ("lm_head_dtype", ctypes.c_uint32),
        ("lm_head_tied", ctypes.c_int32),
        ("tp_rank", ctypes.c_int32),
        ("tp_size", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


_P = ctypes.c_void_p
_SZ = ctypes.c_size_t
_U8P = ctypes.POINTER(ctypes.c_uint8)
_F32P = ctypes.POINTER(ctypes.c_float)
_U32P = ctypes.POINTER(ctypes.c_uint32)
_I32P = ctypes.POINTER(ctypes.c_int)
_I = ctypes.c_int
_U32 = ctypes.c_uint32
_U64 = ctypes.c_uint64
_F = ctypes.c_float

# name -> (restype, argtypes)
SIGNATURES = {
    "hc_last_error": (ctypes.c_char_p, []),
    "hc_version": (_I, []),
    "hc_set_device": (_I, [_I]),
    "hc_kernel_launches": (_U64, []),
    "hc_matmul_vec_auto": (_I, [_P, _P, _SZ, _U32, _P, _P, _SZ, _SZ]),
    "hc_batch_matmul": (_I, [_P, _P, _SZ, _U32, _P, _SZ, _SZ, _SZ]),
    "hc_rms_norm_in_place": (_I, [_P, _P, _SZ, _F]),
    "hc_softmax_in_place": (_I, [_P, _SZ]),
    "hc_silu_in_place": (_I, [_P, _SZ]),
    "hc_rope": (_I, [_P, _P, _SZ, _SZ, _F]),
    "hc_q4_0_quantize": (_I, [_P, _SZ, _P]),
    "hc_q4_0_dequantize": (_I, [_P, _SZ, _P]),
    "hc_q4_0_quantize_dev": (_I, [_P, _SZ, _P, _P]),
    "hc_q4_0_dequantize_dev": (_I, [_P, _SZ, _P, _P]),
    "hc_q4_matrix_upload": (_I, [_P, _SZ, _SZ, _SZ, ctypes.POINTER(_P)]),
    "hc_q4_matrix_from_dev": (_I, [_P, _SZ, _SZ, _SZ, _P, ctypes.POINTER(_P)]),
    "hc_q4_matrix_free": (_I, [_P]),
    "hc_q4_matmul_dev": (_I, [_P, _P, _SZ, _P, _P]),
    "hc_q4_matmul_noalloc": (_I, [_P, _P, _SZ, _P, _P]),
    "hc_model_load": (_I, [_P, _SZ, _I, _I, ctypes.POINTER(_P)]),
    "hc_model_config": (_I, [_P, ctypes.POINTER(HcConfig)]),
    "hc_model_free": (_I, [_P]),
    "hc_sync": (_I, [_P]),
    "hc_model_stream": (_P, [_P]),
    "hc_kv_alloc": (_I, [_P, _I, _I, _I, ctypes.POINTER(_P)]),
    "hc_kv_free": (_I, [_P]),
    "hc_kv_seq_len": (_I, [_P, _I, _I32P]),
    "hc_kv_set_pos": (_I, [_P, _I, _I]),
    "hc_prefill": (_I, [_P, _P, _I, _P, _I, _P]),
    "hc_decode_step": (_I, [_P, _P, _P, _P, _I, _P, _P]),
    "hc_decode_step_dev": (_I, [_P, _P, _P, _P, _I, _P, _P]),
    "hc_decode_step_phases": (_I, [_P, _P, _P, _P, _I, _P, _P]),
    "hc_phase_count": (_I, []),
    "hc_sample_dev": (_I, [_P, _SZ, _I, _I, _P, _P, _P, _P, _P, _P]),
    "hc_argmax_dev": (_I, [_P, _SZ, _I, _I, _I, _P, _P, _P]),
    "hc_phase_name": (ctypes.c_char_p, [_I]),
    "hc_comm_unique_id": (_I, [_P]),
    "hc_comm_init": (_I, [_P, _P, _I, _I, ctypes.c_double]),
    "hc_synth_normal_host": (_I, [_U64, _U64, _U64, _U64, _F, _P]),
    "hc_synth_normal_dev": (_I, [_U64, _U64, _U64, _U64, _F, _P, _P]),
}

_lib = None
_lock = threading.Lock()


def load():
    """Loads (once) and returns the ctypes handle; raises when the library is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m hypno_b200.build` "
                "(the sm_100a backend has no fallback)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(rc):
    """Raises HypnoCudaError for a negative status."""
    if rc != HC_OK:
        msg = load().hc_last_error()
        raise HypnoCudaError(rc, msg.decode(errors="replace") if msg else "")
    return rc


def call(name, *args):
    """Calls an int-returning entry point and raises on failure."""
    return check(getattr(load(), name)(*args))
