"""Model images used by the tests: the reference's own test models
(turbo.rs:381-472 tiny model, turbo.rs:616-711 TinyLlama-dims model) and the
seeded synthetic benchmark configs.  Q4_0 payloads come from the oracle's
quantizer, which is bit-identical to the backend's (tests/test_gpu_ops.py)."""
import numpy as np

from hypno_b200 import hypno_file as hf
from hypno_b200 import synth
from oracle import oracle as orc

TINY = dict(hidden=64, inter=172, heads=4, kv_heads=2, layers=2, vocab=1000, max_pos=512, theta=10000.0,
            lm_head="separate")
TINYLLAMA = dict(hidden=2048, inter=5632, heads=32, kv_heads=4, layers=22, vocab=32000, max_pos=2048,
                 theta=10000.0, lm_head="separate")


def linear_values(scale):
    """((i + 1) as f32) * scale per tensor, as the reference's add_tensor."""
    s = np.float32(scale)

    def f(name, n):
        return np.arange(1, n + 1, dtype=np.float32) * s
    return f


def reference_model_image(cfg, scale, dtype):
    """What sft_convert::convert writes for the reference's synthetic test
    model: every tensor filled with (i+1)*scale, matrices quantized to `dtype`
    subject to effective_dtype's <= 4096-element rule."""
    vals = linear_values(scale)
    tensors = []
    for name, shape, kind in synth.tensor_specs(cfg):
        n = int(np.prod(shape))
        data = vals(name, n)
        dt = hf.effective_dtype(dtype, n)
        if dt == hf.DT_Q4_0:
            payload = np.frombuffer(orc.quantize_f32_to_q4_0(data), dtype=np.uint8)
        else:
            payload = data.view(np.uint8)
        tensors.append((name, shape, dt, payload))
    return hf.write_image(synth.metadata(cfg), tensors)


def synth_image(name, seed=0):
    """A benchmark config built on the host with the oracle's quantizer."""
    cfg = synth.CONFIGS[name]
    return synth.build_image(cfg, seed=seed, quantize=orc.quantize_f32_to_q4_0)
