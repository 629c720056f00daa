"""The converter's default path: Q4_0 packed on the GPU by
hc_q4_0_quantize_dev while converting (sft_convert.rs:248-267 quantizes on
the CPU).  The image must be byte-identical to the one built with the CPU
oracle's quantizer, a ragged tensor included."""
import numpy as np
import pytest

from hypno_b200 import convert as cv
from hypno_b200 import hypno_file as hf
from hypno_b200 import synth
from oracle import oracle as orc

from ._serve_common import SMALL
from .test_convert_cpu import f32, model_dir

pytestmark = pytest.mark.gpu


def test_gpu_quantized_conversion_is_byte_identical(cuda_device, tmp_path):
    cfg = dict(SMALL, embed="q4")
    tensors = {name: f32(synth.normal_host(7, name, int(np.prod(shape)), 0.5).reshape(shape))
               for name, shape, _ in synth.tensor_specs(cfg)}
    tensors["extra.ragged"] = f32(np.linspace(-2, 2, 4100, dtype=np.float32))
    config = {"architectures": ["LlamaForCausalLM"], "hidden_size": cfg["hidden"], "intermediate_size": cfg["inter"],
              "num_attention_heads": cfg["heads"], "num_key_value_heads": cfg["kv_heads"],
              "num_hidden_layers": cfg["layers"], "vocab_size": cfg["vocab"],
              "max_position_embeddings": cfg["max_pos"], "rope_theta": cfg["theta"]}
    d = model_dir(tmp_path, config, {"model.safetensors": tensors})
    on_gpu = cv.convert(d, str(tmp_path / "gpu.hypno"), hf.DT_Q4_0, device=cuda_device)
    on_cpu = cv.convert(d, None, hf.DT_Q4_0, quantize=orc.quantize_f32_to_q4_0)
    assert on_gpu.size == on_cpu.size and np.array_equal(on_gpu, on_cpu)
    assert hf.Manifest(on_gpu).tensors["extra.ragged"][1] == hf.DT_Q4_0
