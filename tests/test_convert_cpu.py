"""The safetensors -> .hypno converter (hypno_b200/convert.py) on the host,
with the oracle's Q4_0 quantizer standing in for the GPU one (bit-identical:
tests/test_gpu_ops.py).  Mirrors the reference's own converter tests
(sft_convert.rs:366-456) and checks that a converted model is byte-identical
to the synthetic image the rest of the suite loads."""
import json

import numpy as np
import pytest

from hypno_b200 import convert as cv
from hypno_b200 import hypno_file as hf
from hypno_b200 import synth
from oracle import oracle as orc

from ._serve_common import SMALL

ORC_Q = orc.quantize_f32_to_q4_0


def write_safetensors(path, tensors):
    """tensors: {name: (dtype string, shape, raw bytes)} -> a safetensors file."""
    header, blobs, off = {}, [], 0
    for name, (dt, shape, raw) in tensors.items():
        raw = bytes(raw)
        header[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(len(h).to_bytes(8, "little") + h + b"".join(blobs))


def model_dir(tmp_path, config, files, tokenizer=None):
    d = tmp_path / "model"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(config))
    if tokenizer is not None:
        (d / "tokenizer.json").write_text(tokenizer)
    for fname, tensors in files.items():
        write_safetensors(d / fname, tensors)
    return str(d)


def f32(a):
    return ("F32", a.shape, np.ascontiguousarray(a, dtype=np.float32).tobytes())


def test_convert_and_validate(tmp_path):
    """sft_convert.rs:366-404."""
    cfg = {"architectures": ["LlamaForCausalLM"], "hidden_size": 64, "intermediate_size": 172,
           "num_attention_heads": 4, "num_key_value_heads": 2, "num_hidden_layers": 2, "vocab_size": 1000,
           "max_position_embeddings": 512, "rms_norm_eps": 1e-5, "rope_theta": 10000.0}
    data = np.arange(64, dtype=np.float32) * np.float32(0.1)
    d = model_dir(tmp_path, cfg, {"model.safetensors": {"weight": f32(data)}})
    out = str(tmp_path / "test.hypno")
    img = cv.convert(d, out, hf.DT_FP32)
    assert np.array_equal(np.fromfile(out, dtype=np.uint8), img)
    m = hf.Manifest(img)
    assert m.metadata["architecture"] == "LlamaForCausalLM" and m.metadata["hidden_size"] == "64"
    assert m.metadata["rms_norm_eps"] == "0.00001" and m.metadata["rope_theta"] == "10000"
    raw, dt = m.tensor_bytes("weight")
    assert dt == hf.DT_FP32 and np.array_equal(np.frombuffer(bytes(raw), np.float32), data)


def test_convert_q4_0(tmp_path):
    """sft_convert.rs:427-456: 128 x 64 elements -> 256 blocks of 18 bytes."""
    cfg = {"architectures": ["LlamaForCausalLM"], "hidden_size": 64, "intermediate_size": 172,
           "num_attention_heads": 4, "num_hidden_layers": 2, "vocab_size": 1000,
           "max_position_embeddings": 512, "rms_norm_eps": 1e-5}
    data = (np.arange(128 * 64, dtype=np.float32) * np.float32(0.1)).reshape(128, 64)
    d = model_dir(tmp_path, cfg, {"model.safetensors": {"weight": f32(data)}})
    img = cv.convert(d, None, hf.DT_Q4_0, quantize=ORC_Q)
    m = hf.Manifest(img)
    raw, dt = m.tensor_bytes("weight")
    assert dt == hf.DT_Q4_0 and len(raw) == 4608 and bytes(raw) == ORC_Q(data)
    assert m.metadata["num_key_value_heads"] == "4"     # defaults to num_attention_heads
    assert m.metadata["rope_theta"] == "10000"           # default


def test_converted_model_equals_synthetic_image(tmp_path):
    """A whole model written as two safetensors shards converts to exactly the
    bytes of synth.build_image (same metadata, tensor table, alignment and Q4_0
    packing)."""
    cfg = dict(SMALL, embed="q4", eps=1e-5)
    want = synth.build_image(cfg, seed=5, std=0.5, quantize=ORC_Q)
    tensors = {}
    for name, shape, kind in synth.tensor_specs(cfg):
        n = int(np.prod(shape))
        tensors[name] = f32(synth.normal_host(5, name, n, 0.5).reshape(shape))
    # two shards, names interleaved between them
    names = sorted(tensors)
    files = {"model-00001-of-00002.safetensors": {k: tensors[k] for k in names[0::2]},
             "model-00002-of-00002.safetensors": {k: tensors[k] for k in names[1::2]}}
    config = {"architectures": ["LlamaForCausalLM"], "hidden_size": cfg["hidden"], "intermediate_size": cfg["inter"],
              "num_attention_heads": cfg["heads"], "num_key_value_heads": cfg["kv_heads"],
              "num_hidden_layers": cfg["layers"], "vocab_size": cfg["vocab"],
              "max_position_embeddings": cfg["max_pos"], "rms_norm_eps": 1e-5, "rope_theta": cfg["theta"]}
    img = cv.convert(model_dir(tmp_path, config, files), None, hf.DT_Q4_0, quantize=ORC_Q)
    assert img.size == want.size and np.array_equal(img, want)
    om = orc.OracleModel(img)   # the oracle's loader (loader.rs) accepts it
    assert om.hidden == cfg["hidden"] and om.layers == cfg["layers"]


def test_source_dtypes_and_fp16_target(tmp_path):
    g = np.random.Generator(np.random.PCG64(1))
    x = g.standard_normal(5000).astype(np.float32)
    bf = (x.view(np.uint32) >> 16).astype(np.uint16)          # BF16 bits
    h = x.astype(np.float16)
    cfg = {"hidden_size": 8}
    files = {"m.safetensors": {"a_bf16": ("BF16", (5000,), bf.tobytes()), "b_f16": ("F16", (5000,), h.tobytes()),
                               "c_f32": f32(x), "d_i64": ("I64", (4,), np.arange(4, dtype=np.int64).tobytes())}}
    logs = []
    img = cv.convert(model_dir(tmp_path, cfg, files), None, hf.DT_FP16, log=logs.append)
    m = hf.Manifest(img)
    a, dta = m.tensor_bytes("a_bf16")
    assert dta == hf.DT_FP16
    assert np.array_equal(np.frombuffer(bytes(a), np.float16), (bf.astype(np.uint32) << 16).view(np.float32).astype(np.float16))
    b, _ = m.tensor_bytes("b_f16")
    assert np.array_equal(np.frombuffer(bytes(b), np.float16), h)
    c, _ = m.tensor_bytes("c_f32")
    assert np.array_equal(np.frombuffer(bytes(c), np.float16), x.astype(np.float16))
    dd, dtd = m.tensor_bytes("d_i64")                      # unsupported source: entry kept, payload zero
    assert dtd == hf.DT_FP16 and len(dd) == 8 and not any(bytes(dd)) and logs  # sized by the target dtype
    assert m.metadata["architecture"] == "unknown" and m.metadata["hidden_size"] == "8"
    assert m.metadata["num_hidden_layers"] == "0" and m.metadata["vocab_size"] == "32000"


def test_ragged_q4_tensor_and_metadata_formats(tmp_path):
    x = np.linspace(-3, 3, 4100, dtype=np.float32)        # 128 full blocks + 4 elements
    cfg = {"architectures": ["MistralForCausalLM"], "hidden_size": 4096.0, "rms_norm_eps": 1e-6,
           "rope_theta": 500000, "num_attention_heads": 32}
    img = cv.convert(model_dir(tmp_path, cfg, {"m.safetensors": {"w": f32(x)}}, tokenizer='{"v": 1}'), None,
                     hf.DT_Q4_0, col_major=True, quantize=ORC_Q)
    m = hf.Manifest(img)
    raw, dt = m.tensor_bytes("w")
    assert dt == hf.DT_Q4_0 and len(raw) == 129 * 18     # table counts ceil(n / 32) blocks
    assert bytes(raw[:128 * 18]) == ORC_Q(x) and not any(bytes(raw[128 * 18:]))
    md = m.metadata
    assert md["architecture"] == "MistralForCausalLM"
    assert md["hidden_size"] == "0"                       # a float is not a u64 in serde_json
    assert md["rms_norm_eps"] == "0.000001" and md["rope_theta"] == "500000"
    assert md["num_key_value_heads"] == "32" and md["weight_layout"] == "col_major"
    assert md["tokenizer_json"] == '{"v": 1}'
    assert list(md)[-1] == "tokenizer_json"


def test_refusals(tmp_path):
    cfg = {"hidden_size": 8}
    x = f32(np.zeros(8, np.float32))
    d = model_dir(tmp_path, cfg, {"a.safetensors": {"w": x}, "b.safetensors": {"w": x}})
    with pytest.raises(ValueError, match="more than one"):
        cv.convert(d, None, hf.DT_FP32)
    with pytest.raises(ValueError, match="not supported"):
        cv.convert(d, None, hf.DT_Q8_0)
    empty = tmp_path / "empty"
    empty.mkdir()
    (empty / "config.json").write_text("{}")
    with pytest.raises(ValueError, match="No .safetensors"):
        cv.convert(str(empty), None)


def test_gpu_quantizer_fails_loudly_without_cuda(tmp_path):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    x = f32(np.ones(8192, np.float32))
    d = model_dir(tmp_path, {"hidden_size": 8}, {"m.safetensors": {"w": x}})
    with pytest.raises(RuntimeError, match="GPU"):
        cv.convert(d, None, hf.DT_Q4_0)
