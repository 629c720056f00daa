"""HuggingFace safetensors -> .hypno conversion, quantizing on the GPU.

Follows `sft_convert::convert` (sft_convert.rs:20-295): the metadata strings
taken from config.json in the same order and with the same defaults (:53-98,
`tokenizer_json` when tokenizer.json exists), every tensor of every
`*.safetensors` file (sorted by file name) in a table sorted by tensor name
(the BTreeMap of :101), payloads 64-byte aligned, the storage type chosen by
`effective_dtype` (:11-17: tensors of at most 4096 elements stay FP32 when
quantizing), BF16 and F16 sources widened to f32 first (:217-236, :335-339).

What changes is where the Q4_0 quantization runs: the reference quantizes
every matrix on one CPU thread (:260-263 -> quant.rs:108-117); here each
tensor goes to the GPU once and `hc_q4_0_quantize_dev` (bit-exact with
quant.rs) packs it there.  The stored bytes are identical, including the
zero tail block of a tensor whose length is not a multiple of 32 (its table
entry counts ceil(n/32) blocks, the quantizer writes floor(n/32)).

Two inputs the reference mishandles are refused instead: a tensor name that
appears in two files (the reference's offset arithmetic underflows,
:270-275) and a Q8_0 target (Q8_0 models are not loaded by this backend).
Tensors of an unsupported source dtype keep their table entry and zero
payload, as in the reference (:237-240 skips them with a warning).
"""
import json
import os
import struct
import sys

import numpy as np

from . import hypno_file as hf

__all__ = ["read_safetensors", "config_metadata", "convert"]

_SF_DTYPES = {"F32": np.float32, "F16": np.float16, "BF16": np.uint16}


def read_safetensors(path):
    """{name: (dtype string, shape tuple, raw little-endian bytes as uint8)}
    of one safetensors file (8-byte header length, JSON header, data)."""
    buf = np.fromfile(path, dtype=np.uint8)
    if buf.size < 8:
        raise ValueError(f"{path}: not a safetensors file (too short)")
    (n,) = struct.unpack("<Q", buf[:8].tobytes())
    if 8 + n > buf.size:
        raise ValueError(f"{path}: header length {n} beyond the file")
    header = json.loads(buf[8: 8 + n].tobytes().decode("utf-8"))
    data = buf[8 + n:]
    out = {}
    for name, d in header.items():
        if name == "__metadata__":
            continue
        b, e = d["data_offsets"]
        if not (0 <= b <= e <= data.size):
            raise ValueError(f"{path}: tensor {name} data offsets out of range")
        out[name] = (d["dtype"], tuple(int(s) for s in d["shape"]), data[b:e])
    return out


def _as_u64(v, default):
    # serde_json's as_u64: non-negative integers only (floats, bools, strings -> default)
    return v if isinstance(v, int) and not isinstance(v, bool) and v >= 0 else default


def _as_f64(v, default):
    return float(v) if isinstance(v, (int, float)) and not isinstance(v, bool) else default


def config_metadata(config, col_major=False, tokenizer_json=None):
    """The metadata list of sft_convert.rs:53-98 from a parsed config.json."""
    archs = config.get("architectures")
    arch = archs[0] if isinstance(archs, list) and archs and isinstance(archs[0], str) else "unknown"
    nh = _as_u64(config.get("num_attention_heads"), 0)
    meta = [
        ("architecture", arch),
        ("hidden_size", str(_as_u64(config.get("hidden_size"), 0))),
        ("intermediate_size", str(_as_u64(config.get("intermediate_size"), 0))),
        ("num_attention_heads", str(nh)),
        ("num_key_value_heads", str(_as_u64(config.get("num_key_value_heads"), nh))),
        ("num_hidden_layers", str(_as_u64(config.get("num_hidden_layers"), 0))),
        ("vocab_size", str(_as_u64(config.get("vocab_size"), 32000))),
        ("max_position_embeddings", str(_as_u64(config.get("max_position_embeddings"), 2048))),
        ("rms_norm_eps", hf.rust_f64_display(_as_f64(config.get("rms_norm_eps"), 1e-5))),
        ("rope_theta", hf.rust_f64_display(_as_f64(config.get("rope_theta"), 10000.0))),
        ("weight_layout", "col_major" if col_major else "row_major"),
    ]
    if tokenizer_json is not None:
        meta.append(("tokenizer_json", tokenizer_json))
    return meta


def _to_f32(dtype, raw):
    if dtype == "F32":
        return raw.view(np.float32)
    if dtype == "F16":
        return raw.view(np.float16).astype(np.float32)
    if dtype == "BF16":  # sft_convert::bf16_to_f32: the 16 bits become the top half
        return (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32)
    return None


def _device_quantizer(device):
    """Q4_0 packing on the GPU (hc_q4_0_quantize_dev); no host fallback."""
    import torch

    from ._lib import call
    if not torch.cuda.is_available():
        raise RuntimeError("convert: Q4_0 quantization runs on the GPU and no CUDA device is available")
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream(dev)

    def quantize(x):
        n = int(x.size)
        nbytes = n // 32 * 18
        if nbytes == 0:
            return b""
        xd = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(dev)
        out = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        call("hc_q4_0_quantize_dev", xd.data_ptr(), n, out.data_ptr(), stream.cuda_stream)
        return out.cpu().numpy().tobytes()
    return quantize


def convert(model_dir, out_path=None, target_dtype=hf.DT_Q4_0, col_major=False, quantize=None, device=None,
            log=None):
    """Converts a HuggingFace model directory; returns the image (numpy
    uint8) and writes it to `out_path` when given.

    quantize(f32 array) -> Q4_0 bytes replaces the GPU quantizer (tests pass
    the CPU oracle's, which is bit-identical)."""
    log = log or (lambda msg: print(msg, file=sys.stderr))
    if target_dtype not in (hf.DT_FP32, hf.DT_FP16, hf.DT_Q4_0):
        raise ValueError(f"convert: target dtype {target_dtype} is not supported (FP32, FP16 or Q4_0)")
    with open(os.path.join(model_dir, "config.json")) as f:
        config = json.load(f)
    tok_path = os.path.join(model_dir, "tokenizer.json")
    tokenizer_json = open(tok_path).read() if os.path.exists(tok_path) else None
    files = sorted(os.path.join(model_dir, n) for n in os.listdir(model_dir) if n.endswith(".safetensors"))
    if not files:
        raise ValueError(f"No .safetensors files found in {model_dir}")
    meta = config_metadata(config, col_major, tokenizer_json)

    sources = {}
    for path in files:
        for name, (dt, shape, raw) in read_safetensors(path).items():
            if name in sources:
                raise ValueError(f"convert: tensor {name} appears in more than one safetensors file")
            sources[name] = (dt, shape, raw)

    entries = []
    for name, (dt, shape, raw) in sources.items():
        n = int(np.prod(shape)) if shape else 1
        edt = hf.effective_dtype(target_dtype, n)
        entries.append((name, shape, edt, hf.data_bytes(edt, n)))
    img, offsets = hf.empty_image(meta, entries)

    if target_dtype == hf.DT_Q4_0 and quantize is None and any(e[2] == hf.DT_Q4_0 for e in entries):
        quantize = _device_quantizer(device)
    for name, shape, edt, nbytes in entries:
        dt, _, raw = sources[name]
        x = _to_f32(dt, raw)
        if x is None:
            log(f"Warning: unsupported dtype for tensor {name}")
            continue
        if edt == hf.DT_FP32:
            payload = np.ascontiguousarray(x, dtype=np.float32).view(np.uint8)
        elif edt == hf.DT_FP16:
            payload = x.astype(np.float16).view(np.uint8)
        else:
            payload = np.frombuffer(quantize(x), dtype=np.uint8)
        if payload.size > nbytes:
            raise ValueError(f"convert: tensor {name} has {payload.size} payload bytes for a {nbytes}-byte entry")
        off = offsets[name]
        img[off: off + payload.size] = payload
    if out_path is not None:
        img.tofile(out_path)
    return img


def main(argv=None):
    import argparse
    ap = argparse.ArgumentParser(description="HuggingFace safetensors -> .hypno (Q4_0 packed on the GPU)")
    ap.add_argument("model_dir")
    ap.add_argument("out_path")
    ap.add_argument("--dtype", default="q4_0", choices=["fp32", "fp16", "q4_0"])
    ap.add_argument("--col-major", action="store_true", help="write weight_layout = col_major (no transposition)")
    a = ap.parse_args(argv)
    dt = {"fp32": hf.DT_FP32, "fp16": hf.DT_FP16, "q4_0": hf.DT_Q4_0}[a.dtype]
    img = convert(a.model_dir, a.out_path, dt, a.col_major)
    print(f"Wrote {img.size} bytes to {a.out_path}")


if __name__ == "__main__":
    main()
