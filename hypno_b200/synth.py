"""Seeded synthetic LLaMA-style models in the .hypno format, for the
benchmark configurations and the parity tests (there is no network for real
checkpoints).

Tensor names, shapes and metadata keys are the ones the reference converter
writes (sft_convert.rs:57-98) and the forward pass reads
(transformer.rs:281-528).  Values come from the seeded stream of
hc_synth_normal_* (a 12-term Irwin-Hall sum of 16-bit uniforms, mean 0,
variance std^2), keyed by the tensor name, so the host and the device
produce identical bytes.  Matrices larger than 4096 elements are quantized to
Q4_0 with the backend's bit-exact quantizer unless the configuration keeps
them FP32 (sft_convert.rs:11-17).
"""
import numpy as np

from . import hypno_file as hf
from ._lib import call

# The benchmark configurations (BASELINE.json "configs").
CONFIGS = {
    # SmolLM-135M shape, FP32 embedding, separate Q4_0 LM head.
    "c1": dict(hidden=576, layers=30, heads=9, kv_heads=3, inter=1536, vocab=49152, theta=10000.0,
               max_pos=2048, embed="fp32", lm_head="separate", prompt=128, decode=128, seqs=1, kv="fp32"),
    # TinyLlama-1.1B shape, all matrices Q4_0, LM head tied to the Q4_0 embedding.
    "c3": dict(hidden=2048, layers=22, heads=32, kv_heads=4, inter=5632, vocab=32000, theta=10000.0,
               max_pos=2048, embed="q4", lm_head="tied", prompt=512, decode=256, seqs=1, kv="fp32"),
    # Llama-3-8B shape, 32 sequences decoding together, fp16 KV.
    "c4": dict(hidden=4096, layers=32, heads=32, kv_heads=8, inter=14336, vocab=128256, theta=500000.0,
               max_pos=2304, embed="q4", lm_head="tied", prompt=2048, decode=256, seqs=32, kv="fp16"),
    # Llama-3.1-70B shape (tensor parallel).
    "c5": dict(hidden=8192, layers=80, heads=64, kv_heads=8, inter=28672, vocab=128256, theta=500000.0,
               max_pos=4608, embed="q4", lm_head="tied", prompt=4096, decode=512, seqs=8, kv="fp16"),
}

# the Q4_0 operator sweep.
SWEEP_NK = [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]
SWEEP_M = [1, 8, 64, 512]


def fnv1a64(s):
    h = 0xCBF29CE484222325
    for c in s.encode():
        h ^= c
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def normal_host(seed, name, n, std=0.02, offset=0):
    """The seeded stream for tensor `name` on the host (n float32 values)."""
    out = np.empty(n, dtype=np.float32)
    if n:
        call("hc_synth_normal_host", seed, fnv1a64(name), offset, n, float(std), out.ctypes.data)
    return out


def tensor_specs(cfg):
    """(name, shape, kind) for every tensor of a LLaMA-style model, kind in
    {"matrix", "norm", "embed", "lm_head"}."""
    H, I, nh, nkv, V = cfg["hidden"], cfg["inter"], cfg["heads"], cfg["kv_heads"], cfg["vocab"]
    hd = H // nh
    specs = [("model.embed_tokens.weight", (V, H), "embed"), ("model.norm.weight", (H,), "norm")]
    if cfg.get("lm_head", "tied") == "separate":
        specs.append(("lm_head.weight", (V, H), "lm_head"))
    for l in range(cfg["layers"]):
        p = f"model.layers.{l}."
        specs += [
            (p + "input_layernorm.weight", (H,), "norm"),
            (p + "post_attention_layernorm.weight", (H,), "norm"),
            (p + "self_attn.q_proj.weight", (nh * hd, H), "matrix"),
            (p + "self_attn.k_proj.weight", (nkv * hd, H), "matrix"),
            (p + "self_attn.v_proj.weight", (nkv * hd, H), "matrix"),
            (p + "self_attn.o_proj.weight", (H, nh * hd), "matrix"),
            (p + "mlp.gate_proj.weight", (I, H), "matrix"),
            (p + "mlp.up_proj.weight", (I, H), "matrix"),
            (p + "mlp.down_proj.weight", (H, I), "matrix"),
        ]
    return specs


def metadata(cfg):
    """The metadata strings sft_convert writes (sft_convert.rs:57-98)."""
    return [
        ("architecture", "LlamaForCausalLM"),
        ("hidden_size", str(cfg["hidden"])),
        ("intermediate_size", str(cfg["inter"])),
        ("num_attention_heads", str(cfg["heads"])),
        ("num_key_value_heads", str(cfg["kv_heads"])),
        ("num_hidden_layers", str(cfg["layers"])),
        ("vocab_size", str(cfg["vocab"])),
        ("max_position_embeddings", str(cfg["max_pos"])),
        ("rms_norm_eps", hf.rust_f64_display(cfg.get("eps", 1e-5))),
        ("rope_theta", hf.rust_f64_display(cfg["theta"])),
        ("weight_layout", "row_major"),
    ]


def _stored_dtype(cfg, kind, n):
    if kind == "norm":
        return hf.DT_FP32
    if kind == "embed" and cfg.get("embed", "q4") == "fp32":
        return hf.DT_FP32
    return hf.effective_dtype(hf.DT_Q4_0, n)


def build_image(cfg, seed=0, std=0.02, values=None, quantize=None, device=None, normal=None):
    """Returns the .hypno image (numpy uint8) of a synthetic model.

    values(name, n) -> float32 array overrides the seeded normal stream.
    quantize(f32 array) -> Q4_0 bytes overrides the backend quantizer (the
    parity-fixture script passes the oracle's, which is bit-identical).
    normal(seed, stream, n, std) -> float32 array overrides the host
    generator of the seeded stream (the CPU reference arm passes the
    oracle's copy, so it never loads the GPU library).
    device: a torch CUDA device to generate and quantize on (fast path for
    the multi-GB benchmark models); None generates on the host.
    """
    if device is not None and values is None and quantize is None:
        return _build_image_device(cfg, seed, std, device)
    if quantize is None:
        from .ops import quantize_f32_to_q4_0
        quantize = quantize_f32_to_q4_0
    specs = [(name, tuple(shape), _stored_dtype(cfg, kind, int(np.prod(shape)))) for name, shape, kind in
             tensor_specs(cfg)]
    # the image is allocated once and filled in place (one tensor's values
    # in flight), so the largest configuration fits in host memory
    img, offsets = hf.empty_image(metadata(cfg), [(nm, sh, dt, hf.data_bytes(dt, int(np.prod(sh))))
                                                  for nm, sh, dt in specs])
    for name, shape, dt in specs:
        n = int(np.prod(shape))
        if values is not None:
            data = values(name, n)
        elif normal is not None:
            data = normal(seed, fnv1a64(name), n, std)
        else:
            data = normal_host(seed, name, n, std)
        if dt == hf.DT_Q4_0:
            payload = np.frombuffer(quantize(data), dtype=np.uint8)
        else:
            payload = np.ascontiguousarray(data, dtype=np.float32).view(np.uint8)
        assert payload.size == hf.data_bytes(dt, n)
        img[offsets[name]: offsets[name] + payload.size] = payload
        del data, payload
    return img


def _device_payloads(cfg, seed, std, device):
    """(layout, iterator of (offset, host uint8 array)): every tensor generated
    and quantized on `device`, copied to one reused pinned host buffer."""
    import torch

    entries = []
    for name, shape, kind in tensor_specs(cfg):
        n = int(np.prod(shape))
        dt = _stored_dtype(cfg, kind, n)
        entries.append((name, tuple(shape), dt, hf.data_bytes(dt, n)))
    lay = hf.layout(metadata(cfg), entries)
    offsets = lay[1]

    def gen():
        stream = torch.cuda.current_stream(device)
        maxn = max(int(np.prod(s)) for _, s, _, _ in entries)
        maxb = max(b for _, _, _, b in entries)
        fbuf = torch.empty(maxn, dtype=torch.float32, device=device)
        qbuf = torch.empty(maxn // 32 * 18 + 64, dtype=torch.uint8, device=device)
        host = torch.empty(maxb, dtype=torch.uint8).pin_memory()
        try:
            for name, shape, dt, nbytes in entries:
                n = int(np.prod(shape))
                call("hc_synth_normal_dev", seed, fnv1a64(name), 0, n, float(std), fbuf.data_ptr(), stream.cuda_stream)
                if dt == hf.DT_Q4_0:
                    call("hc_q4_0_quantize_dev", fbuf.data_ptr(), n, qbuf.data_ptr(), stream.cuda_stream)
                    host[:nbytes].copy_(qbuf[:nbytes])
                else:
                    host[:nbytes].copy_(fbuf[:n].view(torch.uint8))
                yield offsets[name], host[:nbytes].numpy()
        finally:
            del fbuf, qbuf
            torch.cuda.empty_cache()

    return lay, gen()


def _build_image_device(cfg, seed, std, device):
    (head, _, total, _), payloads = _device_payloads(cfg, seed, std, device)
    img = np.zeros(total, dtype=np.uint8)
    img[: len(head)] = np.frombuffer(head, dtype=np.uint8)
    for off, data in payloads:
        img[off: off + data.size] = data
    return img


def write_image_file(cfg, path, seed=0, std=0.02, device=None):
    """Streams the .hypno image of a synthetic model to `path`, one tensor at a
    time (generated and quantized on the CUDA `device`), so models larger than
    host memory (c5: 39 GB) are written without holding the image; the bytes
    are those build_image returns."""
    import torch
    device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    (head, _, total, _), payloads = _device_payloads(cfg, seed, std, device)
    with open(path, "wb") as f:
        f.truncate(total)  # alignment gaps read as zeros
        f.write(head)
        for off, data in payloads:
            f.seek(off)
            f.write(memoryview(data))
    return path


def prompt_ids(vocab, T, seed=0):
    """Uniform-random prompt token ids in [0, vocab) (numpy PCG64)."""
    return np.random.Generator(np.random.PCG64(seed)).integers(0, vocab, size=T, dtype=np.int64).astype(np.uint32)


def model_bytes(cfg):
    """Q4_0 weight bytes read by one decode step (all matrices + LM head)."""
    total = 0
    for name, shape, kind in tensor_specs(cfg):
        n = int(np.prod(shape))
        if kind == "matrix" or kind == "lm_head":
            total += hf.data_bytes(hf.DT_Q4_0, n)
    if cfg.get("lm_head", "tied") == "tied":
        total += hf.data_bytes(hf.DT_Q4_0, cfg["vocab"] * cfg["hidden"])
    return total
