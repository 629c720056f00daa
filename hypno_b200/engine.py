"""Model-level mirror of hypno's forward passes on the sm_100a backend.

    HypnoModel          loader::HypnoModel + transformer::HypnoConfig
                        (loader.rs:39-133, transformer.rs:42-63), resident in HBM
    KVCache             transformer::FlatKVCache (transformer.rs:89-184), for
                        n_seqs independent sequences
    batch_forward       turbo::batch_forward (turbo.rs:22-281)
    model_forward       transformer::model_forward with use_kv_cache = true
                        (transformer.rs:465-528)
    decode_step         model_forward batched over sequences (the serve path
                        without its global mutex)
    DeviceSampler       sample_token + XorShift64 (run.rs:203-278) on the device:
                        a decode step returns token ids, not logits

All of them call the C ABI (include/hypno_cuda.h); errors raise HypnoCudaError.
"""
import ctypes

import numpy as np

from ._lib import KV_FP16, KV_FP32, HcConfig, call, load

__all__ = ["HypnoModel", "KVCache", "batch_forward", "model_forward", "decode_step", "DeviceSampler", "KV_FP32",
           "KV_FP16"]


class HypnoModel:
    """A .hypno model uploaded to the current CUDA device.

    image: the file's bytes (bytes, bytearray, numpy uint8 array) or a path
    (memory-mapped read-only, like HypnoModel::open, loader.rs:39-148).
    The image is parsed and every weight uploaded once; the host buffer is not
    referenced after construction.
    """

    def __init__(self, image, tp_rank=0, tp_size=1):
        if isinstance(image, str):
            buf = np.memmap(image, dtype=np.uint8, mode="r")
        elif isinstance(image, (bytes, bytearray)):
            buf = np.frombuffer(image, dtype=np.uint8)
        else:
            buf = np.ascontiguousarray(image).view(np.uint8).reshape(-1)
        h = ctypes.c_void_p()
        call("hc_model_load", buf.ctypes.data, buf.size, tp_rank, tp_size, ctypes.byref(h))
        self._h = h
        cfg = HcConfig()
        call("hc_model_config", self._h, ctypes.byref(cfg))
        self.config = cfg

    @classmethod
    def open(cls, path, tp_rank=0, tp_size=1):
        return cls(path, tp_rank, tp_size)

    @property
    def handle(self):
        return self._h

    @property
    def stream(self):
        return load().hc_model_stream(self._h)

    def sync(self):
        call("hc_sync", self._h)

    def close(self):
        if getattr(self, "_h", None):
            load().hc_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class KVCache:
    """Device KV cache for n_seqs sequences of max_pos positions each."""

    def __init__(self, model, n_seqs=1, max_pos=0, kv_dtype=KV_FP32):
        h = ctypes.c_void_p()
        call("hc_kv_alloc", model.handle, n_seqs, max_pos, kv_dtype, ctypes.byref(h))
        self._h = h
        self.model = model
        self.n_seqs = n_seqs
        self.max_pos = max_pos if max_pos > 0 else int(model.config.max_position_embeddings)

    @property
    def handle(self):
        return self._h

    def seq_len(self, seq=0):
        """FlatKVCache::seq_len (transformer.rs:157)."""
        v = ctypes.c_int()
        call("hc_kv_seq_len", self._h, seq, ctypes.byref(v))
        return v.value

    def set_pos(self, pos, seq=0):
        """FlatKVCache::set_pos (transformer.rs:176)."""
        call("hc_kv_set_pos", self._h, seq, pos)

    def clear(self, seq=None):
        """FlatKVCache::clear (transformer.rs:118-121): positions back to 0."""
        for s in range(self.n_seqs) if seq is None else [seq]:
            self.set_pos(0, s)

    def close(self):
        if getattr(self, "_h", None):
            load().hc_kv_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def batch_forward(model, token_ids, kv, seq=0):
    """turbo::batch_forward: prefill `token_ids` into sequence `seq`; returns
    the last token's logits (zeros for an empty prompt)."""
    ids = np.ascontiguousarray(token_ids, dtype=np.uint32).reshape(-1)
    logits = np.empty(model.config.vocab_size, dtype=np.float32)
    call("hc_prefill", model.handle, kv.handle, seq, ids.ctypes.data if ids.size else None, ids.size,
         logits.ctypes.data)
    return logits


def model_forward(model, token_id, kv, seq=0):
    """transformer::model_forward(use_kv_cache = true): one token of sequence
    `seq` through all layers; returns its logits."""
    logits, _ = decode_step(model, kv, [seq], [token_id], want_logits=True, want_argmax=False)
    return logits[0]


def decode_step(model, kv, seqs, ids, want_logits=True, want_argmax=True):
    """One decode step for len(seqs) sequences at once.  Returns
    (logits [B, vocab] or None, greedy ids [B] or None); greedy = last maximal
    index (Iterator::max_by, run.rs:234-238)."""
    s = np.ascontiguousarray(seqs, dtype=np.int32).reshape(-1)
    t = np.ascontiguousarray(ids, dtype=np.uint32).reshape(-1)
    B = s.size
    logits = np.empty((B, model.config.vocab_size), dtype=np.float32) if want_logits else None
    am = np.empty(B, dtype=np.uint32) if want_argmax else None
    call("hc_decode_step", model.handle, kv.handle, s.ctypes.data, t.ctypes.data, B,
         logits.ctypes.data if logits is not None else None, am.ctypes.data if am is not None else None)
    return logits, am


class DeviceSampler:
    """sample_token (run.rs:203-251) with per-row XorShift64 states
    (run.rs:267-278), run on the device by hc_sample_dev.

    decode(...) runs one batched decode step with the logits kept in device
    memory and returns, per row, the greedy id (last maximal logit) and the
    sampled id; only 2 x B ids and B states cross to the host.  sample_host()
    samples one row of host logits (the prefill's)."""

    def __init__(self, model, max_rows):
        import torch
        self.model = model
        self.V = int(model.config.vocab_size)
        self.cap = int(max_rows)
        dev = torch.device("cuda", torch.cuda.current_device())
        self.dev = dev
        self.logits = torch.empty((self.cap, self.V), dtype=torch.float32, device=dev)
        self.greedy = torch.empty(self.cap, dtype=torch.int32, device=dev)
        self.out = torch.empty(self.cap, dtype=torch.int32, device=dev)

    def _sample(self, B, logits_ptr, temps, top_ps, top_ks, states):
        import torch
        t = torch.tensor(np.asarray(temps, np.float32), device=self.dev)
        p = torch.tensor(np.asarray(top_ps, np.float32), device=self.dev)
        k = torch.tensor(np.asarray(top_ks, np.int32), device=self.dev)
        st = torch.tensor(np.asarray(states, np.uint64).view(np.int64), device=self.dev)
        torch.cuda.current_stream(self.dev).synchronize()  # the copies above land before the model's stream reads them
        call("hc_sample_dev", logits_ptr, self.V, B, self.V, t.data_ptr(), p.data_ptr(), k.data_ptr(),
             st.data_ptr(), self.out.data_ptr(), self.model.stream)
        self.model.sync()
        return self.out[:B].cpu().numpy().astype(np.uint32), st.cpu().numpy().view(np.uint64)

    def decode(self, kv, seqs, ids, temps, top_ps, top_ks, states):
        """One decode step of len(seqs) sequences; returns (greedy ids,
        sampled ids, new states)."""
        import torch
        B = len(seqs)
        if B > self.cap:
            raise ValueError(f"{B} rows exceed the sampler's {self.cap}")
        s = torch.tensor(np.asarray(seqs, np.int32), device=self.dev)
        t = torch.tensor(np.asarray(ids, np.uint32).view(np.int32), device=self.dev)
        torch.cuda.current_stream(self.dev).synchronize()
        call("hc_decode_step_dev", self.model.handle, kv.handle, s.data_ptr(), t.data_ptr(), B,
             self.logits.data_ptr(), self.greedy.data_ptr())
        picked, new_states = self._sample(B, self.logits.data_ptr(), temps, top_ps, top_ks, states)
        return self.greedy[:B].cpu().numpy().astype(np.uint32), picked, new_states

    def sample_host(self, logits, temperature, top_p, top_k, state):
        """One row of host logits; returns (token id, new state)."""
        import torch
        self.logits[0].copy_(torch.from_numpy(np.ascontiguousarray(logits, np.float32)))
        torch.cuda.synchronize(self.dev)
        picked, st = self._sample(1, self.logits.data_ptr(), [temperature], [top_p], [top_k], [state])
        return int(picked[0]), int(st[0])
