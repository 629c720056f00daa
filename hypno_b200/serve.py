"""Continuous batching for the serve path.

The reference serves one request at a time: every request takes the global
`Mutex<ForwardBuffers>` (serve.rs:40-47,175,193) and runs
`generate_completion` (serve.rs:239-255): `prefill` (serve.rs:226-237, a
cleared cache and `turbo::batch_forward` of the prompt), then up to
`max_tokens` rounds of "pick the next token from the logits; stop on the EOS
id; count it; `model_forward` it".

`BatchScheduler` keeps those per-request semantics and removes the mutex: each
request owns one sequence slot of a multi-sequence `KVCache`, new requests are
prefilled into free slots as they arrive, and every `step()` advances all
running requests with ONE `hc_decode_step` over their slots (sequences at
different positions decode together).  A request finishes exactly when the
reference's loop would end, with the same token count and finish reason:

* "stop"   — the picked token is the EOS id (not counted, not emitted), or
             `max_tokens` is 0;
* "length" — `max_tokens` tokens emitted (serve.rs:253), or the slot's
             positions are used up (the reference's flat cache would index past
             its end here, transformer.rs:89-184).

Differences that do not change the emitted tokens: the reference runs
`model_forward` on its last emitted token although nothing reads those logits;
the scheduler skips that forward.  The default token choice is the greedy
last-maximal index (run.rs:234-238), taken on the device.  A request
submitted with `sampling=dict(temperature=, top_p=, top_k=, seed=)` is
sampled like serve.rs:279-305 (temperature, top-k, top-p, XorShift64 seeded
with `seed`), also on the device: the round's logits stay in device memory
and only token ids come back.  A `sampler(logits, request)` callable gets the
host logits instead.  Under tensor parallelism every rank runs the same
scheduler with the same submissions, so all ranks issue the same collective
steps.
"""
from collections import deque

import numpy as np

from . import engine

__all__ = ["Request", "BatchScheduler", "greedy_last_max"]


def greedy_last_max(logits):
    """Index picked by `max_by(|a, b| a.partial_cmp(b).unwrap_or(Equal))`
    (run.rs:234-238, serve.rs:300): the last index of the maximum; 0 for no
    logits.  A NaN compares Equal with everything, so the fold moves onto it
    and past it; that slow path runs only when a NaN is present."""
    v = np.asarray(logits).reshape(-1)
    if v.size == 0:
        return 0
    if not np.isnan(v).any():
        return int(np.flatnonzero(v == v.max())[-1])
    best = 0
    for i in range(1, v.size):      # fold: keep `best` only while it is strictly greater
        if not (v[best] > v[i]):
            best = i
    return best


class Request:
    """One completion: the `Generation` of serve.rs plus its tokens."""

    def __init__(self, rid, prompt_ids, max_tokens, sampling=None):
        self.id = rid
        self.prompt = np.ascontiguousarray(prompt_ids, dtype=np.uint32).reshape(-1)
        self.max_tokens = int(max_tokens)
        self.sampling = None        # (temperature, top_p, top_k) when sampled
        self.rng = 0                # XorShift64 state (XorShift64::new: seed.max(1))
        if sampling is not None:
            self.sampling = (float(sampling.get("temperature", 1.0)), float(sampling.get("top_p", 1.0)),
                             int(sampling.get("top_k", 0)))
            self.rng = max(int(sampling.get("seed", 0)) & 0xFFFFFFFFFFFFFFFF, 1)
        self.tokens = []            # emitted completion tokens
        self.finish_reason = None   # "stop" | "length" once done
        self.slot = -1
        self.feed = None            # token to run through the model next

    @property
    def prompt_tokens(self):
        return int(self.prompt.size)

    @property
    def completion_tokens(self):
        return len(self.tokens)

    @property
    def done(self):
        return self.finish_reason is not None


class BatchScheduler:
    """Admits requests into the sequence slots of `kv` and decodes all running
    requests together.

    `prefill(slot, prompt) -> logits` (the slot's cache restarted at position
    0) and `decode(slots, ids, want_logits) -> (logits or None, greedy ids or
    None)` default to the device engine
    (`engine.batch_forward`, `engine.decode_step`); they are parameters so the
    bookkeeping can be checked against a host model.
    """

    def __init__(self, model=None, kv=None, eos_id=None, sampler=None, prefill=None, decode=None,
                 n_slots=None, max_pos=None, device_sampler=None):
        if prefill is None or decode is None:
            if model is None or kv is None:
                raise ValueError("BatchScheduler needs a model and a KV cache, or prefill and decode callables")
            def prefill_slot(slot, ids):
                kv.set_pos(0, slot)   # prefill starts from a cleared cache (serve.rs:229, reset_cache)
                return engine.batch_forward(model, ids, kv, seq=slot)
            prefill = prefill or prefill_slot
            decode = decode or (lambda slots, ids, want_logits: engine.decode_step(
                model, kv, slots, ids, want_logits=want_logits, want_argmax=not want_logits))
            n_slots = kv.n_seqs if n_slots is None else n_slots
            max_pos = kv.max_pos if max_pos is None else max_pos
        if n_slots is None or max_pos is None or n_slots < 1 or max_pos < 1:
            raise ValueError("n_slots and max_pos must be positive")
        self._prefill, self._decode = prefill, decode
        self.eos_id = eos_id
        self.sampler = sampler
        # requests submitted with sampling parameters are sampled on the device
        self.device_sampler = device_sampler
        if self.device_sampler is None and model is not None and kv is not None and sampler is None:
            self._model, self._kv = model, kv
        else:
            self._model = self._kv = None
        self.n_slots, self.max_pos = int(n_slots), int(max_pos)
        self.free = list(range(self.n_slots - 1, -1, -1))   # pop() hands out slot 0 first
        self.waiting = deque()
        self.running = {}     # slot -> Request
        self.finished = {}    # id -> Request
        self.pos = [0] * self.n_slots
        self._next_id = 0
        self.decode_steps = 0

    # ---- submission -----------------------------------------------------
    def submit(self, prompt_ids, max_tokens, sampling=None):
        """Queues one request; returns its id.  A prompt that does not fit a
        slot is refused here (the reference's cache would overflow).
        `sampling`: None (greedy) or dict(temperature, top_p, top_k, seed)."""
        r = Request(self._next_id, prompt_ids, max_tokens, sampling)
        if r.sampling is not None and self.sampler is None and self.device_sampler is None:
            if self._model is None:
                raise ValueError("sampled requests need the device engine (or a sampler callable)")
            self.device_sampler = engine.DeviceSampler(self._model, self.n_slots)
        if r.max_tokens < 0:
            raise ValueError("max_tokens must be >= 0")
        if r.prompt_tokens > self.max_pos:
            raise ValueError(f"prompt of {r.prompt_tokens} tokens exceeds the {self.max_pos} positions of a slot")
        self._next_id += 1
        self.waiting.append(r)
        return r.id

    @property
    def idle(self):
        return not self.waiting and not self.running

    # ---- the reference loop body, one token -------------------------------
    def _pick(self, r, logits_row, greedy_id):
        if self.sampler is not None:
            return self.sampler(logits_row, r)
        if r.sampling is not None:  # prefill logits (host): one row through the device sampler
            tok, r.rng = self.device_sampler.sample_host(logits_row, *r.sampling, r.rng)
            return tok
        return int(greedy_id)

    def _advance(self, r, nxt, emitted):
        """serve.rs:246-251 for one picked token; returns True if the request
        needs another forward of `r.feed`."""
        if self.eos_id is not None and nxt == self.eos_id:
            r.finish_reason = "stop"
            return False
        r.tokens.append(nxt)
        emitted.append((r.id, nxt))
        if r.completion_tokens == r.max_tokens:
            r.finish_reason = "length"
            return False
        if self.pos[r.slot] >= self.max_pos:
            r.finish_reason = "length"   # slot full: no position left for the next forward
            return False
        r.feed = nxt
        return True

    def _retire(self, r):
        self.running.pop(r.slot, None)
        self.finished[r.id] = r
        self.free.append(r.slot)
        r.feed = None

    # ---- one scheduling round ---------------------------------------------
    def step(self):
        """Admits waiting requests into free slots (prefill each), then runs one
        batched decode over every running request.  Returns the (request id,
        token) pairs emitted by this call: the admitted requests' first
        tokens in admission order, then the decode's in slot order."""
        emitted = []
        while self.waiting and self.free:
            r = self.waiting.popleft()
            r.slot = self.free.pop()
            self.running[r.slot] = r
            if r.max_tokens == 0:            # the loop body never runs: "stop", no forward
                r.finish_reason = "stop"
                self._retire(r)
                continue
            logits = np.asarray(self._prefill(r.slot, r.prompt))
            self.pos[r.slot] = r.prompt_tokens
            if not self._advance(r, self._pick(r, logits, greedy_last_max(logits)), emitted):
                self._retire(r)
        slots = sorted(s for s, r in self.running.items() if r.feed is not None)
        if slots and self.sampler is None and any(self.running[s].sampling is not None for s in slots):
            # device sampling: logits stay on the device, ids and RNG states come back
            rs = [self.running[s] for s in slots]
            prm = [r.sampling if r.sampling is not None else (1.0, 1.0, 0) for r in rs]
            greedy, picked, states = self.device_sampler.decode(
                self._kv, slots, [r.feed for r in rs], [p[0] for p in prm], [p[1] for p in prm],
                [p[2] for p in prm], [r.rng for r in rs])
            self.decode_steps += 1
            for i, (s, r) in enumerate(zip(slots, rs)):
                self.pos[s] += 1
                if r.sampling is not None:
                    nxt, r.rng = int(picked[i]), int(states[i])
                else:
                    nxt = int(greedy[i])
                if not self._advance(r, nxt, emitted):
                    self._retire(r)
            return emitted
        if slots:
            ids = [self.running[s].feed for s in slots]
            logits, greedy = self._decode(slots, ids, self.sampler is not None)
            self.decode_steps += 1
            for i, s in enumerate(slots):
                r = self.running[s]
                self.pos[s] += 1
                row = logits[i] if logits is not None else None
                g = greedy[i] if greedy is not None else greedy_last_max(row)
                if not self._advance(r, self._pick(r, row, g), emitted):
                    self._retire(r)
        return emitted

    def run(self):
        """Steps until every submitted request has finished; returns them by id."""
        while not self.idle:
            self.step()
        return dict(self.finished)
