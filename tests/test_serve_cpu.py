"""Continuous batching (hypno_b200/serve.py) on a host model: the scheduler's
bookkeeping must give every request exactly the tokens and finish reason of
the reference serving it alone (serve.rs:239-255), while its decodes run many
requests per step."""
import numpy as np
import pytest

from hypno_b200.serve import BatchScheduler, greedy_last_max
from oracle import oracle as orc

from ._serve_common import SMALL, request_mix, serial_generation, small_image


class HostBackend:
    """prefill/decode callables over one oracle cache per slot, recording the
    batches the scheduler forms."""

    def __init__(self, om, n_slots, max_pos):
        self.om = om
        self.kv = [om.new_kv(max_pos) for _ in range(n_slots)]
        self.batches = []

    def prefill(self, slot, ids):
        self.kv[slot].set_pos(0)
        return orc.batch_forward(self.om, ids, self.kv[slot])

    def decode(self, slots, ids, want_logits):
        self.batches.append(list(slots))
        logits = np.stack([orc.model_forward(self.om, int(t), self.kv[s]) for s, t in zip(slots, ids)])
        return (logits, None) if want_logits else (None, np.array([orc.greedy(l) for l in logits]))


@pytest.fixture(scope="module")
def om():
    return orc.OracleModel(small_image())


def _expected(om, reqs, eos_id):
    return [serial_generation(om, p, m, eos_id, SMALL["max_pos"]) for p, m in reqs]


@pytest.mark.parametrize("n_slots", [1, 3, 16])
def test_batched_equals_serial(om, n_slots):
    reqs = request_mix(SMALL["vocab"])
    # an EOS id that one request meets part-way (its 4th greedy token)
    probe, _ = serial_generation(om, reqs[6][0], 20, None, SMALL["max_pos"])
    eos = probe[3]
    want = _expected(om, reqs, eos)
    hb = HostBackend(om, n_slots, SMALL["max_pos"])
    sch = BatchScheduler(prefill=hb.prefill, decode=hb.decode, eos_id=eos, n_slots=n_slots,
                         max_pos=SMALL["max_pos"])
    ids = [sch.submit(p, m) for p, m in reqs]
    out = sch.run()
    assert sorted(out) == ids and sch.idle
    for rid, (toks, reason) in zip(ids, want):
        r = out[rid]
        assert r.tokens == toks, f"request {rid}"
        assert r.finish_reason == reason, f"request {rid}"
        assert r.completion_tokens == len(toks) and r.prompt_tokens == reqs[rid][0].size
    assert any(reason == "stop" and toks for toks, reason in want)          # EOS met part-way
    assert ("length", 5) in [(reason, len(toks)) for toks, reason in want]   # slot end (prompt 44 of 48)
    if n_slots > 1:
        assert max(len(b) for b in hb.batches) > 1                            # decodes were batched
        assert sch.decode_steps < sum(len(t) for t, _ in want)
    assert all(len(set(b)) == len(b) for b in hb.batches)


def test_sampler_gets_host_logits(om):
    reqs = request_mix(SMALL["vocab"])[:4]
    seen = []

    def sampler(logits, req):
        seen.append(req.id)
        return greedy_last_max(logits)

    hb = HostBackend(om, 2, SMALL["max_pos"])
    sch = BatchScheduler(prefill=hb.prefill, decode=hb.decode, sampler=sampler, n_slots=2, max_pos=SMALL["max_pos"])
    for p, m in reqs:
        sch.submit(p, m)
    out = sch.run()
    want = _expected(om, reqs, None)
    assert [out[i].tokens for i in range(len(reqs))] == [t for t, _ in want]
    assert len(seen) == sum(len(t) for t, _ in want)


def test_streaming_order_and_slot_reuse(om):
    hb = HostBackend(om, 2, SMALL["max_pos"])
    sch = BatchScheduler(prefill=hb.prefill, decode=hb.decode, n_slots=2, max_pos=SMALL["max_pos"])
    a = sch.submit(np.array([1, 2, 3], np.uint32), 2)
    b = sch.submit(np.array([4], np.uint32), 6)
    c = sch.submit(np.array([5, 6], np.uint32), 3)
    first = sch.step()
    assert [rid for rid, _ in first] == [a, b, a, b]  # a, b admitted (one token each), then one decode of both
    assert sch.finished[a].finish_reason == "length" and c in [r.id for r in sch.waiting]
    stream = list(first)
    while not sch.idle:
        stream += sch.step()
    assert sch.finished[c].slot == sch.finished[a].slot  # c took the slot a freed
    for rid in (a, b, c):
        assert [t for i, t in stream if i == rid] == sch.finished[rid].tokens


def test_submit_rejects():
    sch = BatchScheduler(prefill=lambda s, i: None, decode=lambda s, i, w: None, n_slots=1, max_pos=8)
    with pytest.raises(ValueError):
        sch.submit(np.zeros(9, np.uint32), 1)
    with pytest.raises(ValueError):
        sch.submit(np.zeros(2, np.uint32), -1)
    with pytest.raises(ValueError):
        BatchScheduler()
    with pytest.raises(ValueError):
        BatchScheduler(prefill=lambda s, i: None, decode=lambda s, i, w: None, n_slots=0, max_pos=8)


def test_planted_decode_error_is_seen(om):
    """The comparison has teeth: one wrong token planted in one batched decode
    (host model, one slot, one round) shows up in exactly the request that
    owned that slot."""
    reqs = request_mix(SMALL["vocab"])
    want = _expected(om, reqs, None)
    hb = HostBackend(om, 3, SMALL["max_pos"])
    calls = {"n": 0}

    def bad_decode(slots, ids, want_logits):
        logits, greedy = hb.decode(slots, ids, want_logits)
        calls["n"] += 1
        if calls["n"] == 3:
            greedy = greedy.copy()
            greedy[-1] = (int(greedy[-1]) + 1) % SMALL["vocab"]
            bad_decode.slot = slots[-1]
        return logits, greedy

    sch = BatchScheduler(prefill=hb.prefill, decode=bad_decode, n_slots=3, max_pos=SMALL["max_pos"])
    ids = [sch.submit(p, m) for p, m in reqs]
    out = sch.run()
    wrong = [rid for rid in ids if out[rid].tokens != want[rid][0]]
    assert len(wrong) == 1 and out[wrong[0]].slot == bad_decode.slot


def test_greedy_pick_follows_max_by():
    nan = float("nan")
    assert greedy_last_max(np.array([1.0, 3.0, 3.0, 2.0], np.float32)) == 2   # last of equal maxima
    assert greedy_last_max(np.array([], np.float32)) == 0
    assert greedy_last_max(np.array([1.0, nan, 0.5], np.float32)) == 2        # the fold moves past a NaN
    assert greedy_last_max(np.array([nan, 1.0, 0.5], np.float32)) == 1
    assert greedy_last_max(np.array([2.0, 1.0, nan], np.float32)) == 2
