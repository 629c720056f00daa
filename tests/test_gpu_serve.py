"""Continuous batching over the sm_100a backend: requests served together by
hypno_b200.serve.BatchScheduler (slots of one device KV cache, one
hc_decode_step per round over sequences at different positions, slots reused
after a request ends) give every request the greedy tokens and finish reason
of the oracle serving it alone (serve.rs:239-255)."""
import numpy as np
import pytest

from hypno_b200 import engine
from hypno_b200.serve import BatchScheduler, greedy_last_max
from oracle import oracle as orc

from ._serve_common import SMALL, request_mix, serial_generation, small_image

pytestmark = pytest.mark.gpu
TOL = 1e-3  # logits: max|gpu - ref| / max(1, max|ref|)


@pytest.fixture(scope="module")
def image():
    return small_image()


@pytest.mark.parametrize("n_slots,with_sampler", [(3, False), (16, False), (4, True)])
def test_scheduler_on_device_equals_serial_oracle(cuda_device, image, n_slots, with_sampler):
    om = orc.OracleModel(image)
    reqs = request_mix(SMALL["vocab"])
    probe, _ = serial_generation(om, reqs[6][0], 20, None, SMALL["max_pos"])
    eos = probe[3]
    ref_logits = [[] for _ in reqs]
    want = [serial_generation(om, p, m, eos, SMALL["max_pos"], seen=ref_logits[i]) for i, (p, m) in enumerate(reqs)]
    model = engine.HypnoModel(image)
    kv = engine.KVCache(model, n_seqs=n_slots, max_pos=SMALL["max_pos"], kv_dtype=engine.KV_FP32)
    got_logits = {}

    def sampler(logits, req):
        got_logits.setdefault(req.id, []).append(np.array(logits, copy=True))
        return greedy_last_max(logits)

    try:
        sch = BatchScheduler(model, kv, eos_id=eos, sampler=sampler if with_sampler else None)
        assert sch.n_slots == n_slots and sch.max_pos == SMALL["max_pos"]
        ids = [sch.submit(p, m) for p, m in reqs]
        out = sch.run()
        for rid, (toks, reason) in zip(ids, want):
            assert out[rid].tokens == toks, f"request {rid}: {out[rid].tokens} vs oracle {toks}"
            assert out[rid].finish_reason == reason, f"request {rid}"
        assert sch.decode_steps < sum(len(t) for t, _ in want)
        if with_sampler:  # the device logits of every pick, batched, against the request served alone
            for rid in ids:
                got, ref = got_logits.get(rid, []), ref_logits[rid]
                assert len(got) == len(ref), f"request {rid}"
                for step, (g, r) in enumerate(zip(got, ref)):
                    err = float(np.max(np.abs(g.astype(np.float64) - r)) / max(1.0, float(np.max(np.abs(r)))))
                    assert err <= TOL, f"request {rid} pick {step}: logits rel err {err:.3e}"
    finally:
        kv.close()
        model.close()


def test_scheduler_device_sampling(cuda_device, image):
    """Requests submitted with temperature / top_p / top_k / seed are sampled on
    the device (logits never leave it) next to greedy ones.  Replaying every
    request's emitted tokens through the oracle, each sampled token is the
    oracle's sample_token on the oracle's logits with the request's XorShift64
    sequence (serve.rs:279-305), or lies at a token boundary within rounding
    of the draw; greedy requests get the oracle's greedy tokens."""
    from ._sampling import boundary_margin
    om = orc.OracleModel(image)
    reqs = request_mix(SMALL["vocab"])
    params = [dict(temperature=0.8, top_p=0.9, top_k=40, seed=11 + i) if i % 2 == 0 else None
              for i in range(len(reqs))]
    params[3] = dict(temperature=1.2, top_p=1.0, top_k=0, seed=5)
    model = engine.HypnoModel(image)
    kv = engine.KVCache(model, n_seqs=4, max_pos=SMALL["max_pos"], kv_dtype=engine.KV_FP32)
    try:
        sch = BatchScheduler(model, kv)
        ids = [sch.submit(p, m, sampling=params[i]) for i, (p, m) in enumerate(reqs)]
        out = sch.run()
    finally:
        kv.close()
        model.close()
    loose = []
    for i, (p, m) in enumerate(reqs):
        toks = out[ids[i]].tokens
        assert len(toks) <= m
        okv = om.new_kv(SMALL["max_pos"])
        logits = orc.batch_forward(om, p, okv)
        rng = orc.XorShift64(params[i]["seed"]) if params[i] else None
        for st, t in enumerate(toks):
            if rng is not None:
                T, tp, tk = params[i]["temperature"], params[i]["top_p"], params[i]["top_k"]
                before = int(rng.state.value)
                want = orc.sample_token(logits, T, tp, tk, rng)
                if t != want:
                    loose.append((i, st, t, want, boundary_margin(logits, T, tp, tk, before, t, want)))
                    break  # the trajectories part here
            else:
                assert t == orc.greedy(logits), (i, st)
            if st + 1 < len(toks):
                logits = orc.model_forward(om, t, okv)
    assert all(x[-1] < 1e-4 for x in loose), loose
    assert len(loose) <= 1, loose
