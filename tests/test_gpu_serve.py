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
