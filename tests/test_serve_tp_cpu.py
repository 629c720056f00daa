"""Continuous batching under tensor parallelism, host side: every rank runs
its own BatchScheduler over the same submissions, and each prefill / decode
call is a collective step (hc_prefill / hc_decode_step all-reduce across the
ranks).  Two gloo ranks check that the schedulers issue the same calls in the
same order (each call's signature is all-reduced and compared) and finish
with the same tokens."""
import datetime
import os
import socket

import numpy as np

from ._serve_common import SMALL, request_mix


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, size, port, q):
    try:
        import torch
        import torch.distributed as dist

        from hypno_b200.serve import BatchScheduler
        from oracle import oracle as orc
        from tests._serve_common import small_image

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=size, timeout=datetime.timedelta(seconds=60))
        om = orc.OracleModel(small_image())
        kvs = [om.new_kv(SMALL["max_pos"]) for _ in range(4)]
        mismatches = []

        def collective(sig):
            # every rank must be at the same call: the max of the signatures equals each rank's own
            t = torch.tensor(sig, dtype=torch.int64)
            m = t.clone()
            dist.all_reduce(m, op=dist.ReduceOp.MAX)
            if not torch.equal(m, t):
                mismatches.append((sig, m.tolist()))

        def prefill(slot, ids):
            collective([1, slot, int(ids.size), int(ids.astype(np.int64).sum())])
            kvs[slot].set_pos(0)
            return orc.batch_forward(om, ids, kvs[slot])

        def decode(slots, ids, want_logits):
            collective([2, len(slots), sum(slots), sum(int(i) for i in ids)])
            logits = [orc.model_forward(om, int(t), kvs[s]) for s, t in zip(slots, ids)]
            return None, np.array([orc.greedy(l) for l in logits])

        sch = BatchScheduler(prefill=prefill, decode=decode, eos_id=7, n_slots=4, max_pos=SMALL["max_pos"])
        for p, m in request_mix(SMALL["vocab"]):
            sch.submit(p, m)
        out = sch.run()
        result = {rid: (r.tokens, r.finish_reason) for rid, r in out.items()}
        dist.destroy_process_group()
        q.put((rank, result, mismatches, None))
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, None, None, repr(e)))


def test_two_rank_schedulers_take_the_same_steps():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    errs = [e for _, _, _, e in results if e]
    assert not errs, errs
    assert all(not mm for _, _, mm, _ in results), results
    a, b = (r for _, r, _, _ in sorted(results, key=lambda x: x[0]))
    assert a == b and len(a) == len(request_mix(SMALL["vocab"]))
