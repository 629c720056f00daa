"""Tensor-parallel host logic on CPU ranks (gloo, world size 2).

The sharding plan is checked against the oracle: every rank computes the
row-parallel / column-parallel pieces of a layer's projections from its
shard only, the pieces are combined with gloo collectives, and the result
must equal the unsharded oracle matvec.  No GPU is used."""
import os
import socket

import numpy as np
import pytest

from hypno_b200 import synth
from hypno_b200.tp import shard_plan

CFG = dict(hidden=256, heads=8, kv_heads=4, inter=512, vocab=1024)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, size, port, q):
    try:
        import torch
        import torch.distributed as dist
        from oracle import oracle as orc
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=size)
        H, im = CFG["hidden"], CFG["inter"]
        plan = shard_plan(CFG, rank, size)
        x = synth.normal_host(9, "tp.x", H, 1.0)
        act = synth.normal_host(9, "tp.act", im, 1.0)
        # o_proj [H, H]: column shard -> partial sums -> all-reduce
        wo = synth.normal_host(0, "tp.o", H * H, 0.02).reshape(H, H)
        c0, c1 = plan["o_cols"]
        part = orc.matmul_q4_0(orc.quantize_f32_to_q4_0(np.ascontiguousarray(wo[:, c0:c1])), x[c0:c1], H, c1 - c0)
        t = torch.from_numpy(part.copy())
        dist.all_reduce(t)
        full = orc.matmul_q4_0(orc.quantize_f32_to_q4_0(wo), x, H, H)
        # down_proj [H, im]: column shard of the FFN activations
        wd = synth.normal_host(0, "tp.down", H * im, 0.02).reshape(H, im)
        d0, d1 = plan["down_cols"]
        dpart = orc.matmul_q4_0(orc.quantize_f32_to_q4_0(np.ascontiguousarray(wd[:, d0:d1])), act[d0:d1], H, d1 - d0)
        td = torch.from_numpy(dpart.copy())
        dist.all_reduce(td)
        dfull = orc.matmul_q4_0(orc.quantize_f32_to_q4_0(wd), act, H, im)
        # LM head: vocabulary row shard -> all-gather
        V = CFG["vocab"]
        wl = synth.normal_host(0, "tp.lm", V * H, 0.02).reshape(V, H)
        v0, v1 = plan["vocab_rows"]
        lpart = orc.matmul_q4_0(orc.quantize_f32_to_q4_0(np.ascontiguousarray(wl[v0:v1])), x, v1 - v0, H)
        gathered = [torch.zeros(v1 - v0) for _ in range(size)]
        dist.all_gather(gathered, torch.from_numpy(lpart.copy()))
        lfull = orc.matmul_q4_0(orc.quantize_f32_to_q4_0(wl), x, V, H)
        ok = (np.allclose(t.numpy(), full, rtol=1e-5, atol=1e-6) and np.allclose(td.numpy(), dfull, rtol=1e-5, atol=1e-6)
              and np.array_equal(torch.cat(gathered).numpy(), lfull))
        dist.destroy_process_group()
        q.put((rank, ok, None))
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, False, repr(e)))


def test_shard_plan_covers_everything():
    for size in (1, 2, 4):
        plans = [shard_plan(CFG, r, size) for r in range(size)]
        for key, total in (("q_rows", CFG["hidden"]), ("ffn_rows", CFG["inter"]), ("vocab_rows", CFG["vocab"])):
            ranges = sorted(p[key] for p in plans)
            assert ranges[0][0] == 0 and ranges[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
    with pytest.raises(ValueError):
        shard_plan(CFG, 0, 3)


def test_two_rank_sharded_projections_match_oracle():
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
    assert all(ok for _, ok, _ in results), results
