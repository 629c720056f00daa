"""Committed golden fixtures (tests/golden/*.json, made by
tests/golden/make_golden.py from the oracle) against the oracle itself (CPU,
regression of the checker) and against the sm_100a backend (GPU)."""
import hashlib
import json
import os

import numpy as np
import pytest

from hypno_b200 import engine, hypno_file as hf, synth
from oracle import oracle as orc
from tests import _models

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TOL = 1e-3


def load(name):
    with open(os.path.join(HERE, name)) as f:
        return json.load(f)


def image(name):
    if name == "tiny_q4":
        return _models.reference_model_image(_models.TINY, 0.01, hf.DT_Q4_0)
    return _models.synth_image(name)


def check_record(logits, rec, stride):
    ref_sample = np.array(rec["sample"], np.float64)
    denom = max(1.0, float(np.max(np.abs([v for _, v in rec["top"]]))))
    err = float(np.max(np.abs(logits[::stride].astype(np.float64) - ref_sample))) / denom
    assert err <= TOL, err
    for i, v in rec["top"]:
        assert abs(float(logits[i]) - v) / denom <= TOL
    return err


@pytest.mark.parametrize("name", ["tiny_q4", "c1"])
def test_oracle_reproduces_golden(name):
    g = load(f"{name}.json")
    img = image(name)
    assert hashlib.sha256(img.tobytes()).hexdigest() == g["image_sha256"]
    om = orc.OracleModel(img)
    kv = om.new_kv()
    logits = orc.batch_forward(om, np.array(g["prompt"], np.uint32), kv)
    steps = min(g["steps"], 16)
    for st in range(steps):
        rec = g["records"][st]
        assert orc.greedy(logits) == g["greedy"][st]
        assert np.array_equal(logits[::g["stride"]], np.array(rec["sample"], np.float32))
        if st + 1 < steps:
            logits = orc.model_forward(om, g["greedy"][st], kv)


@pytest.mark.gpu
@pytest.mark.parametrize("name,steps", [("tiny_q4", 16), ("c1", 128), ("c3", 64)])
def test_backend_matches_golden(cuda_device, name, steps):
    """Greedy ids identical to the oracle's for every recorded step (the bar
    is the first 32), logits within tolerance on the recorded samples."""
    g = load(f"{name}.json")
    img = image(name)
    assert hashlib.sha256(img.tobytes()).hexdigest() == g["image_sha256"]
    m = engine.HypnoModel(img)
    kv = engine.KVCache(m)
    logits = engine.batch_forward(m, np.array(g["prompt"], np.uint32), kv)
    worst, mism = 0.0, []
    for st in range(steps):
        rec = g["records"][st]
        worst = max(worst, check_record(logits, rec, g["stride"]))
        tok = orc.greedy(logits)
        if tok != g["greedy"][st]:
            mism.append((st, tok, g["greedy"][st], rec["margin"]))
            tok = g["greedy"][st]  # keep following the golden trajectory
        if st + 1 < steps:
            lg, _ = engine.decode_step(m, kv, [0], [tok])
            logits = lg[0]
    print(f"{name}: max sampled-logit rel err {worst:.2e}, greedy mismatches {mism}")
    assert not [x for x in mism if x[0] < 32], mism


@pytest.mark.gpu
@pytest.mark.parametrize("nk", list(load("sweep_pack.json")["tensors"]))
def test_sweep_pack_sha(cuda_device, nk):
    """configs[1] weights packed on the GPU hash to the oracle's bytes."""
    import torch
    from hypno_b200._lib import call
    N, K = map(int, nk.split("x"))
    w = torch.empty(N * K, dtype=torch.float32, device=cuda_device)
    call("hc_synth_normal_dev", 0, synth.fnv1a64(f"sweep.W.{N}x{K}"), 0, N * K, 0.02, w.data_ptr(), None)
    q = torch.empty(N * K // 32 * 18, dtype=torch.uint8, device=cuda_device)
    call("hc_q4_0_quantize_dev", w.data_ptr(), N * K, q.data_ptr(), None)
    torch.cuda.synchronize()
    assert hashlib.sha256(q.cpu().numpy().tobytes()).hexdigest() == load("sweep_pack.json")["tensors"][nk]["sha256"]


@pytest.mark.gpu
@pytest.mark.skipif(not os.path.exists(os.path.join(HERE, "c4.json")), reason="c4 fixture not generated")
def test_backend_matches_golden_c4(cuda_device):
    """BASELINE configs[3] at full size (Llama-3-8B shape, 32 layers): the
    device-built image hashes to the oracle's, and sequence 0's 2048-token
    prefill plus 32 greedy steps through an FP32 KV cache give the oracle's
    greedy ids, logits within tolerance on the recorded samples."""
    g = load("c4.json")
    cfg = synth.CONFIGS["c4"]
    img = synth.build_image(cfg, seed=0, device=cuda_device)
    assert hashlib.sha256(img.tobytes()).hexdigest() == g["image_sha256"]
    m = engine.HypnoModel(img)
    del img
    kv = engine.KVCache(m, n_seqs=1, max_pos=cfg["max_pos"], kv_dtype=engine.KV_FP32)
    logits = engine.batch_forward(m, np.array(g["prompt"], np.uint32), kv)
    worst, mism = 0.0, []
    for st in range(g["steps"]):
        rec = g["records"][st]
        worst = max(worst, check_record(logits, rec, g["stride"]))
        tok = orc.greedy(logits)
        if tok != g["greedy"][st]:
            mism.append((st, tok, g["greedy"][st], rec["margin"]))
            tok = g["greedy"][st]
        if st + 1 < g["steps"]:
            lg, _ = engine.decode_step(m, kv, [0], [tok])
            logits = lg[0]
    kv.close()
    m.close()
    print(f"c4: max sampled-logit rel err {worst:.2e}, greedy mismatches {mism}")
    assert not mism, mism
