"""Generates the golden fixtures in tests/golden/ from the CPU oracle.

    python tests/golden/make_golden.py [--skip-c3]
    python tests/golden/make_golden.py --c4      (BASELINE configs[3] at full size; ~40 min on 8 cores)
    python tests/golden/make_golden.py --c5      (BASELINE configs[4] at full size; ~45 GB of host memory)

The reference (Rust) cannot be built in this image and ships no golden
vectors, so the fixtures come from the oracle (oracle/hypno_oracle.c, pinned
by the reference's own unit tests).  They freeze, per model:
  * the SHA-256 of the .hypno image (guards the synthetic generator),
  * the greedy ids after a prefill (argmax, last maximal index),
  * per step: the top-8 (id, logit), the top-1/top-2 margin, the sum and the
    sum of squares of the logits, and every 499th logit.
and, for BASELINE configs[1], the SHA-256 of the bit-exact Q4_0 packing of
each sweep weight tensor.  GPU tests compare the backend against these.
The c4 fixture is the full Llama-3-8B-shaped model (32 layers, hidden 4096):
sequence 0's 2048-token prompt, then the prefill logits and 32 greedy steps,
with the reference's FP32 KV cache (the oracle's faithful per-token path).
The c5 fixture is the full Llama-3.1-70B-shaped model (80 layers, hidden
8192, 39 GB): a 32-token prompt (seed 0), then the prefill logits and 32
greedy steps; the bench's 4096-token prompts would take the oracle hours.
"""
import argparse
import hashlib
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from hypno_b200 import hypno_file as hf  # noqa: E402
from hypno_b200 import synth  # noqa: E402
from oracle import oracle as orc  # noqa: E402
from tests import _models  # noqa: E402

STRIDE = 499


def step_record(logits):
    l = np.asarray(logits, np.float32)
    order = np.argsort(-l, kind="stable")[:8]
    s = np.sort(l)
    return {"top": [[int(i), float(l[i])] for i in order], "margin": float(s[-1] - s[-2]),
            "sum": float(l.astype(np.float64).sum()), "sumsq": float((l.astype(np.float64) ** 2).sum()),
            "sample": [float(v) for v in l[::STRIDE]], "greedy": orc.greedy(l)}


def image_sha256(img):
    """SHA-256 of the image bytes, hashed in place in 1 GiB pieces (the c5
    image is 39 GB: a copy would not fit beside it in host memory)."""
    h = hashlib.sha256()
    flat = np.ascontiguousarray(img).view(np.uint8).reshape(-1)
    for i in range(0, flat.size, 1 << 30):
        h.update(memoryview(flat[i:i + (1 << 30)]))
    return h.hexdigest()


def run_model(img, prompt, steps):
    om = orc.OracleModel(img)
    kv = om.new_kv()
    logits = orc.batch_forward(om, prompt, kv)
    recs = [step_record(logits)]
    tok = recs[-1]["greedy"]
    for _ in range(steps - 1):
        logits = orc.model_forward(om, tok, kv)
        recs.append(step_record(logits))
        tok = recs[-1]["greedy"]
    return recs


def model_fixture(name, img, prompt, steps):
    t0 = time.time()
    recs = run_model(img, prompt, steps)
    return {"model": name, "image_sha256": image_sha256(img), "image_bytes": int(img.size),
            "prompt": [int(t) for t in prompt], "steps": steps, "stride": STRIDE,
            "greedy": [r["greedy"] for r in recs], "records": recs, "oracle_seconds": round(time.time() - t0, 1)}


def sweep_fixture():
    out = {}
    for (N, K) in synth.SWEEP_NK:
        w = synth.normal_host(0, f"sweep.W.{N}x{K}", N * K, 0.02)
        q = orc.quantize_f32_to_q4_0(w)
        out[f"{N}x{K}"] = {"sha256": hashlib.sha256(q).hexdigest(), "bytes": len(q)}
        del w, q
    return {"generator": "hc_synth_normal_host(seed 0, stream fnv1a64('sweep.W.<N>x<K>'), std 0.02)",
            "tensors": out}


def c4_fixture():
    cfg = synth.CONFIGS["c4"]
    orc.use_all_cores()
    img = synth.build_image(cfg, seed=0, quantize=orc.quantize_f32_to_q4_0,
                            normal=lambda sd, st, n, std: orc.synth_normal(sd, st, n, std))
    return model_fixture("configs[3] (c4), sequence 0", img, synth.prompt_ids(cfg["vocab"], cfg["prompt"], seed=0), 33)


C5_PROMPT = 32


def c5_fixture():
    cfg = synth.CONFIGS["c5"]
    orc.use_all_cores()
    img = synth.build_image(cfg, seed=0, quantize=orc.quantize_f32_to_q4_0,
                            normal=lambda sd, st, n, std: orc.synth_normal(sd, st, n, std))
    return model_fixture(f"configs[4] (c5), a {C5_PROMPT}-token prompt", img,
                         synth.prompt_ids(cfg["vocab"], C5_PROMPT, seed=0), 33)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--skip-c3", action="store_true")
    ap.add_argument("--c4", action="store_true", help="only the full-size configs[3] fixture")
    ap.add_argument("--c5", action="store_true", help="only the full-size configs[4] fixture")
    args = ap.parse_args()
    if args.c5:
        v = c5_fixture()
        with open(os.path.join(HERE, "c5.json"), "w") as f:
            json.dump(v, f)
        print("c5 greedy =", v["greedy"], "oracle s =", v["oracle_seconds"])
        return
    if args.c4:
        v = c4_fixture()
        with open(os.path.join(HERE, "c4.json"), "w") as f:
            json.dump(v, f)
        print("c4 greedy =", v["greedy"], "oracle s =", v["oracle_seconds"])
        return
    fx = {}
    tiny = _models.reference_model_image(_models.TINY, 0.01, hf.DT_Q4_0)
    fx["tiny_q4"] = model_fixture("reference tiny model (turbo.rs:381-472), Q4_0", tiny,
                                  [1, 5, 10, 42, 100, 7, 3], 16)
    cfg = synth.CONFIGS["c1"]
    fx["c1"] = model_fixture("configs[0] (c1)", _models.synth_image("c1"),
                             synth.prompt_ids(cfg["vocab"], cfg["prompt"], seed=0), cfg["decode"])
    if not args.skip_c3:
        cfg = synth.CONFIGS["c3"]
        fx["c3"] = model_fixture("configs[2] (c3)", _models.synth_image("c3"),
                                 synth.prompt_ids(cfg["vocab"], cfg["prompt"], seed=0), 64)
    for k, v in fx.items():
        with open(os.path.join(HERE, f"{k}.json"), "w") as f:
            json.dump(v, f)
        print(k, "greedy[:16] =", v["greedy"][:16], "oracle s =", v["oracle_seconds"])
    sw = sweep_fixture()
    with open(os.path.join(HERE, "sweep_pack.json"), "w") as f:
        json.dump(sw, f, indent=1)
    print("sweep", sw)


if __name__ == "__main__":
    main()
