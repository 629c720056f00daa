#!/usr/bin/env python
"""Benchmark: Q4_0 decode throughput of the Llama-3-8B-shaped model
("c4"): 32 sequences, each with a 2048-token random
prompt prefilled, decoding greedily together with an fp16 KV cache.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one batched decode step of all 32 sequences (32 tokens).
  value  : whole-job decode tok/s, inputs resident in HBM (hc_decode_step_dev),
           device-timed with CUDA events on the model's stream, max over ranks.
  e2e    : the same through the host-buffer C ABI call (hc_decode_step: ids
           and sequence ids copied in from pinned host memory, greedy ids
           copied back every step), wall-clocked, max over ranks.
  prefill_tok_s : the 32 prompt prefills (hc_prefill), device-timed.
  roofline      : the dominant kernel (the Q4_0 matmul of the fused gate/up
           projection, N = 28672, K = 4096, M = 32) timed alone with CUDA events
           over rotating weight copies larger than L2, against the measured
           HBM copy bandwidth.
  cpu_baseline  : the CPU oracle (restatement of hypno's CPU path) decoding
           one sequence at context 2048 on the host cores (rank 0).
With --gpus N > 1 (torchrun) the model is tensor-parallel over the N ranks
(attention heads and FFN columns sharded, NCCL
all-reduce after o_proj / down_proj, vocabulary-sharded LM head): the same
32 sequences, strong scaling, value = 32 x steps / the slowest rank's time.
--parallel dp instead runs N independent replicas (weak scaling).
--impl reference times the CPU oracle on the same workload (rank 0 only).
"""
import argparse
import ctypes
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SHAPES = {"c1": "SmolLM-135M shape", "c3": "TinyLlama-1.1B shape", "c4": "Llama-3-8B shape",
          "c5": "Llama-3.1-70B shape"}
GOLDEN_STEPS = 32  # greedy steps compared with the oracle's fixture


def metric_name(name):
    from hypno_b200 import synth
    c = synth.CONFIGS[name]
    n = c["seqs"]
    return f"Q4_0 decode tok/s ({SHAPES[name]}, {n} sequence{'s' if n > 1 else ''} x {c['prompt']} context)"


UNIT = "tok/s"
# What the path computes in: Q4_0 weights; the tensor-core GEMMs multiply each
# weight as two exact fp16 terms by each activation as fp16 hi + lo with f32
# accumulation (an f32 dot product to ~1e-6); everything else is f32 (fp16 KV).
DTYPE = "q4_0 weights; fp16 hi+lo tensor-core operands (f32-exact products), f32 accumulate; fp16 KV"
FALLBACK_HBM_GBS = 6650.0


def _env_int(k, d):
    try:
        return int(os.environ.get(k, d))
    except ValueError:
        return d


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """SM clock / clock-event-reason sampling during the timed region: an NVML
    polling thread (every 5 ms, read-only queries) writing one CSV line per
    sample, so that even a timed region of a few tens of milliseconds has
    samples; nvidia-smi when NVML is unavailable."""

    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4))

    def __init__(self, index, path, period_s=0.005):
        self.path = path
        self.index = index
        self.period = period_s
        self.proc = None
        self.thread = None
        self.rows = []
        self.start = 0

    def wait_first(self, limit_s=2.0):
        """Wait (bounded) until the sampling thread has taken its first sample."""
        t_end = time.perf_counter() + limit_s
        while self.thread is not None and not self.rows and time.perf_counter() < t_end:
            time.sleep(0.001)

    def mark(self):
        """Start of the timed region: the summary keeps the samples from here on."""
        self.start = len(self.rows)

    def _handle(self, nv):
        try:
            import torch
            p = torch.cuda.get_device_properties(self.index)
            bus = f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
            return nv.nvmlDeviceGetHandleByPciBusId(bus.encode())
        except Exception:
            return nv.nvmlDeviceGetHandleByIndex(self.index)

    def __enter__(self):
        try:
            import threading
            import pynvml as nv
            nv.nvmlInit()
            h = self._handle(nv)
            smax = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            self.stop = threading.Event()

            def poll():
                while not self.stop.is_set():
                    try:
                        sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                        rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                        pw = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
                        self.rows.append((float(sm), float(smax), int(rs), pw))
                    except Exception:
                        pass
                    self.stop.wait(self.period)

            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
            return self
        except Exception:
            self.thread = None
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=5)
            try:
                with open(self.path, "w") as f:
                    f.write("sm_mhz,sm_max_mhz,reasons_mask,power_w\n")
                    for r in self.rows:
                        f.write(f"{r[0]:.0f},{r[1]:.0f},{r[2]:#x},{r[3]:.1f}\n")
            except OSError:
                pass
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.thread is not None:
            rows = self.rows[self.start:] or self.rows[-1:]
            if not rows:
                return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "source": "nvml"}
            sm = sorted(r[0] for r in rows)
            reasons = sorted({n for r in rows for n, bit in self.REASONS if r[2] & bit})
            return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons,
                    "samples": len(rows), "source": "nvml"}
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[4:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = sorted(r[0] for r in rows)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[2][i + 1].lower() == "active"})
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons,
                "samples": len(rows)}


def cuda_time_ms(stream_ptr, fn, reps):
    """Average milliseconds of fn() over reps launches, CUDA events recorded on
    the given raw stream (the stream the kernels run on)."""
    import torch
    s = torch.cuda.ExternalStream(stream_ptr) if stream_ptr else torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(s)
    for i in range(reps):
        fn(i)
    e1.record(s)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def graph_time_ms(fn, n, replays=3):
    """Average milliseconds per call of fn(i, stream) for i in range(n), the n
    calls captured once in a CUDA graph and replayed, CUDA events recorded on
    the replay stream; host launch overhead is not part of the number."""
    import torch
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    torch.cuda.synchronize()
    with torch.cuda.graph(g, stream=s, capture_error_mode="relaxed"):
        for i in range(n):
            fn(i, s.cuda_stream)
    cur = torch.cuda.current_stream()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    for _ in range(replays):
        g.replay()
    e1.record(cur)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / (replays * n)
    del g
    return ms


def roofline_gemv(dev, M=32, N=28672, K=4096, copies=0, reps=20):
    """Times the Q4_0 matmul of the fused gate/up shape over `copies` rotating
    weight matrices (together larger than L2: 256 MB or more) and returns the
    roofline dict."""
    import torch
    from hypno_b200 import synth
    from hypno_b200._lib import call
    mats = []
    if copies <= 0:
        copies = max(2, -(-256 * 2 ** 20 // (N * K // 32 * 18)))
    reps = max(reps, copies)
    w32 = torch.empty(N * K, dtype=torch.float32, device=dev)
    wq = torch.empty(N * K // 32 * 18, dtype=torch.uint8, device=dev)
    for c in range(copies):
        call("hc_synth_normal_dev", 100 + c, synth.fnv1a64("roofline.W"), 0, N * K, 0.02, w32.data_ptr(), None)
        call("hc_q4_0_quantize_dev", w32.data_ptr(), N * K, wq.data_ptr(), None)
        h = ctypes.c_void_p()
        call("hc_q4_matrix_from_dev", wq.data_ptr(), wq.numel(), N, K, None, ctypes.byref(h))
        mats.append(h)
    torch.cuda.synchronize()
    del w32, wq
    X = torch.empty(M * K, dtype=torch.float32, device=dev)
    call("hc_synth_normal_dev", 5, 5, 0, M * K, 1.0, X.data_ptr(), None)
    Y = torch.empty(M * N, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream().cuda_stream

    def run(i, st=stream):
        call("hc_q4_matmul_dev", mats[i % copies], X.data_ptr(), M, Y.data_ptr(), st)

    for i in range(6):
        run(i)
    ms = graph_time_ms(run, reps)
    for h in mats:
        call("hc_q4_matrix_free", h)
    algo = 0.5625 * N * K + 4.0 * M * K + 4.0 * M * N
    peak, src = measured_peaks()
    achieved = algo / (ms * 1e-3) / 1e9
    # DRAM bytes per launch need an ncu capture of this very run, which a
    # timed run does not take: the captured figure lives in profiles/
    return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "traffic": None,
            "kernel": f"q4_0 matmul N={N} K={K} M={M}", "algorithmic_bytes": int(algo), "copies": copies,
            "avg_launch_us": round(ms * 1e3, 2), "peak_source": f"{src} (hbm_gbs)"}


def q4_sweep(dev, reps=10):
    """Y = X W^T for (N, K) in the sweep and M in {1, 8, 64, 512},
    each timed as a CUDA graph of launches over rotating weight copies (> L2
    in total).
    M <= 64 is graded against HBM bandwidth, M = 512 against dense tensor peak."""
    import torch
    from hypno_b200 import synth
    from hypno_b200._lib import call
    peak_gbs, src = measured_peaks()
    peak_tf = None
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            peak_tf = float(json.load(f).get("bf16_tflops", 0)) or None
    peak_tf = peak_tf or 1590.0
    out = []
    stream = torch.cuda.current_stream().cuda_stream
    for (N, K) in synth.SWEEP_NK:
        wbytes = N * K // 32 * 18
        copies = max(2, -(-400 * 2 ** 20 // wbytes))  # > L2 (126 MB) in total for every shape
        w32 = torch.empty(N * K, dtype=torch.float32, device=dev)
        wq = torch.empty(wbytes, dtype=torch.uint8, device=dev)
        mats = []
        for c in range(copies):
            call("hc_synth_normal_dev", 200 + c, synth.fnv1a64(f"sweep.W.{N}x{K}"), 0, N * K, 0.02, w32.data_ptr(), None)
            call("hc_q4_0_quantize_dev", w32.data_ptr(), N * K, wq.data_ptr(), None)
            h = ctypes.c_void_p()
            call("hc_q4_matrix_from_dev", wq.data_ptr(), wbytes, N, K, None, ctypes.byref(h))
            mats.append(h)
        torch.cuda.synchronize()
        del w32, wq
        for M in synth.SWEEP_M:
            X = torch.empty(M * K, dtype=torch.float32, device=dev)
            call("hc_synth_normal_dev", 1, synth.fnv1a64(f"sweep.X.{M}x{K}"), 0, M * K, 1.0, X.data_ptr(), None)
            Y = torch.empty(M * N, dtype=torch.float32, device=dev)

            def run(i, st=stream):
                call("hc_q4_matmul_dev", mats[i % copies], X.data_ptr(), M, Y.data_ptr(), st)

            for i in range(3):
                run(i)
            ms = graph_time_ms(run, max(reps, copies))
            algo = 0.5625 * N * K + 4.0 * M * K + 4.0 * M * N
            flops = 2.0 * M * N * K
            row = {"N": N, "K": K, "M": M, "us": round(ms * 1e3, 2), "gbs": round(algo / (ms * 1e-3) / 1e9, 1),
                   "tflops": round(flops / (ms * 1e-3) / 1e12, 2)}
            if M <= 64:
                row["bound"], row["frac"] = "hbm", round(row["gbs"] / peak_gbs, 4)
            else:
                row["bound"], row["frac"] = "tensor", round(row["tflops"] / peak_tf, 4)
            out.append(row)
            del X, Y
        for h in mats:
            call("hc_q4_matrix_free", h)
        torch.cuda.empty_cache()
    return {"rows": out, "peaks": {"hbm_gbs": peak_gbs, "bf16_tflops": peak_tf, "source": src}}


def cpu_baseline(img, cfg, budget_s=12.0, max_tokens=24, name="c4"):
    """The oracle decoding one sequence at the prompt's context on the host cores."""
    from oracle import oracle as orc
    orc.use_all_cores()  # torchrun sets OMP_NUM_THREADS=1 for every rank
    om = orc.OracleModel(img)
    kv = om.new_kv(cfg["max_pos"])
    kv.set_pos(cfg["prompt"])
    orc.model_forward(om, 1, kv)  # warm-up
    n = 0
    t0 = time.perf_counter()
    while n < max_tokens and (time.perf_counter() - t0) < budget_s:
        orc.model_forward(om, 1 + n, kv)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": round(n / dt, 3), "unit": UNIT, "cores": orc.lib().orc_num_threads(), "kind": "port",
            "sample": f"{name} model_forward, 1 sequence at context {cfg['prompt']} (KV positions set, zero-filled), "
                      f"{n} tokens in {dt:.1f} s; the reference serialises sequences (serve.rs:175,193)"}


def prefill_roofline(cfg, tok_s, tp):
    """Prefill as a fraction of the sustained dense bf16 tensor peak: the
    useful flops per prompt token (2 x the matrix weights + the LM head on
    the last token only, ignored, + causal attention scores and weighted V at
    the prompt's mean context) per GPU."""
    H, I, L = cfg["hidden"], cfg["inter"], cfg["layers"]
    nh, nkv = cfg["heads"], cfg["kv_heads"]
    hd = H // nh
    w = L * (H * (nh + 2 * nkv) * hd + nh * hd * H + 3 * H * I)
    attn = L * 2 * 2 * nh * hd * (cfg["prompt"] / 2)
    fl = 2 * w + attn
    peak = None
    pth = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pth):
        with open(pth) as f:
            peak = float(json.load(f).get("bf16_tflops_sustained", 0)) or None
    src = "MEASURED_PEAKS.json bf16_tflops_sustained" if peak else "fallback 1400 TFLOP/s (sustained)"
    peak = peak or 1400.0
    ach = fl * tok_s / tp / 1e12
    return {"bound": "tensor", "achieved": round(ach, 1), "peak": peak, "unit": "TFLOP/s per GPU",
            "frac": round(ach / peak, 4), "flop_per_token": int(fl), "peak_source": src}


def golden_parity(model, cfg, name, img_sha, engine):
    """The oracle's committed fixture for this configuration
    (tests/golden/<config>.json: the prompt of the workload's sequence 0, or a
    short prompt for c5, then greedy steps), replayed through an FP32 KV cache:
    greedy ids over the first 32 steps and the relative error of the recorded
    logits.  Every rank runs it (tensor parallel collectives inside); rank 0
    reports."""
    path = os.path.join(ROOT, "tests", "golden", f"{name}.json")
    if cfg["layers"] != synth_layers(name) or not os.path.exists(path):
        return None
    with open(path) as f:
        g = json.load(f)
    steps = min(GOLDEN_STEPS, g["steps"])
    kv = engine.KVCache(model, n_seqs=1, max_pos=min(cfg["max_pos"], len(g["prompt"]) + steps + 1),
                        kv_dtype=engine.KV_FP32)
    logits = engine.batch_forward(model, np.array(g["prompt"], np.uint32), kv)
    worst, match, first_bad = 0.0, 0, None
    for st in range(steps):
        rec = g["records"][st]
        denom = max(1.0, max(abs(v) for _, v in rec["top"]))
        err = float(np.max(np.abs(logits[::g["stride"]].astype(np.float64) - np.array(rec["sample"]))))
        err = max([err] + [abs(float(logits[i]) - v) for i, v in rec["top"]]) / denom
        worst = max(worst, err)
        tok = int(np.nonzero(logits == logits.max())[0][-1])
        if tok == g["greedy"][st]:
            match += 1
        elif first_bad is None:
            first_bad = st
        if st + 1 < steps:
            lg, _ = engine.decode_step(model, kv, [0], [g["greedy"][st]])
            logits = lg[0]
    kv.close()
    return {"fixture": f"tests/golden/{name}.json (CPU oracle: {len(g['prompt'])}-token prompt + {steps} greedy steps)",
            "kv": "fp32", "image_sha256_match": None if img_sha is None else img_sha == g["image_sha256"],
            "greedy_match": f"{match}/{steps}", "first_mismatch_step": first_bad,
            "max_rel_err": float(f"{worst:.3e}"), "tolerance": 1e-3, "ok": match == steps and worst <= 1e-3}


def synth_layers(name):
    from hypno_b200 import synth
    return synth.CONFIGS[name]["layers"]


def workload_config(world, mode="tp", name="c4"):
    from hypno_b200 import synth
    c = synth.CONFIGS[name]
    par = "single" if world == 1 else (f"tp{world}" if mode == "tp" else f"replicas{world}")
    S, P = c["seqs"], c["prompt"]
    wgb = synth.model_bytes(c) / 1e9
    desc = (f"{name} decode: {SHAPES[name]} (hidden {c['hidden']}, {c['layers']} layers, {c['heads']}/{c['kv_heads']} "
            f"heads, im {c['inter']}, vocab {c['vocab']}), {S} sequence{'s' if S > 1 else ''} each prefilled with {P} "
            f"random tokens, greedy batched decode, {c['kv']} KV")
    return {"workload": desc, "model": SHAPES[name].lower().replace(" ", "-").replace(".", "") + "-random-q4_0",
            "global_batch": S if mode == "tp" else S * world, "seq_len": P, "parallelism": par,
            "l2": f"inputs larger than L2 ({wgb:.2f} GB of Q4_0 weights read per step)" if wgb > 0.126 else
                  f"weights ({wgb * 1e3:.0f} MB) fit in L2: decode reads them from L2 after the first step"}


def image_for(cfg, name, rank, world, dev, tp):
    """The synthetic .hypno image of the configuration.  c5 (39 GB) is written
    once to a file by rank 0 and memory-mapped by every rank (the page cache
    holds one copy, as the reference's mmap loader would); the others are
    built in host memory by each rank."""
    from hypno_b200 import synth
    if name != "c5":
        return synth.build_image(cfg, seed=0, device=dev)
    d = os.environ.get("HC_IMAGE_DIR", "/tmp")
    path = os.path.join(d, f"hypno_synth_{name}_l{cfg['layers']}_seed0.hypno")
    if rank == 0 and not os.path.exists(path):
        synth.write_image_file(cfg, path + ".part", seed=0, device=dev)
        os.replace(path + ".part", path)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    return np.memmap(path, dtype=np.uint8, mode="r")


def run_ours(args):
    import torch
    rank, world, local = _env_int("RANK", 0), _env_int("WORLD_SIZE", 1), _env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        # c5 writes its 39 GB image before the first barrier
        tmo = 900 if args.config == "c5" else 180
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=tmo), device_id=dev)
    from hypno_b200 import build, engine, synth
    from hypno_b200._lib import call, load
    if rank == 0:
        build.build()
    if dist:
        dist.barrier()
    lib = load()
    call("hc_set_device", local)
    name = args.config
    cfg = dict(synth.CONFIGS[name])
    if args.layers:
        cfg["layers"] = args.layers  # smaller model with the same per-layer kernels (profiling captures)
    S, P = cfg["seqs"], cfg["prompt"]
    tp = world > 1 and args.parallel == "tp"
    img = image_for(cfg, name, rank, world, dev, tp)
    torch.cuda.synchronize()
    t_load = time.perf_counter()
    model = engine.HypnoModel(img, rank if tp else 0, world if tp else 1)
    t_load = time.perf_counter() - t_load
    load = {"seconds": t_load, "image_gb": img.nbytes / 1e9}
    if tp:
        from hypno_b200 import tp as tpmod
        tpmod.join(model, rank, world)
    img_sha = None
    if rank == 0:
        import hashlib
        img_sha = hashlib.sha256(img.data).hexdigest()
    if rank != 0:
        del img
        img = None
    kv = engine.KVCache(model, n_seqs=S, max_pos=cfg["max_pos"],
                        kv_dtype=engine.KV_FP16 if cfg["kv"] == "fp16" else engine.KV_FP32)
    stream = model.stream

    # ---- prefill (32 prompts), device-timed
    prompts = [synth.prompt_ids(cfg["vocab"], P, seed=s) for s in range(S)]
    first = np.empty(S, np.uint32)
    import torch.cuda as tc
    e0, e1 = tc.Event(enable_timing=True), tc.Event(enable_timing=True)
    es = torch.cuda.ExternalStream(stream)
    # one untimed prefill first (first launches load the kernels, scratch and
    # tensor maps are set up), then the sequence is emptied again: a config
    # with one short prompt (c1, c3) would otherwise time mostly that set-up
    engine.batch_forward(model, prompts[0], kv, seq=0)
    kv.clear(0)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
        torch.cuda.synchronize()
    e0.record(es)
    torch.cuda.nvtx.range_push("timed_prefill")
    for s in range(S):
        logits = engine.batch_forward(model, prompts[s], kv, seq=s)
        first[s] = int(np.nonzero(logits == logits.max())[0][-1])
    torch.cuda.nvtx.range_pop()
    e1.record(es)
    torch.cuda.synchronize()
    prefill_ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([prefill_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        prefill_ms = float(t.item())
    prefill_tok_s = (1 if tp else world) * S * P / (prefill_ms * 1e-3)
    prefill_roof = prefill_roofline(cfg, S * P / (prefill_ms * 1e-3), world if tp else 1)

    # ---- decode, device-resident inputs
    seqs_dev = torch.arange(S, dtype=torch.int32, device=dev)
    ids_dev = torch.from_numpy(first.astype(np.int32)).to(dev)

    def step(_i):
        call("hc_decode_step_dev", model.handle, kv.handle, seqs_dev.data_ptr(), ids_dev.data_ptr(), S, None,
             ids_dev.data_ptr())

    def reset_pos():
        for s in range(S):
            kv.set_pos(P, s)

    for i in range(args.warmup):
        step(i)
    reset_pos()
    torch.cuda.synchronize()
    # The sampler starts (NVML init takes a different time in each process)
    # before the ranks line up: a rank that starts its timed region early
    # would otherwise spend the difference waiting in the first step's
    # cross-rank exchange, inside its own events.
    clk_dir = os.environ.get("HC_CLOCKS_DIR", "/tmp")  # where the per-rank clock samples are kept
    with ClockSampler(local, os.path.join(clk_dir, f"clocks_rank{rank}.csv")) as clk:
        clk.wait_first()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        clk.mark()
        l0 = lib.hc_kernel_launches()
        torch.cuda.nvtx.range_push("timed_decode")
        ms = cuda_time_ms(stream, step, args.steps) * args.steps
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        launches = lib.hc_kernel_launches() - l0
    if dist:
        dist.barrier()
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    jobs = 1 if tp else world  # tensor parallel: one model instance across all ranks
    value = jobs * S * args.steps / (ms * 1e-3)

    # ---- end to end through the host-buffer C ABI call
    reset_pos()
    h_seqs = torch.arange(S, dtype=torch.int32).pin_memory()
    h_ids = torch.from_numpy(first.astype(np.int32)).pin_memory()
    h_out = torch.empty(S, dtype=torch.int32).pin_memory()
    for _ in range(2):
        call("hc_decode_step", model.handle, kv.handle, h_seqs.data_ptr(), h_ids.data_ptr(), S, None,
             h_out.data_ptr())
        h_ids.copy_(h_out)
    reset_pos()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        call("hc_decode_step", model.handle, kv.handle, h_seqs.data_ptr(), h_ids.data_ptr(), S, None,
             h_out.data_ptr())
        h_ids.copy_(h_out)
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = {"value": round(jobs * S * args.steps / e2e_s, 2), "unit": UNIT,
           "h2d_bytes_per_step": 2 * 4 * S, "d2h_bytes_per_step": 4 * S}

    # ---- per-phase device time of a decode step (eager launches with an event
    # between phases, averaged over 3 steps; max over ranks per phase)
    phases = None
    if not args.no_phases:
        names = [lib.hc_phase_name(i).decode() for i in range(lib.hc_phase_count())]
        acc = (ctypes.c_float * len(names))()
        reset_pos()
        nrep = 3
        for _ in range(nrep):
            call("hc_decode_step_phases", model.handle, kv.handle, seqs_dev.data_ptr(), ids_dev.data_ptr(), S,
                 ids_dev.data_ptr(), acc)
        vals = torch.tensor([acc[i] / nrep for i in range(len(names))], device=dev)
        if dist:
            dist.all_reduce(vals, op=dist.ReduceOp.MAX)
        phases = {"ms_per_step": {n: round(float(v), 4) for n, v in zip(names, vals.tolist())},
                  "sum_ms": round(float(vals.sum()), 4),
                  "how": "one eager decode step (no CUDA graph) with a CUDA event between phases, mean of 3 steps, "
                         "max over ranks per phase"}

    # ---- parity of this very model against the oracle's fixture
    parity = None if args.no_parity else golden_parity(model, cfg, name, img_sha, engine)

    # ---- optional: the same 32 requests through the continuous-batching
    # scheduler (prefill of each prompt + `steps` greedy tokens each), wall-clocked
    serve = None
    if not args.no_serve:
        from hypno_b200.serve import BatchScheduler
        sch = BatchScheduler(model, kv)
        for s in range(S):
            sch.submit(prompts[s], args.steps)
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        done = sch.run()
        serve_s = time.perf_counter() - t0
        if dist:
            t = torch.tensor([serve_s], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            serve_s = float(t.item())
        ntok = sum(r.completion_tokens for r in done.values())
        serve = {"requests": S, "prompt_tokens": S * P, "completion_tokens": ntok, "seconds": round(serve_s, 3),
                 "completion_tok_s": round(ntok / serve_s, 1), "decode_rounds": sch.decode_steps}

    # model load: host image -> device weights (pinned chunked upload overlapped
    # with the Q4_0 repack), wall-clocked per rank, max over ranks
    lt = torch.tensor([load["seconds"]], device=dev)
    if dist:
        dist.all_reduce(lt, op=dist.ReduceOp.MAX)
    load = {"seconds": round(float(lt.item()), 3), "image_gb": round(load["image_gb"], 3),
            "image_gb_s": round(load["image_gb"] / float(lt.item()), 2),
            "how": "hc_model_load of the whole .hypno image from host memory; with tensor parallelism each rank "
                   "uploads its shard of it"}
    # the dominant kernel: this rank's fused gate/up projection at the batch
    rows_l = 2 * cfg["inter"] // (world if tp else 1)
    roof = roofline_gemv(dev, M=S, N=rows_l, K=cfg["hidden"]) if rank == 0 else None
    sweep = q4_sweep(dev) if rank == 0 and not args.no_sweep and name == "c4" else None
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:  # the CPU baseline is taken at N = 1 only
        cpu = cpu_baseline(img, cfg, name=name)
    if dist:
        dist.barrier()
    if rank == 0:
        line = {"metric": metric_name(name), "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
                "scaling": "strong" if tp else "weak", "vs_baseline": None, "dtype": DTYPE, "data": "synthetic",
                "config": dict(workload_config(world, "tp" if tp else "dp", name), layers=cfg["layers"]), "e2e": e2e,
                "gpu_launches": int(launches), "prefill_tok_s": round(prefill_tok_s, 1), "prefill": prefill_roof, "clocks": clk.summary(), "roofline": roof,
                "cpu_baseline": cpu, "q4_sweep": sweep}
        if serve is not None:
            line["serve"] = serve
        if phases is not None:
            line["decode_phases"] = phases
        line["model_load"] = load
        if parity is not None:
            line["parity"] = parity
        print(json.dumps(line), flush=True)
    kv.close()
    model.close()
    if dist:
        dist.destroy_process_group()


def run_reference(args):
    rank, world = _env_int("RANK", 0), _env_int("WORLD_SIZE", 1)
    if rank != 0:
        return
    from hypno_b200 import synth
    from oracle import oracle as orc
    cores = orc.use_all_cores()  # torchrun sets OMP_NUM_THREADS=1 for every rank
    name = args.config
    cfg = dict(synth.CONFIGS[name])
    if args.layers:
        cfg["layers"] = args.layers
    # built on the CPU with the oracle's generator and quantizer: this arm never
    # loads the GPU library
    img = synth.build_image(cfg, seed=0, quantize=orc.quantize_f32_to_q4_0,
                            normal=lambda sd, st, n, std: orc.synth_normal(sd, st, n, std))
    om = orc.OracleModel(img)
    kv = om.new_kv(cfg["max_pos"])
    kv.set_pos(cfg["prompt"])
    for i in range(args.warmup):
        orc.model_forward(om, 1 + i, kv)
    kv.set_pos(cfg["prompt"])
    t0 = time.perf_counter()
    for i in range(args.steps):
        orc.model_forward(om, 1 + i, kv)
    dt = time.perf_counter() - t0
    v = args.steps / dt
    cpu = {"value": round(v, 3), "unit": UNIT, "cores": cores, "kind": "port",
           "sample": f"each step = one model_forward of one sequence at context {cfg['prompt']} (the reference "
                     f"decodes sequences one at a time, serve.rs:175,193); {args.steps} steps in {dt:.1f} s"}
    line = {"impl": "reference", "metric": metric_name(name), "value": round(v, 3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 2),
            "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
            "dtype": "q4_0 weights, f32 compute (CPU restatement of hypno)", "data": "synthetic",
            "config": dict(workload_config(world, "tp", name), layers=cfg["layers"]),
            "cpu_baseline": cpu,
            "e2e": {"value": round(v, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--no-sweep", action="store_true", help="skip the configs[1] operator sweep report")
    ap.add_argument("--no-phases", action="store_true", help="skip the per-phase decode timing")
    ap.add_argument("--no-parity", action="store_true", help="skip the check against tests/golden/<config>.json")
    ap.add_argument("--config", default="c4", choices=["c4", "c5", "c1", "c3"],
                    help="BASELINE configuration (default c4, the headline; c5 writes its image under $HC_IMAGE_DIR)")
    ap.add_argument("--layers", type=int, default=0,
                    help="override the layer count (a small case for ncu captures; reported in config)")
    ap.add_argument("--no-serve", action="store_true",
                    help="skip timing the requests end to end through hypno_b200.serve.BatchScheduler")
    ap.add_argument("--parallel", default="tp", choices=["tp", "dp"],
                    help="N > 1: tensor parallel over the ranks (default) or independent replicas")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.steps < 1:
        ap.error("--steps must be >= 1")
    from hypno_b200 import synth
    room = synth.CONFIGS[args.config]["decode"] - 6
    if args.steps + args.warmup > room:
        ap.error(f"steps + warmup must fit the {room + 6} decode positions of the {args.config} workload")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
