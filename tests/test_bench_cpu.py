"""Host-side pieces of bench.py that need no GPU: the workload description per
parallel layout, the clock-sample summary (samples taken before the timed
region do not count), and the argument rules of the timing contract."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_workload_config_layouts():
    one = bench.workload_config(1)
    assert one["parallelism"] == "single" and one["global_batch"] == 32 and one["seq_len"] == 2048
    tp = bench.workload_config(4, "tp")
    assert tp["parallelism"] == "tp4" and tp["global_batch"] == 32  # strong scaling: same 32 sequences
    dp = bench.workload_config(4, "dp")
    assert dp["parallelism"] == "replicas4" and dp["global_batch"] == 128  # one c4 job per rank
    c5 = bench.workload_config(8, "tp", "c5")
    assert c5["parallelism"] == "tp8" and c5["global_batch"] == 8 and c5["seq_len"] == 4096
    assert "hidden 8192, 80 layers" in c5["workload"] and "70B" in bench.metric_name("c5")
    c1 = bench.workload_config(1, "tp", "c1")
    assert c1["global_batch"] == 1 and "fit in L2" in c1["l2"]


def test_clock_summary_keeps_timed_samples_only():
    c = bench.ClockSampler(0, os.devnull)
    c.thread = object()  # as if the NVML thread ran
    c.rows = [(900.0, 1965.0, 0x0, 100.0), (1200.0, 1965.0, 0x8, 200.0)]  # before the timed region
    c.mark()
    c.rows += [(1965.0, 1965.0, 0x4, 900.0), (1950.0, 1965.0, 0x0, 950.0), (1965.0, 1965.0, 0x0, 940.0)]
    s = c.summary()
    assert s["samples"] == 3 and s["sm_mhz"] == 1965.0 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"]  # the hw_slowdown sample came before the mark


def test_clock_summary_without_timed_samples_uses_last():
    c = bench.ClockSampler(0, os.devnull)
    c.thread = object()
    c.rows = [(1965.0, 1965.0, 0x0, 120.0)]
    c.mark()
    s = c.summary()
    assert s["samples"] == 1 and s["sm_mhz"] == 1965.0


def test_clock_wait_first_is_bounded():
    c = bench.ClockSampler(0, os.devnull)
    c.thread = object()  # a thread that never samples
    c.wait_first(limit_s=0.05)
    assert c.rows == []


@pytest.mark.parametrize("argv", [["--warmup", "2"], ["--steps", "0"], ["--steps", "248", "--warmup", "3"]])
def test_timing_contract_arguments(argv):
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py")] + argv, capture_output=True, text=True,
                       timeout=120)
    assert r.returncode != 0 and ("warmup" in r.stderr or "steps" in r.stderr)


def test_reference_arm_inputs_without_gpu_library():
    """The reference arm builds its model from the oracle's copy of the seeded
    generator and quantizer: the same image bytes as the GPU library's host
    generator, without loading that library in the arm's process."""
    import numpy as np
    from hypno_b200 import synth
    from oracle import oracle as orc
    cfg = dict(hidden=256, inter=512, heads=4, kv_heads=2, layers=2, vocab=512, theta=10000.0, max_pos=64,
               embed="q4", lm_head="tied")
    a = synth.build_image(cfg, seed=3, quantize=orc.quantize_f32_to_q4_0,
                          normal=lambda sd, st, n, std: orc.synth_normal(sd, st, n, std))
    b = synth.build_image(cfg, seed=3, quantize=orc.quantize_f32_to_q4_0)
    assert np.array_equal(a, b)
    x = orc.synth_normal(5, synth.fnv1a64("w"), 4096, 0.02, offset=77)
    assert np.array_equal(x, synth.normal_host(5, "w", 4096, 0.02, offset=77))
    code = ("import sys, types; sys.argv = ['bench.py']; sys.path.insert(0, %r); import bench; "
            "bench.run_reference(types.SimpleNamespace(warmup=3, steps=1, layers=1, config='c4')); "
            "print('GPULIB', 'libhypno_cuda' in open('/proc/self/maps').read())" % ROOT)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600,
                       env=dict(os.environ, OMP_NUM_THREADS="1"))
    assert r.returncode == 0, r.stderr[-2000:]
    lines = r.stdout.strip().splitlines()
    import json
    line = json.loads(lines[-2])
    assert lines[-1] == "GPULIB False"
    assert line["impl"] == "reference" and line["config"]["layers"] == 1
    assert line["cpu_baseline"]["cores"] == (len(os.sched_getaffinity(0)))  # not torchrun's OMP_NUM_THREADS=1
