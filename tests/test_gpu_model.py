"""Model-level parity of the sm_100a backend (hc_prefill / hc_decode_step)
against the CPU oracle's batch_forward / model_forward, through the C ABI.

Bars (north_star): logits within max|gpu - ref| / max(1, max|ref|) <= 1e-3,
greedy ids identical for the first 32 steps; the top-1/top-2 margin is
reported so a flip on a sub-tolerance margin is visible."""
import numpy as np
import pytest

from hypno_b200 import engine, hypno_file as hf, synth
from hypno_b200._lib import HypnoCudaError
from oracle import oracle as orc
from tests import _models

pytestmark = pytest.mark.gpu
TOL = 1e-3


def rel_err(a, ref):
    return float(np.max(np.abs(a.astype(np.float64) - ref)) / max(1.0, float(np.max(np.abs(ref)))))


def margin(l):
    s = np.sort(l)
    return float(s[-1] - s[-2])


def run_greedy_gpu(model, prompt, steps, kv_dtype=engine.KV_FP32, max_pos=0):
    kv = engine.KVCache(model, 1, max_pos, kv_dtype)
    logits = engine.batch_forward(model, prompt, kv)
    out_logits = [logits]
    ids = [orc.greedy(logits)]
    for _ in range(steps - 1):
        lg, am = engine.decode_step(model, kv, [0], [ids[-1]])
        assert int(am[0]) == orc.greedy(lg[0])
        out_logits.append(lg[0])
        ids.append(int(am[0]))
    return ids, out_logits


def run_greedy_oracle(om, prompt, steps):
    kv = om.new_kv()
    logits = orc.batch_forward(om, prompt, kv)
    out_logits = [logits]
    ids = [orc.greedy(logits)]
    for _ in range(steps - 1):
        logits = orc.model_forward(om, ids[-1], kv)
        out_logits.append(logits)
        ids.append(orc.greedy(logits))
    return ids, out_logits


def compare(gpu, ref, label):
    gids, glog = gpu
    rids, rlog = ref
    worst = 0.0
    for step, (g, r) in enumerate(zip(glog, rlog)):
        e = rel_err(g, r)
        worst = max(worst, e)
        assert e <= TOL, f"{label}: step {step} logits rel err {e:.3e}"
    first_diff = next((i for i, (a, b) in enumerate(zip(gids, rids)) if a != b), None)
    assert first_diff is None, (f"{label}: greedy ids diverge at step {first_diff} "
                                f"(oracle margin there {margin(rlog[first_diff]):.3e})")
    print(f"{label}: max logits rel err {worst:.3e}, min top-2 margin {min(margin(r) for r in rlog):.3e}")


@pytest.fixture(scope="module")
def tiny_images():
    return {dt: _models.reference_model_image(_models.TINY, 0.01, dt) for dt in (hf.DT_FP32, hf.DT_Q4_0)}


@pytest.mark.parametrize("dt", [hf.DT_FP32, hf.DT_Q4_0])
def test_tiny_reference_model(cuda_device, tiny_images, dt):
    """The reference's own test model (turbo.rs:381-472) in FP32 and Q4_0
    (its Q4_0 form mixes FP32 q/k/v/o with Q4_0 matrices whose width 172 is
    not a multiple of 32)."""
    img = tiny_images[dt]
    m = engine.HypnoModel(img)
    om = orc.OracleModel(img)
    prompt = np.array([1, 5, 10, 42, 100, 7, 3], np.uint32)
    compare(run_greedy_gpu(m, prompt, 12), run_greedy_oracle(om, prompt, 12), f"tiny dt={dt}")


def test_tiny_batch_equals_sequential_on_gpu(cuda_device, tiny_images):
    """turbo.rs:474-568 on the GPU: prefill then decode == all-decode."""
    m = engine.HypnoModel(tiny_images[hf.DT_FP32])
    prompt, nxt = [1, 5, 10, 42], 100
    kv_a = engine.KVCache(m)
    engine.batch_forward(m, prompt, kv_a)
    a = engine.model_forward(m, nxt, kv_a)
    kv_b = engine.KVCache(m)
    for t in prompt:
        engine.model_forward(m, t, kv_b)
    b = engine.model_forward(m, nxt, kv_b)
    assert np.max(np.abs(a - b)) < 1e-5
    assert kv_a.seq_len() == kv_b.seq_len() == 5


def test_edge_cases(cuda_device, tiny_images):
    m = engine.HypnoModel(tiny_images[hf.DT_FP32])
    kv = engine.KVCache(m, n_seqs=2, max_pos=8)
    out = engine.batch_forward(m, [], kv)  # turbo.rs:255-258
    assert np.all(out == 0) and kv.seq_len() == 0
    with pytest.raises(HypnoCudaError):
        engine.batch_forward(m, list(range(9)), kv)  # past capacity
    with pytest.raises(HypnoCudaError):
        engine.decode_step(m, kv, [0, 0], [1, 2])  # same sequence twice
    with pytest.raises(HypnoCudaError):
        engine.decode_step(m, kv, [0], [1000])  # id >= vocab
    engine.batch_forward(m, list(range(8)), kv)
    with pytest.raises(HypnoCudaError) as e:
        engine.decode_step(m, kv, [0], [1])  # cache full
    assert e.value.code == -7
    kv.clear(0)
    assert kv.seq_len(0) == 0
    with pytest.raises(HypnoCudaError):
        engine.HypnoModel(np.frombuffer(b"HYPX" + b"\0" * 60, np.uint8))


@pytest.fixture(scope="module")
def c1_image():
    return _models.synth_image("c1")


def test_c1_greedy_32_steps(cuda_device, c1_image):
    """128-token prompt + greedy decode, logits and ids vs oracle."""
    cfg = synth.CONFIGS["c1"]
    prompt = synth.prompt_ids(cfg["vocab"], cfg["prompt"], seed=0)
    m = engine.HypnoModel(c1_image)
    assert m.config.lm_head_tied == 0 and m.config.embed_dtype == hf.DT_FP32
    om = orc.OracleModel(c1_image)
    compare(run_greedy_gpu(m, prompt, 32), run_greedy_oracle(om, prompt, 32), "c1")


def test_c1_batched_sequences_equal_single(cuda_device, c1_image):
    """Several sequences decoded in one batched step give the same logits as
    each decoded alone (and as the oracle), with different prompt lengths."""
    cfg = synth.CONFIGS["c1"]
    m = engine.HypnoModel(c1_image)
    om = orc.OracleModel(c1_image)
    prompts = [synth.prompt_ids(cfg["vocab"], T, seed=s) for s, T in ((1, 5), (2, 1), (3, 33), (4, 0))]
    kv = engine.KVCache(m, n_seqs=4, max_pos=64)
    okvs = []
    for s, p in enumerate(prompts):
        engine.batch_forward(m, p, kv, seq=s)
        okv = om.new_kv(64)
        orc.batch_forward(om, p, okv)
        okvs.append(okv)
    toks = [7, 8, 9, 10]
    for step in range(3):
        lg, am = engine.decode_step(m, kv, [0, 1, 2, 3], toks)
        for s in range(4):
            ref = orc.model_forward(om, toks[s], okvs[s])
            assert rel_err(lg[s], ref) <= TOL, (step, s)
        toks = [int(a) for a in am]
    assert [kv.seq_len(s) for s in range(4)] == [len(p) + 3 for p in prompts]


@pytest.mark.parametrize("max_pos,kv_dtype", [(162, engine.KV_FP32), (161, engine.KV_FP16), (37, engine.KV_FP32)])
def test_c1_ragged_cache_capacity(cuda_device, c1_image, max_pos, kv_dtype):
    """configs[0]'s 9 query heads over 3 KV heads take the per-head attention
    kernel; a cache capacity that is not a multiple of 4 (the bench's parity
    replay allocates prompt + steps + 1 positions) must not disturb its
    shared-memory layout.  Logits and greedy ids against the oracle."""
    cfg = synth.CONFIGS["c1"]
    T = min(cfg["prompt"], max_pos - 5)
    prompt = synth.prompt_ids(cfg["vocab"], T, seed=1)
    m = engine.HypnoModel(c1_image)
    om = orc.OracleModel(c1_image)
    kv = engine.KVCache(m, n_seqs=1, max_pos=max_pos, kv_dtype=kv_dtype)
    okv = om.new_kv(max_pos)
    g = engine.batch_forward(m, prompt, kv)
    r = orc.batch_forward(om, prompt, okv)
    assert rel_err(g, r) <= TOL
    tok = orc.greedy(r)
    for _ in range(4):
        lg, am = engine.decode_step(m, kv, [0], [tok])
        ref = orc.model_forward(om, tok, okv)
        assert rel_err(lg[0], ref) <= TOL
        assert int(am[0]) == orc.greedy(ref)
        tok = int(am[0])


def test_c1_fp16_kv(cuda_device, c1_image):
    """fp16 KV cache (new in this backend; the reference cache is FP32):
    logits stay within tolerance of the FP32-KV oracle."""
    cfg = synth.CONFIGS["c1"]
    prompt = synth.prompt_ids(cfg["vocab"], cfg["prompt"], seed=0)
    m = engine.HypnoModel(c1_image)
    om = orc.OracleModel(c1_image)
    compare(run_greedy_gpu(m, prompt, 16, kv_dtype=engine.KV_FP16), run_greedy_oracle(om, prompt, 16), "c1 fp16-kv")


@pytest.mark.slow
def test_c3_greedy_32_steps(cuda_device):
    """512-token prefill + greedy decode vs the oracle."""
    cfg = synth.CONFIGS["c3"]
    img = _models.synth_image("c3")
    prompt = synth.prompt_ids(cfg["vocab"], cfg["prompt"], seed=0)
    m = engine.HypnoModel(img)
    assert m.config.lm_head_tied == 1 and m.config.embed_dtype == hf.DT_Q4_0
    om = orc.OracleModel(img)
    compare(run_greedy_gpu(m, prompt, 32), run_greedy_oracle(om, prompt, 32), "c3")


C4_GEOMETRY = dict(hidden=1024, layers=2, heads=8, kv_heads=2, inter=2816, vocab=8192, theta=500000.0,
                   max_pos=1024, embed="q4", lm_head="tied")


@pytest.mark.parametrize("kv_dtype", [engine.KV_FP32, engine.KV_FP16])
def test_c4_geometry_batched_decode(cuda_device, kv_dtype):
    """head_dim 128, 4 query heads per KV head, theta 5e5 (configs[3]'s
    attention geometry) on a 2-layer model: ragged prompts (600, 300, 17, 1
    and 0 tokens) prefilled, then batched greedy decode vs the oracle; fp16 KV
    within the same tolerance."""
    from hypno_b200 import synth as sy
    img = sy.build_image(C4_GEOMETRY, seed=3, quantize=orc.quantize_f32_to_q4_0)
    m = engine.HypnoModel(img)
    om = orc.OracleModel(img)
    lens = [600, 300, 17, 1, 0]
    kv = engine.KVCache(m, n_seqs=len(lens), max_pos=1024, kv_dtype=kv_dtype)
    okvs, toks = [], []
    for s, T in enumerate(lens):
        p = sy.prompt_ids(C4_GEOMETRY["vocab"], T, seed=10 + s)
        g = engine.batch_forward(m, p, kv, seq=s)
        okv = om.new_kv(1024)
        r = orc.batch_forward(om, p, okv)
        assert rel_err(g, r) <= TOL, (s, rel_err(g, r))
        okvs.append(okv)
        toks.append(orc.greedy(r) if T else 5)
    seqs = list(range(len(lens)))
    for step in range(6):
        lg, am = engine.decode_step(m, kv, seqs, toks)
        nxt = []
        for s in seqs:
            ref = orc.model_forward(om, toks[s], okvs[s])
            assert rel_err(lg[s], ref) <= TOL, (step, s, rel_err(lg[s], ref))
            assert int(am[s]) == orc.greedy(ref), (step, s, margin(ref))
            nxt.append(int(am[s]))
        toks = nxt


# More 128-row weight tiles than SMs in the fused gate/up projection (160)
# and in the LM head (160): at decode batches of up to 32 rows both run the
# stream-K GEMM (a CTA per SM, runs of (tile, K stage) units, partial tiles
# added by the tile's owner), the gate/up one with the SiLU epilogue.
WIDE_MLP = dict(hidden=256, layers=1, heads=4, kv_heads=2, inter=10240, vocab=20480, theta=10000.0,
                max_pos=256, embed="q4", lm_head="separate")


@pytest.mark.parametrize("n_seqs", [3, 32])
def test_stream_k_decode(cuda_device, n_seqs):
    from hypno_b200 import synth as sy
    img = sy.build_image(WIDE_MLP, seed=5, quantize=orc.quantize_f32_to_q4_0)
    m = engine.HypnoModel(img)
    om = orc.OracleModel(img)
    rng = np.random.default_rng(7 + n_seqs)
    lens = [int(v) for v in rng.integers(1, 25, n_seqs)]
    kv = engine.KVCache(m, n_seqs=n_seqs, max_pos=256, kv_dtype=engine.KV_FP16)
    okvs, toks = [], []
    for s, T in enumerate(lens):
        p = sy.prompt_ids(WIDE_MLP["vocab"], T, seed=200 + s)
        engine.batch_forward(m, p, kv, seq=s)
        okv = om.new_kv(256)
        r = orc.batch_forward(om, p, okv)
        okvs.append(okv)
        toks.append(orc.greedy(r))
    seqs = list(range(n_seqs))
    for step in range(3):
        lg, am = engine.decode_step(m, kv, seqs, toks)
        nxt = []
        for s in seqs:
            ref = orc.model_forward(om, toks[s], okvs[s])
            assert rel_err(lg[s], ref) <= TOL, (step, s, rel_err(lg[s], ref))
            assert int(am[s]) == orc.greedy(ref), (step, s, margin(ref))
            nxt.append(int(am[s]))
        toks = nxt
    kv.close()
    m.close()


@pytest.mark.parametrize("n_seqs", [16, 40, 60, 120])
def test_decode_attention_paths(cuda_device, n_seqs):
    """Batched decode over 16, 40, 60 and 120 sequences of a 2-KV-head model:
    32 and 80 (sequence, KV head) pairs run the cluster-split attention
    (clusters of 8 and 4 CTAs, contexts split at 128- and 256-position
    boundaries), 120 pairs one 16-warp tensor-core CTA each, 240 pairs the
    single fused pass (its tensor-core form for the fp16 cache).  Ragged contexts (0..299 cached positions, so
    some cluster CTAs own no positions) against the oracle for 2 steps."""
    from hypno_b200 import synth as sy
    img = sy.build_image(C4_GEOMETRY, seed=3, quantize=orc.quantize_f32_to_q4_0)
    m = engine.HypnoModel(img)
    om = orc.OracleModel(img)
    rng = np.random.default_rng(n_seqs)
    lens = [int(v) for v in rng.integers(0, 300, n_seqs)]
    kv = engine.KVCache(m, n_seqs=n_seqs, max_pos=1024, kv_dtype=engine.KV_FP16)
    okvs, toks = [], []
    for s, T in enumerate(lens):
        p = sy.prompt_ids(C4_GEOMETRY["vocab"], T, seed=100 + s)
        engine.batch_forward(m, p, kv, seq=s)
        okv = om.new_kv(1024)
        r = orc.batch_forward(om, p, okv)
        okvs.append(okv)
        toks.append(orc.greedy(r) if T else 5)
    seqs = list(range(n_seqs))
    for step in range(2):
        lg, am = engine.decode_step(m, kv, seqs, toks)
        nxt = []
        for s in seqs:
            ref = orc.model_forward(om, toks[s], okvs[s])
            assert rel_err(lg[s], ref) <= TOL, (step, s, lens[s], rel_err(lg[s], ref))
            nxt.append(orc.greedy(ref))
        toks = nxt
