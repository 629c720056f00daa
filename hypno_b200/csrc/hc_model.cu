// Host runtime of the hypno sm_100a backend: .hypno image parsing, one-time
// weight upload (Q4_0 repacked into nibble/scale planes, projections that share
// an input concatenated), the device KV cache, and the two forward passes:
// hc_prefill (turbo::batch_forward) and hc_decode_step (model_forward,
// batched over sequences).
#include "hc_internal.h"
#include "hc_attention.h"
#include "hc_gemm.h"
#include "hc_comm.h"
#include "hc_common.cuh"

#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

// ============================================================ .hypno parsing
// format.rs:1-131 and loader.rs:39-133: 16-byte header ("HYPN", version 1,
// metadata count, tensor count), length-prefixed metadata strings, then the
// tensor table (name, ndim, u64 shape, dtype u32, offset u64, len u64).
namespace {

struct TensorEntry {
    uint32_t dtype = 0;
    std::vector<uint64_t> shape;
    uint64_t offset = 0, len = 0;
};

struct HypnoImage {
    const uint8_t* data = nullptr;
    size_t size = 0;
    std::unordered_map<std::string, std::string> meta;
    std::unordered_map<std::string, TensorEntry> tensors;

    const TensorEntry* find(const std::string& name) const {
        auto it = tensors.find(name);
        return it == tensors.end() ? nullptr : &it->second;
    }
    const uint8_t* payload(const TensorEntry& t) const { return data + t.offset; }
};

int parse_image(const uint8_t* data, size_t size, HypnoImage& img) {
    img.data = data;
    img.size = size;
    HC_CHECK(data != nullptr && size >= 16, HC_ERR_FORMAT, "hypno: buffer too short: needed 16 bytes, got %zu", size);
    HC_CHECK(std::memcmp(data, "HYPN", 4) == 0, HC_ERR_FORMAT, "hypno: invalid magic bytes");
    uint32_t ver, nkv, nt;
    std::memcpy(&ver, data + 4, 4);
    std::memcpy(&nkv, data + 8, 4);
    std::memcpy(&nt, data + 12, 4);
    HC_CHECK(ver == 1, HC_ERR_FORMAT, "hypno: unsupported format version %u (expected 1)", ver);
    size_t cur = 16;
    auto rd32 = [&](uint32_t& v) -> bool {
        if (cur + 4 > size) return false;
        std::memcpy(&v, data + cur, 4);
        cur += 4;
        return true;
    };
    auto rd64 = [&](uint64_t& v) -> bool {
        if (cur + 8 > size) return false;
        std::memcpy(&v, data + cur, 8);
        cur += 8;
        return true;
    };
    auto rdstr = [&](uint32_t len, std::string& s) -> bool {
        if (cur + len > size) return false;
        s.assign(reinterpret_cast<const char*>(data + cur), len);
        cur += len;
        return true;
    };
    for (uint32_t i = 0; i < nkv; i++) {
        uint32_t kl, vl;
        std::string k, v;
        HC_CHECK(rd32(kl) && rdstr(kl, k) && rd32(vl) && rdstr(vl, v), HC_ERR_FORMAT,
                 "hypno: buffer too short in metadata entry %u", i);
        img.meta[k] = v;
    }
    for (uint32_t i = 0; i < nt; i++) {
        uint32_t nl, ndim, dt;
        std::string name;
        TensorEntry t;
        HC_CHECK(rd32(nl) && rdstr(nl, name) && rd32(ndim), HC_ERR_FORMAT, "hypno: buffer too short in tensor %u", i);
        HC_CHECK(ndim <= 16, HC_ERR_FORMAT, "hypno: tensor '%s' has ndim %u", name.c_str(), ndim);
        t.shape.resize(ndim);
        for (uint32_t d = 0; d < ndim; d++)
            HC_CHECK(rd64(t.shape[d]), HC_ERR_FORMAT, "hypno: buffer too short in tensor '%s'", name.c_str());
        HC_CHECK(rd32(dt) && rd64(t.offset) && rd64(t.len), HC_ERR_FORMAT, "hypno: buffer too short in tensor '%s'",
                 name.c_str());
        HC_CHECK(dt <= 3, HC_ERR_FORMAT, "hypno: unknown dtype code: %u", dt);
        HC_CHECK(t.offset <= size && t.offset + t.len <= size, HC_ERR_FORMAT,
                 "hypno: invalid tensor offset %llu: out of file bounds (%zu)", (unsigned long long)t.offset, size);
        t.dtype = dt;
        // Duplicate names: the reference's linear find returns the first.
        if (!img.tensors.count(name)) img.tensors.emplace(name, std::move(t));
    }
    return HC_OK;
}

bool meta_u64(const HypnoImage& img, const char* key, uint64_t& out) {
    auto it = img.meta.find(key);
    if (it == img.meta.end()) return false;
    const char* s = it->second.c_str();
    char* end = nullptr;
    unsigned long long v = std::strtoull(s, &end, 10);
    if (end == s || *end != 0) return false;  // str::parse::<usize> rejects junk
    out = v;
    return true;
}

bool meta_f32(const HypnoImage& img, const char* key, float& out) {
    auto it = img.meta.find(key);
    if (it == img.meta.end()) return false;
    const char* s = it->second.c_str();
    char* end = nullptr;
    float v = std::strtof(s, &end);
    if (end == s || *end != 0) return false;
    out = v;
    return true;
}

}  // namespace

// ============================================================ host f16 / RoPE table

uint16_t hc_f32_to_f16_host(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u, exp = (x >> 23) & 0xFFu, man = x & 0x7FFFFFu;
    if (exp == 0xFF) return (uint16_t)(sign | 0x7C00u | (man ? 0x200u | (man >> 13) : 0));
    int e = (int)exp - 112;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        if (exp == 0) return (uint16_t)sign;
        uint32_t full = man | 0x800000u;
        int sh = 14 - e;
        if (sh > 24) return (uint16_t)sign;
        uint32_t m = full >> sh, rem = full & ((1u << sh) - 1u), half = 1u << (sh - 1);
        if (rem > half || (rem == half && (m & 1u))) m++;
        return (uint16_t)(sign | m);
    }
    uint32_t m = man >> 13, rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (m & 1u))) m++;
    return (uint16_t)((sign | ((uint32_t)e << 10)) + m);
}

float hc_f16_to_f32_host(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16, exp = ((uint32_t)h >> 10) & 0x1Fu, man = (uint32_t)h & 0x3FFu;
    uint32_t out;
    if (exp == 0) {
        if (man == 0) out = sign;
        else {
            int e = -1;
            do { e++; man <<= 1; } while (!(man & 0x400u));
            out = sign | ((uint32_t)(112 - e) << 23) | ((man & 0x3FFu) << 13);
        }
    } else if (exp == 0x1F) out = sign | 0x7F800000u | (man << 13);
    else out = sign | ((exp + 112) << 23) | (man << 13);
    float f;
    std::memcpy(&f, &out, 4);
    return f;
}

std::vector<float2> hc_rope_table(size_t max_pos, size_t hd, float theta) {
    size_t half = hd / 2;
    std::vector<float2> t(max_pos * half);
    std::vector<float> freq(half);
    for (size_t j = 0; j < half; j++) freq[j] = 1.0f / powf(theta, (float)(2 * j) / (float)hd);
    for (size_t p = 0; p < max_pos; p++)
        for (size_t j = 0; j < half; j++) {
            float a = (float)p * freq[j];
            t[p * half + j] = make_float2(cosf(a), sinf(a));
        }
    return t;
}

// ============================================================ model structures

struct LayerW {
    DevWeight qkv;   // rows: q (nq), k (nk), v (nk)
    DevWeight o;     // [hidden x nq]
    DevWeight gu;    // rows: gate (im), up (im); gu_blocked: alternating blocks of GU_BLOCK gate / up rows
    bool gu_blocked = false;
    DevWeight down;  // [hidden x im]
    float* in_norm = nullptr;
    float* post_norm = nullptr;
};

constexpr size_t kPartRows = 256;  // largest row count (decode batch) using split-K slabs
constexpr int kPartSplits = 8;      // most slabs one projection writes
// fused gate/up weights of at most this many rows (74 tiles of 128, half the
// SMs of a B200) split K into slabs in decode instead of applying the SiLU
// gate in the GEMM epilogue
constexpr size_t kGuSlabRows = 74 * 128;

struct Scratch {
    uint64_t generation = 0;  // bumped whenever a buffer moves
    size_t cap_tokens = 0, cap_logit_rows = 0;
    float *hidden = nullptr, *xn = nullptr, *qkv = nullptr, *attn = nullptr, *gu = nullptr, *act = nullptr;
    // fp16 copies in the tensor-core GEMM's K order, written by the producers
    __half *xn16 = nullptr, *attn16 = nullptr, *act16 = nullptr;
    float* logits = nullptr;
    uint32_t* ids = nullptr;
    int* seqs = nullptr;
    int* rowpos = nullptr;
    uint32_t* argmax = nullptr;
    float* tp_tmp = nullptr;      // [tokens][hidden] partial sums to all-reduce
    float* split_part = nullptr;  // [kPartSplits][min(tokens, kPartRows)][max(hidden, qkv)] split-K slabs
    float* tp_gather = nullptr;   // [tp][rows][vocab_shard] gathered logits
    float2* tp_pairs = nullptr;   // [1 + tp][rows] (max logit, index bits): this rank's, then the gathered ones
    // grouped decode attention workspace
    size_t attn_cap = 0;
    float* attn_ws = nullptr;
};

// Per-phase device timing of one decode step (instrumentation): an event is
// recorded on the model's stream at the start of every phase; the time to the
// next event is charged to that phase.
enum Phase : int {
    PH_EMBED, PH_NORM, PH_QKV, PH_ROPE, PH_ATTN, PH_O, PH_REDUCE, PH_GATEUP, PH_DOWN, PH_LMHEAD, PH_LOGITS_X,
    PH_ARGMAX, PH_COUNT
};
const char* const kPhaseNames[PH_COUNT] = {"embed",      "rmsnorm",   "qkv_gemm",       "rope_kv_store",
                                           "attention",  "o_gemm",    "reduce_residual_norm", "gate_up_gemm",
                                           "down_gemm",  "lm_head_gemm", "logits_exchange",  "argmax"};

struct PhaseProf {
    std::vector<cudaEvent_t> ev;
    std::vector<int> ph;
    size_t n = 0;
    int mark(int p, cudaStream_t s) {
        if (n == ev.size()) {
            cudaEvent_t e;
            HC_CUDA(cudaEventCreate(&e));
            ev.push_back(e);
            ph.push_back(0);
        }
        ph[n] = p;
        HC_CUDA(cudaEventRecord(ev[n], s));
        n++;
        return HC_OK;
    }
    ~PhaseProf() {
        for (cudaEvent_t e : ev) cudaEventDestroy(e);
    }
};

struct hc_model {
    int refs = 1;            // the caller's handle + one per live hc_kv
    PhaseProf* prof = nullptr;  // set only inside hc_decode_step_phases
    hc_config cfg{};
    int device = 0;
    cudaStream_t stream = nullptr;
    std::vector<LayerW> layers;
    DevWeight embed, lm_head;
    float* final_norm = nullptr;
    float2* rope = nullptr;
    size_t rope_rows = 0;
    size_t nq = 0, nk = 0;  // q rows, k (= v) rows per shard
    Scratch sc;
    std::vector<void*> allocs;
    hc::GemmWorkspace* gemm_ws = nullptr;
    // tensor parallelism: this rank's vocabulary slice of the LM head, the
    // communicator, and the host watchdog limit for one step
    size_t vocab0 = 0, vocab_shard = 0;
    hc::Comm* comm = nullptr;
    hc::PeerAr* par = nullptr;  // one-shot peer all-reduce (decode sizes), when peers are mapped
    double comm_timeout_s = 60.0;
};

// A captured decode step: replayed while the key (batch, device pointers,
// buffer generations) is unchanged.
struct DecodeGraph {
    int B = 0;
    const void *seqs = nullptr, *ids = nullptr;
    void *logits = nullptr, *argmax = nullptr;
    uint64_t gen = 0;
    size_t kernels = 0;  // kernel nodes in the graph (counted per replay)
    cudaGraphExec_t exec = nullptr;
};

struct hc_kv {
    std::vector<DecodeGraph> graphs;
    bool host_stale = false;
    hc_model* model = nullptr;
    int n_seqs = 0, max_pos = 0, kv_fp16 = 0;
    void* k = nullptr;
    void* v = nullptr;
    int* pos_dev = nullptr;
    std::vector<int> pos_host;
    size_t seq_stride = 0, head_stride = 0, layer_stride = 0;
};

static int sync_pos(hc_kv* kv);

namespace {

int dev_alloc(hc_model* m, void** p, size_t bytes) {
    if (bytes == 0) bytes = 16;
    cudaError_t e = cudaMalloc(p, bytes);
    if (e != cudaSuccess) {
        hc_set_error("cudaMalloc(%zu) failed: %s", bytes, cudaGetErrorString(e));
        cudaGetLastError();
        return HC_ERR_OOM;
    }
    m->allocs.push_back(*p);
    return HC_OK;
}

// Host -> device upload of the image's weights (loader.rs:39-148 mmaps the
// file; here the bytes go to HBM once): a ring of pinned host chunks, each
// filled by OpenMP threads from the image (gathering a tensor-parallel
// shard's rows or columns), copied asynchronously to a device chunk on a copy
// stream, and repacked (Q4_0 blocks -> nibble and scale planes) on the
// model's stream, so the gather of one chunk, the copy of the next and the
// repack of the one before overlap.
struct UploadPipe {
    static constexpr int NSLOT = 4;
    static constexpr size_t CHUNK = size_t(32) << 20;  // bytes per slot
    uint8_t* host[NSLOT] = {};
    uint8_t* dev[NSLOT] = {};
    cudaEvent_t copied[NSLOT] = {};  // the slot's host -> device copy landed
    cudaEvent_t done[NSLOT] = {};    // the slot's buffers are free again
    bool used[NSLOT] = {};
    cudaStream_t cs = nullptr;
    int next = 0, threads = 1;
    size_t bytes = 0;  // moved so far

    int init() {
        for (int i = 0; i < NSLOT; i++) {
            HC_CUDA(cudaHostAlloc((void**)&host[i], CHUNK, cudaHostAllocDefault));
            HC_CUDA(cudaMalloc((void**)&dev[i], CHUNK));
            HC_CUDA(cudaEventCreateWithFlags(&copied[i], cudaEventDisableTiming));
            HC_CUDA(cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming));
        }
        HC_CUDA(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
        threads = std::max(1, std::min(16, omp_get_num_procs()));  // torchrun's OMP_NUM_THREADS=1 does not apply
        return HC_OK;
    }
    void release() {
        if (cs) cudaStreamSynchronize(cs);
        for (int i = 0; i < NSLOT; i++) {
            if (done[i] && used[i]) cudaEventSynchronize(done[i]);
            if (host[i]) cudaFreeHost(host[i]);
            if (dev[i]) cudaFree(dev[i]);
            if (copied[i]) cudaEventDestroy(copied[i]);
            if (done[i]) cudaEventDestroy(done[i]);
            host[i] = dev[i] = nullptr;
            copied[i] = done[i] = nullptr;
        }
        if (cs) cudaStreamDestroy(cs);
        cs = nullptr;
    }
    // The next slot, once its previous chunk has been copied and repacked.
    int acquire(int* s) {
        const int k = next;
        next = (next + 1) % NSLOT;
        if (used[k]) HC_CUDA(cudaEventSynchronize(done[k]));
        used[k] = true;
        *s = k;
        return HC_OK;
    }
    // host[s] <- `rows` runs of `run` bytes, run i starting at src + i * pitch
    void gather(int s, const uint8_t* src, size_t rows, size_t run, size_t pitch) {
        uint8_t* dst = host[s];
        if (run == pitch) {  // one contiguous range: split it over the threads
            const size_t n = rows * run, sl = size_t(1) << 20;
            const long long pieces = (long long)((n + sl - 1) / sl);
#pragma omp parallel for schedule(static) num_threads(threads)
            for (long long i = 0; i < pieces; i++) {
                const size_t o = (size_t)i * sl;
                std::memcpy(dst + o, src + o, std::min(sl, n - o));
            }
        } else {
#pragma omp parallel for schedule(static) num_threads(threads)
            for (long long i = 0; i < (long long)rows; i++)
                std::memcpy(dst + (size_t)i * run, src + (size_t)i * pitch, run);
        }
        bytes += rows * run;
    }
    // host[s] -> dev[s] on the copy stream; the model's stream waits for it
    int copy_in(int s, size_t n, cudaStream_t model_stream) {
        HC_CUDA(cudaMemcpyAsync(dev[s], host[s], n, cudaMemcpyHostToDevice, cs));
        HC_CUDA(cudaEventRecord(copied[s], cs));
        HC_CUDA(cudaStreamWaitEvent(model_stream, copied[s], 0));
        return HC_OK;
    }
};

// One dense 1-D f32 vector (norm weights): FP32 / FP16 converted, anything
// else (or absent) -> ones (load_1d_f32, transformer.rs:250-264).
int upload_norm(hc_model* m, const HypnoImage& img, const std::string& name, size_t len, float** out) {
    std::vector<float> h(len, 1.0f);
    const TensorEntry* t = img.find(name);
    if (t && t->dtype == HC_DTYPE_FP32 && t->len >= len * 4) {
        std::memcpy(h.data(), img.payload(*t), len * 4);
    } else if (t && t->dtype == HC_DTYPE_FP16 && t->len >= len * 2) {
        const uint8_t* p = img.payload(*t);
        for (size_t i = 0; i < len; i++) h[i] = hc_f16_to_f32_host((uint16_t)(p[2 * i] | (p[2 * i + 1] << 8)));
    }
    HC_TRY(dev_alloc(m, (void**)out, len * 4));
    HC_CUDA(cudaMemcpyAsync(*out, h.data(), len * 4, cudaMemcpyHostToDevice, m->stream));
    HC_CUDA(cudaStreamSynchronize(m->stream));
    return HC_OK;
}

struct Part {
    const TensorEntry* t;
    size_t row0, rows;  // rows of this tensor to take (TP shard)
    size_t col0, cols;  // columns to take (TP shard of the K dim)
};

// Uploads the row concatenation of `parts` (each an [rows x k_full] slice) as
// one device weight of shape [sum rows x cols] through the upload pipeline.
// All parts share dtype.
int upload_weight(hc_model* m, const HypnoImage& img, const std::vector<Part>& parts, size_t k_full, DevWeight& w,
                  UploadPipe& pipe) {
    uint32_t dt = parts[0].t->dtype;
    size_t n = 0, cols = parts[0].cols;
    for (auto& p : parts) {
        HC_CHECK(p.t->dtype == dt, HC_ERR_UNSUPPORTED, "fused weight parts must share a dtype");
        HC_CHECK(p.cols == cols, HC_ERR_INVALID, "fused weight parts must share a width");
        n += p.rows;
    }
    w.dtype = dt;
    w.n = n;
    w.k = cols;
    w.present = true;
    if (dt == HC_DTYPE_Q4_0) {
        bool full_cols = (parts[0].col0 == 0 && cols == k_full);
        HC_CHECK(k_full % 32 == 0 || (parts.size() == 1 && full_cols && parts[0].row0 == 0), HC_ERR_UNSUPPORTED,
                 "Q4_0 weights with width %% 32 != 0 cannot be fused or sharded");
        HC_CHECK(cols % 32 == 0 || full_cols, HC_ERR_UNSUPPORTED, "Q4_0 shard width must be a multiple of 32");
        size_t total_blocks;
        if (k_full % 32 == 0) total_blocks = n * (cols / 32);
        else total_blocks = parts[0].t->len / 18;
        w.q4.n = n;
        w.q4.k = cols;
        w.q4.nblocks = total_blocks;
        HC_TRY(dev_alloc(m, (void**)&w.q4.qs, total_blocks * 16));
        HC_TRY(dev_alloc(m, (void**)&w.q4.sc, total_blocks * 2));
        size_t blk_off = 0;
        for (auto& p : parts) {
            const uint8_t* src = img.payload(*p.t);
            const size_t kb_full = k_full / 32;
            // a run = the blocks of one row of the shard (or, for the flattened
            // layout of widths % 32 != 0, one whole stretch of blocks)
            size_t runs, run_blocks, pitch_blocks;
            const uint8_t* base;
            if (k_full % 32 != 0) {
                runs = 1;
                run_blocks = p.t->len / 18;
                pitch_blocks = run_blocks;
                base = src;
            } else {
                HC_CHECK(p.t->len >= (p.row0 + p.rows) * kb_full * 18, HC_ERR_FORMAT,
                         "Q4_0 tensor payload shorter than its shape");
                runs = p.rows;
                run_blocks = cols / 32;
                pitch_blocks = kb_full;
                base = src + (p.row0 * kb_full + p.col0 / 32) * 18;
            }
            if (runs == 1) {  // one long run: chunks of whole blocks
                const size_t per = UploadPipe::CHUNK / 18;
                for (size_t b0 = 0; b0 < run_blocks; b0 += per) {
                    const size_t nb = std::min(per, run_blocks - b0);
                    int sl;
                    HC_TRY(pipe.acquire(&sl));
                    pipe.gather(sl, base + b0 * 18, 1, nb * 18, nb * 18);
                    HC_TRY(pipe.copy_in(sl, nb * 18, m->stream));
                    HC_TRY(hc::launch_q4_split(pipe.dev[sl], nb, w.q4.qs + blk_off, w.q4.sc + blk_off, m->stream));
                    HC_CUDA(cudaEventRecord(pipe.done[sl], m->stream));
                    blk_off += nb;
                }
                continue;
            }
            const size_t per = std::max<size_t>(1, UploadPipe::CHUNK / (run_blocks * 18));  // rows per chunk
            HC_CHECK(run_blocks * 18 <= UploadPipe::CHUNK, HC_ERR_UNSUPPORTED, "a row of %zu blocks exceeds an upload chunk",
                     run_blocks);
            for (size_t r0 = 0; r0 < runs; r0 += per) {
                const size_t nr = std::min(per, runs - r0);
                int sl;
                HC_TRY(pipe.acquire(&sl));
                pipe.gather(sl, base + r0 * pitch_blocks * 18, nr, run_blocks * 18, pitch_blocks * 18);
                HC_TRY(pipe.copy_in(sl, nr * run_blocks * 18, m->stream));
                HC_TRY(hc::launch_q4_split(pipe.dev[sl], nr * run_blocks, w.q4.qs + blk_off, w.q4.sc + blk_off,
                                           m->stream));
                HC_CUDA(cudaEventRecord(pipe.done[sl], m->stream));
                blk_off += nr * run_blocks;
            }
        }
        return HC_OK;
    }
    size_t es = (dt == HC_DTYPE_FP32) ? 4 : (dt == HC_DTYPE_FP16 ? 2 : 0);
    HC_CHECK(es != 0, HC_ERR_UNSUPPORTED, "weight dtype %u (Q8_0) is not supported by the GPU backend", dt);
    HC_TRY(dev_alloc(m, &w.dense, n * cols * es));
    const size_t row_bytes = cols * es;
    HC_CHECK(row_bytes <= UploadPipe::CHUNK, HC_ERR_UNSUPPORTED, "a row of %zu bytes exceeds an upload chunk", row_bytes);
    const size_t per = UploadPipe::CHUNK / row_bytes;
    size_t row_off = 0;
    for (auto& p : parts) {
        HC_CHECK(p.t->len >= (p.row0 + p.rows) * k_full * es, HC_ERR_FORMAT, "tensor payload shorter than its shape");
        const uint8_t* src = img.payload(*p.t) + (p.row0 * k_full + p.col0) * es;
        for (size_t r0 = 0; r0 < p.rows; r0 += per) {
            const size_t nr = std::min(per, p.rows - r0);
            int sl;
            HC_TRY(pipe.acquire(&sl));
            pipe.gather(sl, src + r0 * k_full * es, nr, row_bytes, k_full * es);
            HC_CUDA(cudaMemcpyAsync((uint8_t*)w.dense + (row_off + r0) * row_bytes, pipe.host[sl], nr * row_bytes,
                                    cudaMemcpyHostToDevice, pipe.cs));
            HC_CUDA(cudaEventRecord(pipe.done[sl], pipe.cs));
        }
        row_off += p.rows;
    }
    return HC_OK;
}

void free_model(hc_model* m) {
    if (!m) return;
    cudaSetDevice(m->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    for (void* p : m->allocs) cudaFree(p);
    void* scr[] = {m->sc.hidden, m->sc.xn, m->sc.qkv, m->sc.attn, m->sc.gu, m->sc.act, m->sc.logits, m->sc.ids,
                   m->sc.seqs, m->sc.rowpos, m->sc.argmax, m->rope, m->sc.attn_ws, m->sc.xn16, m->sc.attn16,
                   m->sc.act16};
    for (void* p : scr)
        if (p) cudaFree(p);
    if (m->gemm_ws) hc::gemm_workspace_free(m->gemm_ws);
    if (m->sc.tp_tmp) cudaFree(m->sc.tp_tmp);
    if (m->sc.split_part) cudaFree(m->sc.split_part);
    if (m->sc.tp_gather) cudaFree(m->sc.tp_gather);
    if (m->sc.tp_pairs) cudaFree(m->sc.tp_pairs);
    if (m->par) hc::peer_ar_free(m->par, m->cfg.tp_rank, m->cfg.tp_size);
    if (m->comm) hc::comm_free(m->comm);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

int ensure_scratch(hc_model* m, size_t tokens, size_t logit_rows) {
    Scratch& s = m->sc;
    const hc_config& c = m->cfg;
    if (tokens > s.cap_tokens) {
        size_t t = std::max<size_t>(tokens, 8);
        float** bufs[] = {&s.hidden, &s.xn, &s.qkv, &s.attn, &s.gu, &s.act};
        size_t widths[] = {c.hidden_size, c.hidden_size, m->nq + 2 * m->nk, m->nq, 2 * (m->layers.empty() ? 0 : m->layers[0].gu.n / 2),
                           m->layers.empty() ? 0 : m->layers[0].gu.n / 2};
        for (int i = 0; i < 6; i++) {
            if (*bufs[i]) cudaFree(*bufs[i]);
            *bufs[i] = nullptr;
            HC_CUDA(cudaMalloc((void**)bufs[i], std::max<size_t>(t * widths[i], 4) * sizeof(float)));
        }
        if (s.ids) cudaFree(s.ids);
        if (s.seqs) cudaFree(s.seqs);
        if (s.rowpos) cudaFree(s.rowpos);
        {
            __half** h16[] = {&s.xn16, &s.attn16, &s.act16};
            size_t w16[] = {c.hidden_size, m->nq, m->layers.empty() ? 0 : m->layers[0].gu.n / 2};
            for (int i = 0; i < 3; i++) {
                if (*h16[i]) cudaFree(*h16[i]);
                *h16[i] = nullptr;
                // the GEMM's split rows: hi then lo halves of every row (store_x16)
                HC_CUDA(cudaMalloc((void**)h16[i], std::max<size_t>(2 * t * w16[i], 8) * sizeof(__half)));
            }
        }
        if (s.tp_tmp) cudaFree(s.tp_tmp);
        s.tp_tmp = nullptr;
        if (m->cfg.tp_size > 1) HC_CUDA(cudaMalloc((void**)&s.tp_tmp, t * c.hidden_size * sizeof(float)));
        if (s.split_part) cudaFree(s.split_part);
        s.split_part = nullptr;
        // widest slab user: o/down (hidden), qkv, or a narrow gate/up (see run_layers)
        const size_t gu_w = m->layers.empty() ? 0 : m->layers[0].gu.n;
        HC_CUDA(cudaMalloc((void**)&s.split_part,
                           (size_t)kPartSplits * std::min(t, kPartRows) *
                               std::max<size_t>(std::max<size_t>(c.hidden_size, m->nq + 2 * m->nk),
                                                gu_w <= kGuSlabRows ? gu_w : 0) *
                               sizeof(float)));
        HC_CUDA(cudaMalloc((void**)&s.ids, t * sizeof(uint32_t)));
        HC_CUDA(cudaMalloc((void**)&s.seqs, t * sizeof(int)));
        HC_CUDA(cudaMalloc((void**)&s.rowpos, t * sizeof(int)));
        s.cap_tokens = t;
        s.generation++;
    }
    if (logit_rows > s.cap_logit_rows) {
        size_t r = std::max<size_t>(logit_rows, 1);
        if (s.logits) cudaFree(s.logits);
        if (s.argmax) cudaFree(s.argmax);
        HC_CUDA(cudaMalloc((void**)&s.logits, r * c.vocab_size * sizeof(float)));
        if (s.tp_gather) cudaFree(s.tp_gather);
        s.tp_gather = nullptr;
        if (s.tp_pairs) cudaFree(s.tp_pairs);
        s.tp_pairs = nullptr;
        if (m->cfg.tp_size > 1) {
            HC_CUDA(cudaMalloc((void**)&s.tp_gather, r * m->vocab_shard * m->cfg.tp_size * sizeof(float)));
            HC_CUDA(cudaMalloc((void**)&s.tp_pairs, r * (1 + m->cfg.tp_size) * sizeof(float2)));
        }
        HC_CUDA(cudaMalloc((void**)&s.argmax, r * sizeof(uint32_t)));
        s.cap_logit_rows = r;
        s.generation++;
    }
    return HC_OK;
}

int ensure_rope(hc_model* m, size_t rows) {
    if (rows <= m->rope_rows) return HC_OK;
    std::vector<float2> t = hc_rope_table(rows, m->cfg.head_dim, m->cfg.rope_theta);
    if (m->rope) cudaFree(m->rope);
    m->rope = nullptr;
    HC_CUDA(cudaMalloc((void**)&m->rope, t.size() * sizeof(float2)));
    HC_CUDA(cudaMemcpy(m->rope, t.data(), t.size() * sizeof(float2), cudaMemcpyHostToDevice));
    m->rope_rows = rows;
    m->sc.generation++;
    return HC_OK;
}

int ensure_attn_ws(hc_model* m, size_t rows, size_t nh, size_t max_pos, size_t nsplit, size_t hd) {
    Scratch& s = m->sc;
    size_t need = rows * nh * (max_pos + 2 * nsplit + nsplit * hd);
    if (need > s.attn_cap) {
        if (s.attn_ws) cudaFree(s.attn_ws);
        s.attn_ws = nullptr;
        s.attn_cap = 0;
        HC_CUDA(cudaMalloc((void**)&s.attn_ws, need * sizeof(float)));
        s.attn_cap = need;
        s.generation++;
    }
    return HC_OK;
}

inline int phase(hc_model* m, int p) { return m->prof ? m->prof->mark(p, m->stream) : HC_OK; }

// y = W . x for `tokens` rows (the Q4_0 path picks the CUDA-core matvec for
// few tokens and the tcgen05 GEMM otherwise).
int matmul(hc_model* m, const DevWeight& w, const float* x, size_t ldx, size_t tokens, float* y, size_t ldy, int epi,
           const float* res, size_t ldres, const __half* x16 = nullptr) {
    if (w.dtype == HC_DTYPE_Q4_0 && hc::gemm_tc_eligible(w.q4, tokens))
        return hc::gemm_tc(m->gemm_ws, w.q4, x, ldx, tokens, y, ldy, epi, res, ldres, m->stream, x16);
    return hc::launch_matmul(w, x, ldx, tokens, y, ldy, epi, res, ldres, m->stream);
}

__global__ void k_add_rows(float* __restrict__ y, const float* __restrict__ a, size_t n) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = a[i] + y[i];
}

// hidden (+)= W x for a projection whose K dimension is split across the
// tensor-parallel ranks (o_proj, down_proj): each rank's partial product is
// summed by an all-reduce, then added to the residual stream (the reference's
// `hidden[i] = residual[i] + proj[i]`, transformer.rs:561-563, 595-598).
// Decode-sized outputs use the one-shot peer all-reduce, which also applies
// the next RMSNorm (weight next_norm, when given) and then sets *normed; other
// sizes (prefill) use NCCL and leave the norm to the caller.
int row_parallel(hc_model* m, const DevWeight& w, const float* x, size_t ldx, size_t rows, const __half* x16,
                 int gemm_phase, const float* next_norm = nullptr, bool* normed = nullptr) {
    const size_t H = m->cfg.hidden_size;
    Scratch& s = m->sc;
    if (normed) *normed = false;
    HC_TRY(phase(m, gemm_phase));
    if (m->cfg.tp_size <= 1) {
        // decode sizes: K split over CTAs whose partial slabs are added by the
        // residual + next-RMSNorm kernel (no cluster reduction in the GEMM)
        if (s.split_part && rows <= kPartRows && w.dtype == HC_DTYPE_Q4_0 && hc::gemm_tc_eligible(w.q4, rows) &&
            hc::residual_splits_norm_ok(H, H, H)) {
            int splits = 1;
            HC_TRY(hc::gemm_tc_partials(m->gemm_ws, w.q4, x, ldx, rows, s.split_part, kPartSplits, &splits, m->stream,
                                        x16));
            HC_TRY(phase(m, PH_REDUCE));
            HC_TRY(hc::launch_residual_splits_norm(s.split_part, splits, rows, H, s.hidden, H, next_norm,
                                                   m->cfg.rms_norm_eps, s.xn, H, s.xn16, m->stream));
            if (normed) *normed = next_norm != nullptr;
            return HC_OK;
        }
        return matmul(m, w, x, ldx, rows, s.hidden, H, hc::EPI_ADD, s.hidden, H, x16);
    }
    HC_CHECK(m->comm, HC_ERR_STATE, "tensor-parallel model used before hc_comm_init");
    if (m->par && hc::peer_ar_fits(m->par, rows, H)) {
        // o_proj and down_proj alternate, each with its own partial buffer
        const int slot = gemm_phase == PH_DOWN ? 1 : 0;
        const float* slabs = nullptr;
        int splits = 0;
        if (s.split_part && rows <= kPartRows && w.dtype == HC_DTYPE_Q4_0 && hc::gemm_tc_eligible(w.q4, rows)) {
            // split-K slabs in local memory (as on one GPU); the all-reduce
            // kernel adds them into the peer-visible partial
            HC_TRY(hc::gemm_tc_partials(m->gemm_ws, w.q4, x, ldx, rows, s.split_part, kPartSplits, &splits, m->stream,
                                        x16));
            slabs = s.split_part;
        } else {
            HC_TRY(matmul(m, w, x, ldx, rows, hc::peer_ar_partial(m->par, slot), H, hc::EPI_STORE, nullptr, 0, x16));
        }
        HC_TRY(phase(m, PH_REDUCE));
        HC_TRY(hc::peer_ar_residual_norm(m->par, slot, m->cfg.tp_rank, m->cfg.tp_size, rows, slabs, splits, s.hidden,
                                         H, next_norm, m->cfg.rms_norm_eps, s.xn, H, s.xn16,
                                         hc::gemm_error_flag(m->gemm_ws), m->stream));
        if (normed) *normed = next_norm != nullptr;
        return HC_OK;
    }
    HC_TRY(matmul(m, w, x, ldx, rows, s.tp_tmp, H, hc::EPI_STORE, nullptr, 0, x16));
    HC_TRY(phase(m, PH_REDUCE));
    HC_TRY(hc::comm_allreduce_sum(m->comm, s.tp_tmp, rows * H, m->stream));
    size_t n = rows * H;
    k_add_rows<<<(unsigned)((n + 255) / 256), 256, 0, m->stream>>>(s.hidden, s.tp_tmp, n);
    HC_LAUNCH_CHECK();
    return HC_OK;
}

__global__ void k_unshard_logits(const float* __restrict__ g, float* __restrict__ out, int rows, int vs, int tp) {
    size_t n = (size_t)rows * vs * tp;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        size_t r = i / ((size_t)vs * tp), rem = i % ((size_t)vs * tp);
        size_t rank = rem / vs, v = rem % vs;
        out[i] = g[(rank * rows + r) * vs + v];
    }
}

// logits[rows][vocab] = W_lm x; with tensor parallelism each rank computes
// its vocabulary slice and the slices are all-gathered.
int lm_head_logits(hc_model* m, const float* x, size_t rows, float* logits, const __half* x16 = nullptr) {
    const hc_config& c = m->cfg;
    if (!m->lm_head.present) {
        HC_CUDA(cudaMemsetAsync(logits, 0, rows * c.vocab_size * sizeof(float), m->stream));
        return HC_OK;
    }
    HC_TRY(phase(m, PH_LMHEAD));
    if (c.tp_size <= 1)
        return matmul(m, m->lm_head, x, c.hidden_size, rows, logits, c.vocab_size, hc::EPI_STORE, nullptr, 0, x16);
    HC_CHECK(m->comm, HC_ERR_STATE, "tensor-parallel model used before hc_comm_init");
    const size_t vs = m->vocab_shard;
    float* mine = m->sc.tp_gather + (size_t)c.tp_rank * rows * vs;
    HC_TRY(matmul(m, m->lm_head, x, c.hidden_size, rows, mine, vs, hc::EPI_STORE, nullptr, 0, x16));
    HC_TRY(phase(m, PH_LOGITS_X));
    HC_TRY(hc::comm_allgather(m->comm, mine, m->sc.tp_gather, rows * vs, m->stream));
    size_t n = rows * c.vocab_size;
    unsigned grid = (unsigned)std::min<size_t>((n + 255) / 256, 4096);
    k_unshard_logits<<<grid, 256, 0, m->stream>>>(m->sc.tp_gather, logits, (int)rows, (int)vs, c.tp_size);
    HC_LAUNCH_CHECK();
    return HC_OK;
}

// Greedy ids of a vocabulary-sharded LM head without gathering the logits:
// each rank takes the pick of its slice (k_argmax), the ranks exchange
// (value, index, NaN bit) pairs, and every rank folds them in rank order
// (k_pick_pairs), which gives the pick over the whole vocabulary
// (run.rs:234-238).
int lm_head_argmax_tp(hc_model* m, const float* x, size_t rows, uint32_t* argmax, const __half* x16) {
    const hc_config& c = m->cfg;
    HC_CHECK(m->comm, HC_ERR_STATE, "tensor-parallel model used before hc_comm_init");
    HC_TRY(phase(m, PH_LMHEAD));
    const size_t vs = m->vocab_shard;
    float* mine = m->sc.tp_gather + (size_t)c.tp_rank * rows * vs;
    HC_TRY(matmul(m, m->lm_head, x, c.hidden_size, rows, mine, vs, hc::EPI_STORE, nullptr, 0, x16));
    HC_TRY(phase(m, PH_ARGMAX));
    float2* local = m->sc.tp_pairs;
    float2* all = local + rows;
    HC_TRY(hc::launch_argmax_pairs(mine, rows, vs, vs, (uint32_t)m->vocab0, local, m->stream));
    HC_TRY(phase(m, PH_LOGITS_X));
    HC_TRY(hc::comm_allgather(m->comm, reinterpret_cast<const float*>(local), reinterpret_cast<float*>(all), rows * 2,
                              m->stream));
    return hc::launch_pick_pairs(all, rows, c.tp_size, argmax, m->stream);
}

// Waits for the model's stream; with a communicator the wait is watched
// (a peer that stopped participating aborts the communicator).
int model_wait(hc_model* m) {
    if (m->comm) return hc::comm_wait(m->comm, m->stream, m->comm_timeout_s);
    HC_CUDA(cudaStreamSynchronize(m->stream));
    return HC_OK;
}

// The per-layer body shared by prefill (prefill = true, rows = prompt
// tokens of one sequence) and decode (rows = sequences).
// tail_norm: the norm that follows the last layer (the final norm in decode);
// *tail_normed reports whether the last projection's all-reduce already
// applied it to s.xn.
int run_layers(hc_model* m, hc_kv* kv, size_t rows, bool prefill, int seq, int pos0,
               const float* tail_norm = nullptr, bool* tail_normed = nullptr) {
    const hc_config& c = m->cfg;
    Scratch& s = m->sc;
    const size_t hd = c.head_dim, H = c.hidden_size;
    const size_t nq = m->nq, nk = m->nk, ldqkv = nq + 2 * nk;
    const size_t nh_l = nq / hd, nkv_l = nk / hd;
    const float scale = 1.0f / sqrtf((float)hd);
    bool xn_ready = false;  // s.xn already holds this layer's input norm
    if (tail_normed) *tail_normed = false;
    for (size_t li = 0; li < m->layers.size(); li++) {
        LayerW& L = m->layers[li];
        // one token: the qkv matvec applies the input norm itself and writes
        // a single slab, which the RoPE kernel rotates and stores into the
        // cache (three kernels fewer per layer with the gate/up one below)
        const bool one = rows == 1 && s.split_part && !hc::gemm_tc_eligible(L.qkv.q4, rows);
        const bool qkv_fused = one && !xn_ready && hc::gemv1_fusable(L.qkv, s.hidden, L.in_norm, false);
        if (!xn_ready && !qkv_fused) {
            HC_TRY(phase(m, PH_NORM));
            HC_TRY(hc::launch_rmsnorm(s.hidden, H, L.in_norm, s.xn, H, rows, H, c.rms_norm_eps, m->stream, s.xn16));
        }
        xn_ready = false;
        HC_TRY(phase(m, PH_QKV));
        size_t lofs = li * kv->layer_stride * (kv->kv_fp16 ? 2 : 4);
        void* kc = (uint8_t*)kv->k + lofs;
        void* vc = (uint8_t*)kv->v + lofs;
        const bool qkv_tc = s.split_part && rows <= kPartRows && L.qkv.dtype == HC_DTYPE_Q4_0 &&
                            hc::gemm_tc_eligible(L.qkv.q4, rows);
        if (qkv_tc || qkv_fused) {
            // decode sizes: K split over CTAs into slabs (or the one-token
            // matvec's single slab) that the RoPE kernel adds, also storing k
            // and v into the cache
            int splits = 1;
            if (qkv_tc)
                HC_TRY(hc::gemm_tc_partials(m->gemm_ws, L.qkv.q4, s.xn, H, rows, s.split_part, kPartSplits, &splits,
                                            m->stream, s.xn16));
            else
                HC_TRY(hc::launch_gemv1_fused(L.qkv, s.hidden, s.split_part, L.in_norm, c.rms_norm_eps, false,
                                              m->stream));
            hc::KvStoreArgs ka;
            ka.kc = kc;
            ka.vc = vc;
            ka.kv_fp16 = kv->kv_fp16;
            ka.seq_stride = kv->seq_stride;
            ka.head_stride = kv->head_stride;
            ka.max_pos = kv->max_pos;
            ka.seqs = prefill ? nullptr : s.seqs;
            ka.pos = kv->pos_dev;
            ka.fixed_seq = seq;
            ka.pos0 = pos0;
            ka.nq = (int)nq;
            ka.nk = (int)nk;
            HC_TRY(phase(m, PH_ROPE));
            HC_TRY(hc::launch_rope_rows_slabs(s.split_part, splits, s.qkv, ldqkv, rows, ldqkv, nh_l + nkv_l, hd,
                                              m->rope, m->rope_rows, prefill ? nullptr : s.rowpos, pos0, m->stream,
                                              &ka));
        } else {
            HC_TRY(matmul(m, L.qkv, s.xn, H, rows, s.qkv, ldqkv, hc::EPI_STORE, nullptr, 0, s.xn16));
            HC_TRY(phase(m, PH_ROPE));
            HC_TRY(hc::launch_rope_rows(s.qkv, ldqkv, rows, nh_l + nkv_l, hd, m->rope, m->rope_rows,
                                        prefill ? nullptr : s.rowpos, pos0, m->stream));
            HC_TRY(hc::launch_kv_store(s.qkv + nq, s.qkv + nq + nk, ldqkv, (int)rows, (int)nkv_l, (int)hd, kc, vc,
                                       kv->kv_fp16, kv->seq_stride, kv->head_stride, kv->max_pos,
                                       prefill ? nullptr : s.seqs, kv->pos_dev, seq, pos0, m->stream));
        }
        HC_TRY(phase(m, PH_ATTN));
        hc::AttnParams P{};
        P.out16 = s.attn16;
        P.q = s.qkv;
        P.ldq = ldqkv;
        P.out = s.attn;
        P.ldo = nq;
        P.vself = s.qkv + nq + nk;
        P.ldself = ldqkv;
        P.nh = (int)nh_l;
        P.nkv = (int)nkv_l;
        P.hd = (int)hd;
        P.scale = scale;
        if (prefill) {
            P.mode_prefill = 1;
            P.smem_n = (int)rows;
            P.kp = s.qkv + nq;
            P.vp = s.qkv + nq + nk;
            P.ldkv = ldqkv;
            // the gate/up buffer is free until the MLP: it holds the fp16 K/V
            // planes of the tensor-core prefill attention (2 * nk floats a row)
            if (L.gu.n >= 2 * nk) P.kv16 = reinterpret_cast<__half*>(s.gu);
            if (hc::pattn_supported((int)hd))
                HC_TRY(hc::launch_prefill_attention(P, (int)rows, m->stream));
            else
                HC_TRY(hc::launch_attention(P, (int)rows, 0, m->stream));
        } else if (hc::dattn_supported((int)nh_l, (int)nkv_l, (int)hd)) {
            hc::DecAttnParams D{};
            D.out16 = s.attn16;
            D.q = s.qkv;
            D.ldq = ldqkv;
            D.out = s.attn;
            D.ldo = nq;
            D.vself = s.qkv + nq + nk;
            D.ldself = ldqkv;
            D.nh = (int)nh_l;
            D.nkv = (int)nkv_l;
            D.hd = (int)hd;
            D.scale = scale;
            D.kc = kc;
            D.vc = vc;
            D.seq_stride = kv->seq_stride;
            D.head_stride = kv->head_stride;
            D.seqs = s.seqs;
            D.pos = kv->pos_dev;
            D.max_pos = kv->max_pos;
            // One CTA per (sequence, KV head) streams the whole context when
            // that already fills most of the 2 x 148 CTA slots and its scores
            // fit in shared memory; with fewer pairs (tensor-parallel shards)
            // a cluster of 2-8 CTAs shares each pair; with fewer still (a
            // single sequence) the context is split over CTAs that exchange
            // through global scratch, so that about one wave of CTAs runs.
            const int G = (int)(nh_l / nkv_l);
            const size_t ctas = rows * nkv_l, slots = 2 * 148;
            const int red_floats = (hc::DA_REDUCE_WARPS + 1) * G * (int)hd;
            const int smem_floats = 110 * 1024 / 4;
            const bool whole = ctas * 4 >= slots * 3 || kv->max_pos <= 256;
            int ncl = 1;  // CTAs of a cluster sharing one (sequence, KV head) when the pairs are too few
            while (!whole && ncl < 8 && ctas * ncl * 4 < slots * 3) ncl *= 2;
            const int cl_chunk = (kv->max_pos + ncl - 1) / ncl;
            // about one pair per SM: one 16-warp tensor-core CTA each
            const bool wide = !whole && ctas * 3 >= 148 * 2 && ctas <= 148 &&
                              hc::dattn_wide_ok((int)nh_l, (int)nkv_l, (int)hd, kv->max_pos, kv->kv_fp16);
            if (wide) {
                D.chunk = kv->max_pos;
                D.nsplit = 1;
                D.wide = 1;
            } else if (whole && G * kv->max_pos + 4 + red_floats <= smem_floats) {
                D.chunk = kv->max_pos;
                D.nsplit = 1;
            } else if (!whole && ctas * ncl * 4 >= slots * 3 && G * cl_chunk + 4 + red_floats <= smem_floats) {
                D.cluster = ncl;
                D.chunk = cl_chunk;
                D.nsplit = 1;
            } else {
                int max_chunk = std::max(64, (smem_floats - 4 - red_floats) / G);
                int want_splits = (int)std::max<size_t>(1, (slots + ctas - 1) / ctas);
                int chunk = std::max(256, (kv->max_pos + want_splits - 1) / want_splits);
                chunk = std::min(chunk, max_chunk);
                chunk = std::min(chunk, kv->max_pos);
                D.chunk = chunk;
                D.nsplit = (kv->max_pos + chunk - 1) / chunk;
                if (D.nsplit == 1) D.chunk = kv->max_pos;
            }
            HC_TRY(ensure_attn_ws(m, rows, nh_l, (size_t)kv->max_pos, (size_t)D.nsplit, hd));
            D.S = s.attn_ws;
            D.smax = D.S + rows * nh_l * (size_t)kv->max_pos;
            D.spart = D.smax + rows * nh_l * (size_t)D.nsplit;
            D.opart = D.spart + rows * nh_l * (size_t)D.nsplit;
            HC_TRY(hc::launch_decode_attention(D, (int)rows, kv->kv_fp16, m->stream));
        } else {
            P.mode_prefill = 0;
            P.smem_n = kv->max_pos;
            P.kc = kc;
            P.vc = vc;
            P.seq_stride = kv->seq_stride;
            P.head_stride = kv->head_stride;
            P.seqs = s.seqs;
            P.pos = kv->pos_dev;
            HC_TRY(hc::launch_attention(P, (int)rows, kv->kv_fp16, m->stream));
        }
        bool normed = false;
        HC_TRY(row_parallel(m, L.o, s.attn, nq, rows, s.attn16, PH_O, L.post_norm, &normed));
        // one token: the gate/up matvec applies the norm and the SiLU gate
        const bool gu_fused = one && !normed && L.gu_blocked && hc::gemv1_fusable(L.gu, s.hidden, L.post_norm, true);
        if (!normed && !gu_fused) {
            HC_TRY(phase(m, PH_NORM));
            HC_TRY(hc::launch_rmsnorm(s.hidden, H, L.post_norm, s.xn, H, rows, H, c.rms_norm_eps, m->stream, s.xn16));
        }
        size_t im = L.gu.n / 2;
        HC_TRY(phase(m, PH_GATEUP));
        if (gu_fused) {
            HC_TRY(hc::launch_gemv1_fused(L.gu, s.hidden, s.act, L.post_norm, c.rms_norm_eps, true, m->stream));
        } else if (s.split_part && rows <= kPartRows && L.gu_blocked && L.gu.n <= kGuSlabRows &&
            hc::gemm_tc_eligible(L.gu.q4, rows)) {
            // a narrow gate/up (a tensor-parallel rank's shard) has too few
            // 128-row tiles to fill the GPU, and the SiLU epilogue needs whole
            // sums: split K into slabs and apply the gate in the consumer
            int splits = 1;
            HC_TRY(hc::gemm_tc_partials(m->gemm_ws, L.gu.q4, s.xn, H, rows, s.split_part, kPartSplits, &splits,
                                        m->stream, s.xn16));
            HC_TRY(hc::launch_silu_mul(s.split_part, L.gu.n, s.act, im, rows, im, m->stream, s.act16, true, splits));
        } else if (L.gu_blocked && hc::gemm_tc_eligible(L.gu.q4, rows)) {
            HC_TRY(hc::gemm_tc_silu(m->gemm_ws, L.gu.q4, s.xn, H, rows, s.act, im, s.act16, m->stream, s.xn16));
        } else {
            HC_TRY(matmul(m, L.gu, s.xn, H, rows, s.gu, 2 * im, hc::EPI_STORE, nullptr, 0, s.xn16));
            HC_TRY(hc::launch_silu_mul(s.gu, 2 * im, s.act, im, rows, im, m->stream, s.act16, L.gu_blocked));
        }
        const bool last = li + 1 == m->layers.size();
        const float* next = last ? tail_norm : m->layers[li + 1].in_norm;
        HC_TRY(row_parallel(m, L.down, s.act, im, rows, s.act16, PH_DOWN, next, &normed));
        if (last) {
            if (tail_normed) *tail_normed = normed;
        } else {
            xn_ready = normed;
        }
    }
    return HC_OK;
}

__global__ void k_gather_pos(const int* __restrict__ seqs, const int* __restrict__ pos, int* __restrict__ rowpos,
                             int B) {
    hc::pdl_trigger();
    hc::pdl_wait();
    int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < B) rowpos[b] = pos[seqs[b]];
}

int decode_dev_impl(hc_model* m, hc_kv* kv, const int* seqs_dev, const uint32_t* ids_dev, int B, float* logits_dev,
                    uint32_t* argmax_dev) {
    const hc_config& c = m->cfg;
    Scratch& s = m->sc;
    HC_TRY(ensure_scratch(m, (size_t)B, (size_t)B));
    if (seqs_dev != s.seqs) HC_CUDA(cudaMemcpyAsync(s.seqs, seqs_dev, B * sizeof(int), cudaMemcpyDeviceToDevice, m->stream));
    if (ids_dev != s.ids) HC_CUDA(cudaMemcpyAsync(s.ids, ids_dev, B * sizeof(uint32_t), cudaMemcpyDeviceToDevice, m->stream));
    HC_TRY(phase(m, PH_EMBED));
    HC_TRY(hc::launch_pdl(k_gather_pos, dim3((B + 127) / 128), dim3(128), 0, m->stream, (const int*)s.seqs,
                          (const int*)kv->pos_dev, s.rowpos, B));
    HC_TRY(hc::launch_embed(m->embed, s.ids, (size_t)B, s.hidden, c.hidden_size, m->stream));
    bool final_normed = false;
    HC_TRY(run_layers(m, kv, (size_t)B, false, 0, 0, m->final_norm, &final_normed));
    HC_TRY(phase(m, PH_NORM));
    HC_TRY(hc::launch_advance(s.seqs, kv->pos_dev, B, m->stream));
    // one token on one GPU: the LM head's matvec applies the final norm
    const bool head_fused = !final_normed && B == 1 && c.tp_size <= 1 && m->lm_head.present &&
                            !hc::gemm_tc_eligible(m->lm_head.q4, 1) &&
                            hc::gemv1_fusable(m->lm_head, s.hidden, m->final_norm, false);
    if (!final_normed && !head_fused)
        HC_TRY(hc::launch_rmsnorm(s.hidden, c.hidden_size, m->final_norm, s.xn, c.hidden_size, (size_t)B,
                                  c.hidden_size, c.rms_norm_eps, m->stream, s.xn16));
    if (head_fused) {
        float* logits = logits_dev ? logits_dev : s.logits;
        HC_TRY(phase(m, PH_LMHEAD));
        HC_TRY(hc::launch_gemv1_fused(m->lm_head, s.hidden, logits, m->final_norm, c.rms_norm_eps, false, m->stream));
        HC_TRY(phase(m, PH_ARGMAX));
        if (argmax_dev) HC_TRY(hc::launch_argmax(logits, (size_t)B, c.vocab_size, argmax_dev, m->stream));
    } else if (c.tp_size > 1 && !logits_dev && argmax_dev && m->lm_head.present) {
        // greedy ids only: exchange (max, index) pairs instead of the logits
        HC_TRY(lm_head_argmax_tp(m, s.xn, (size_t)B, argmax_dev, s.xn16));
    } else {
        float* logits = logits_dev ? logits_dev : s.logits;
        HC_TRY(lm_head_logits(m, s.xn, (size_t)B, logits, s.xn16));
        HC_TRY(phase(m, PH_ARGMAX));
        if (argmax_dev) HC_TRY(hc::launch_argmax(logits, (size_t)B, c.vocab_size, argmax_dev, m->stream));
    }
    HC_TRY(phase(m, PH_COUNT));
    return HC_OK;
}

}  // namespace

// ============================================================ C ABI: model

HC_EXPORT int hc_model_load(const uint8_t* image, size_t len, int tp_rank, int tp_size, hc_model** out) {
    cudaGetLastError();  // a stale error of an earlier unrelated call is not ours
    HC_CHECK(out != nullptr, HC_ERR_INVALID, "hc_model_load: out is NULL");
    *out = nullptr;
    HC_CHECK(tp_size >= 1 && tp_rank >= 0 && tp_rank < tp_size, HC_ERR_INVALID, "hc_model_load: bad tp rank/size %d/%d",
             tp_rank, tp_size);
    HypnoImage img;
    HC_TRY(parse_image(image, len, img));
    hc_config c{};
    // HypnoConfig::from_model, transformer.rs:42-63
    HC_CHECK(meta_u64(img, "hidden_size", c.hidden_size), HC_ERR_FORMAT, "hypno: metadata hidden_size missing");
    HC_CHECK(meta_u64(img, "num_attention_heads", c.num_attention_heads), HC_ERR_FORMAT,
             "hypno: metadata num_attention_heads missing");
    if (!meta_u64(img, "num_key_value_heads", c.num_key_value_heads)) c.num_key_value_heads = c.num_attention_heads;
    HC_CHECK(c.num_attention_heads > 0 && c.num_key_value_heads > 0, HC_ERR_FORMAT, "hypno: zero heads");
    c.head_dim = c.hidden_size / c.num_attention_heads;
    if (!meta_u64(img, "intermediate_size", c.intermediate_size)) c.intermediate_size = c.hidden_size * 8 / 3;
    if (!meta_u64(img, "num_hidden_layers", c.num_hidden_layers)) c.num_hidden_layers = 0;
    if (!meta_u64(img, "vocab_size", c.vocab_size)) c.vocab_size = 32000;
    if (!meta_u64(img, "max_position_embeddings", c.max_position_embeddings)) c.max_position_embeddings = 2048;
    if (!meta_f32(img, "rms_norm_eps", c.rms_norm_eps)) c.rms_norm_eps = 1e-5f;
    if (!meta_f32(img, "rope_theta", c.rope_theta)) c.rope_theta = 10000.0f;
    c.tp_rank = tp_rank;
    c.tp_size = tp_size;
    const size_t H = c.hidden_size, hd = c.head_dim, nh = c.num_attention_heads, nkv = c.num_key_value_heads;
    const size_t im = c.intermediate_size;
    HC_CHECK(hd % 2 == 0 && hd > 0, HC_ERR_UNSUPPORTED, "head_dim %zu must be even", hd);
    HC_CHECK(nh % nkv == 0, HC_ERR_UNSUPPORTED, "num_attention_heads must be a multiple of num_key_value_heads");
    HC_CHECK(nkv % (size_t)tp_size == 0 && nh % (size_t)tp_size == 0, HC_ERR_UNSUPPORTED,
             "tensor parallel size %d must divide the query and KV heads", tp_size);
    HC_CHECK(im % tp_size == 0 && (tp_size == 1 || (im / tp_size) % 32 == 0), HC_ERR_UNSUPPORTED,
             "tensor parallel size %d must split intermediate_size into multiples of 32", tp_size);

    hc_model* m = new hc_model();
    m->cfg = c;
    cudaGetDevice(&m->device);
    if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess) {
        hc_set_error("hc_model_load: no usable CUDA device (%s)", cudaGetErrorString(cudaGetLastError()));
        delete m;
        return HC_ERR_CUDA;
    }
    UploadPipe pipe;
    auto fail = [&](int r) {
        pipe.release();
        free_model(m);
        return r;
    };
    if (int r0 = pipe.init()) return fail(r0);
    const size_t nh_l = nh / tp_size, nkv_l = nkv / tp_size, im_l = im / tp_size;
    m->nq = nh_l * hd;
    m->nk = nkv_l * hd;
    m->layers.resize(c.num_hidden_layers);
    for (size_t li = 0; li < c.num_hidden_layers; li++) {
        std::string p = "model.layers." + std::to_string(li) + ".";
        const TensorEntry *tq = img.find(p + "self_attn.q_proj.weight"), *tk = img.find(p + "self_attn.k_proj.weight"),
                          *tv = img.find(p + "self_attn.v_proj.weight"), *to = img.find(p + "self_attn.o_proj.weight"),
                          *tg = img.find(p + "mlp.gate_proj.weight"), *tu = img.find(p + "mlp.up_proj.weight"),
                          *td = img.find(p + "mlp.down_proj.weight");
        if (!(tq && tk && tv && to && tg && tu && td)) {
            hc_set_error("hypno: layer %zu is missing a projection tensor", li);
            return fail(HC_ERR_UNSUPPORTED);
        }
        LayerW& L = m->layers[li];
        int r;
        if (tq->dtype == tk->dtype && tk->dtype == tv->dtype && (tq->dtype != HC_DTYPE_Q4_0 || H % 32 == 0)) {
            r = upload_weight(m, img,
                              {{tq, tp_rank * nh_l * hd, nh_l * hd, 0, H},
                               {tk, tp_rank * nkv_l * hd, nkv_l * hd, 0, H},
                               {tv, tp_rank * nkv_l * hd, nkv_l * hd, 0, H}},
                              H, L.qkv, pipe);
        } else {
            hc_set_error("hypno: q/k/v projections of layer %zu must share a dtype and (for Q4_0) a width that is a "
                         "multiple of 32", li);
            r = HC_ERR_UNSUPPORTED;
        }
        if (r) return fail(r);
        if ((r = upload_weight(m, img, {{to, 0, H, tp_rank * nh_l * hd, nh_l * hd}}, nh * hd, L.o, pipe)))
            return fail(r);
        if (tg->dtype != tu->dtype) {
            hc_set_error("hypno: gate/up projections of layer %zu must share a dtype", li);
            return fail(HC_ERR_UNSUPPORTED);
        }
        // Q4_0 gate/up rows are interleaved in blocks of GU_BLOCK so that the
        // tensor-core GEMM can apply the SiLU gate in its epilogue
        L.gu_blocked = tg->dtype == HC_DTYPE_Q4_0 && im_l % hc::GU_BLOCK == 0 && H % 32 == 0;
        if (L.gu_blocked) {
            std::vector<Part> parts;
            parts.reserve(2 * im_l / hc::GU_BLOCK);
            for (size_t b = 0; b < im_l; b += hc::GU_BLOCK) {
                parts.push_back({tg, tp_rank * im_l + b, (size_t)hc::GU_BLOCK, 0, H});
                parts.push_back({tu, tp_rank * im_l + b, (size_t)hc::GU_BLOCK, 0, H});
            }
            r = upload_weight(m, img, parts, H, L.gu, pipe);
        } else {
            r = upload_weight(m, img, {{tg, tp_rank * im_l, im_l, 0, H}, {tu, tp_rank * im_l, im_l, 0, H}}, H, L.gu, pipe);
        }
        if (r) return fail(r);
        if ((r = upload_weight(m, img, {{td, 0, H, tp_rank * im_l, im_l}}, im, L.down, pipe)))
            return fail(r);
        if ((r = upload_norm(m, img, p + "input_layernorm.weight", H, &L.in_norm))) return fail(r);
        if ((r = upload_norm(m, img, p + "post_attention_layernorm.weight", H, &L.post_norm))) return fail(r);
    }
    int r;
    if ((r = upload_norm(m, img, "model.norm.weight", H, &m->final_norm))) return fail(r);
    const TensorEntry* te = img.find("model.embed_tokens.weight");
    const TensorEntry* tl = img.find("lm_head.weight");
    if (te) {
        if ((r = upload_weight(m, img, {{te, 0, c.vocab_size, 0, H}}, H, m->embed, pipe)))
            return fail(r);
        m->cfg.embed_dtype = te->dtype;
    }
    // LM head: with tensor parallelism each rank keeps a vocabulary slice.
    const size_t V = c.vocab_size;
    const bool shard_vocab = tp_size > 1 && V % (size_t)tp_size == 0;
    m->vocab_shard = shard_vocab ? V / tp_size : V;
    m->vocab0 = shard_vocab ? (size_t)tp_rank * m->vocab_shard : 0;
    if (tp_size > 1 && !shard_vocab) {
        hc_set_error("tensor parallel size %d must divide the vocabulary (%zu)", tp_size, V);
        return fail(HC_ERR_UNSUPPORTED);
    }
    if (tl) {
        if ((r = upload_weight(m, img, {{tl, m->vocab0, m->vocab_shard, 0, H}}, H, m->lm_head, pipe)))
            return fail(r);
        m->cfg.lm_head_dtype = tl->dtype;
        m->cfg.lm_head_tied = 0;
    } else if (te) {
        // tied: a view of the embedding rows of this rank (transformer.rs:521-524)
        m->lm_head = m->embed;
        m->lm_head.n = m->vocab_shard;
        if (m->embed.dtype == HC_DTYPE_Q4_0) {
            size_t kb = H / 32;
            m->lm_head.q4.n = m->vocab_shard;
            m->lm_head.q4.qs = m->embed.q4.qs + m->vocab0 * kb;
            m->lm_head.q4.sc = m->embed.q4.sc + m->vocab0 * kb;
            m->lm_head.q4.nblocks = m->vocab_shard * kb;
        } else if (m->embed.dense) {
            size_t es = m->embed.dtype == HC_DTYPE_FP32 ? 4 : 2;
            m->lm_head.dense = (uint8_t*)m->embed.dense + m->vocab0 * H * es;
        }
        m->cfg.lm_head_dtype = te->dtype;
        m->cfg.lm_head_tied = 1;
    }
    // every chunk repacked or copied before the pinned ring goes away
    if (cudaStreamSynchronize(m->stream) != cudaSuccess || cudaStreamSynchronize(pipe.cs) != cudaSuccess) {
        hc_set_error("hypno: weight upload failed (%s)", cudaGetErrorString(cudaGetLastError()));
        return fail(HC_ERR_CUDA);
    }
    pipe.release();
    m->gemm_ws = hc::gemm_workspace_new();
    if (!hc::gemm_error_flag(m->gemm_ws)) {  // allocated now: kernels captured later refer to it
        hc_set_error("cannot allocate the pipeline error flag");
        return fail(HC_ERR_OOM);
    }
    if ((r = ensure_rope(m, c.max_position_embeddings))) return fail(r);
    *out = m;
    return HC_OK;
}

HC_EXPORT int hc_model_config(const hc_model* model, hc_config* out) {
    HC_CHECK(model && out, HC_ERR_INVALID, "hc_model_config: NULL argument");
    *out = model->cfg;
    return HC_OK;
}

static void model_release(hc_model* m) {
    if (m && --m->refs == 0) free_model(m);
}

// Releases the caller's handle; the device state stays alive until the last
// KV cache built on it is freed too.
HC_EXPORT int hc_model_free(hc_model* model) {
    cudaGetLastError();
    model_release(model);
    cudaGetLastError();
    return HC_OK;
}

HC_EXPORT int hc_sync(hc_model* model) {
    HC_CHECK(model, HC_ERR_INVALID, "hc_sync: NULL model");
    HC_CUDA(cudaSetDevice(model->device));
    HC_TRY(model_wait(model));
    return hc::gemm_check(model->gemm_ws);
}

HC_EXPORT void* hc_model_stream(hc_model* model) { return model ? (void*)model->stream : nullptr; }

HC_EXPORT int hc_kv_alloc(hc_model* model, int n_seqs, int max_pos, int kv_dtype, hc_kv** out) {
    cudaGetLastError();  // a stale error of an earlier unrelated call is not ours
    HC_CHECK(model && out, HC_ERR_INVALID, "hc_kv_alloc: NULL argument");
    HC_CHECK(n_seqs > 0, HC_ERR_INVALID, "hc_kv_alloc: n_seqs must be > 0");
    HC_CHECK(kv_dtype == HC_KV_FP32 || kv_dtype == HC_KV_FP16, HC_ERR_INVALID, "hc_kv_alloc: bad kv dtype %d", kv_dtype);
    HC_CUDA(cudaSetDevice(model->device));
    if (max_pos <= 0) max_pos = (int)model->cfg.max_position_embeddings;
    hc_kv* kv = new hc_kv();
    kv->model = model;
    kv->n_seqs = n_seqs;
    kv->max_pos = max_pos;
    kv->kv_fp16 = kv_dtype == HC_KV_FP16;
    const size_t hd = model->cfg.head_dim, nkv_l = model->nk / hd, L = model->cfg.num_hidden_layers;
    kv->head_stride = (size_t)max_pos * hd;
    kv->layer_stride = nkv_l * kv->head_stride;
    kv->seq_stride = L * kv->layer_stride;
    size_t bytes = (size_t)n_seqs * kv->seq_stride * (kv->kv_fp16 ? 2 : 4);
    cudaError_t e1 = cudaMalloc(&kv->k, std::max<size_t>(bytes, 16));
    cudaError_t e2 = e1 == cudaSuccess ? cudaMalloc(&kv->v, std::max<size_t>(bytes, 16)) : e1;
    cudaError_t e3 = e2 == cudaSuccess ? cudaMalloc((void**)&kv->pos_dev, n_seqs * sizeof(int)) : e2;
    if (e3 != cudaSuccess) {
        cudaGetLastError();
        if (kv->k) cudaFree(kv->k);
        if (kv->v) cudaFree(kv->v);
        delete kv;
        hc_set_error("hc_kv_alloc: cannot allocate %zu bytes of KV cache", 2 * bytes);
        return HC_ERR_OOM;
    }
    kv->pos_host.assign(n_seqs, 0);
    model->refs++;
    HC_CUDA(cudaMemsetAsync(kv->pos_dev, 0, n_seqs * sizeof(int), model->stream));
    HC_CUDA(cudaMemsetAsync(kv->k, 0, bytes, model->stream));
    HC_CUDA(cudaMemsetAsync(kv->v, 0, bytes, model->stream));
    int r = ensure_rope(model, (size_t)max_pos);
    if (r) {
        hc_kv_free(kv);
        return r;
    }
    HC_CUDA(cudaStreamSynchronize(model->stream));
    *out = kv;
    return HC_OK;
}

HC_EXPORT int hc_kv_free(hc_kv* kv) {
    if (!kv) return HC_OK;
    cudaSetDevice(kv->model->device);
    cudaStreamSynchronize(kv->model->stream);
    for (auto& g : kv->graphs)
        if (g.exec) cudaGraphExecDestroy(g.exec);
    if (kv->k) cudaFree(kv->k);
    if (kv->v) cudaFree(kv->v);
    if (kv->pos_dev) cudaFree(kv->pos_dev);
    hc_model* m = kv->model;
    delete kv;
    model_release(m);
    cudaGetLastError();  // leave no stale error for the caller's next call
    return HC_OK;
}

HC_EXPORT int hc_kv_seq_len(const hc_kv* kv, int seq, int* out) {
    HC_CHECK(kv && out, HC_ERR_INVALID, "hc_kv_seq_len: NULL argument");
    HC_CHECK(seq >= 0 && seq < kv->n_seqs, HC_ERR_INVALID, "hc_kv_seq_len: seq %d out of range", seq);
    HC_CUDA(cudaSetDevice(kv->model->device));
    HC_TRY(sync_pos(const_cast<hc_kv*>(kv)));
    *out = kv->pos_host[seq];
    return HC_OK;
}

HC_EXPORT int hc_kv_set_pos(hc_kv* kv, int seq, int pos) {
    HC_CHECK(kv, HC_ERR_INVALID, "hc_kv_set_pos: NULL kv");
    HC_CHECK(seq >= 0 && seq < kv->n_seqs, HC_ERR_INVALID, "hc_kv_set_pos: seq %d out of range", seq);
    HC_CHECK(pos >= 0 && pos <= kv->max_pos, HC_ERR_INVALID, "hc_kv_set_pos: pos %d out of range", pos);
    HC_CUDA(cudaSetDevice(kv->model->device));
    HC_TRY(sync_pos(kv));
    kv->pos_host[seq] = pos;
    HC_CUDA(cudaMemcpyAsync(kv->pos_dev + seq, &kv->pos_host[seq], sizeof(int), cudaMemcpyHostToDevice,
                            kv->model->stream));
    HC_CUDA(cudaStreamSynchronize(kv->model->stream));
    return HC_OK;
}

HC_EXPORT int hc_prefill(hc_model* m, hc_kv* kv, int seq, const uint32_t* ids, int T, float* logits_out) {
    cudaGetLastError();  // a stale error of an earlier unrelated call is not ours
    HC_CHECK(m && kv && kv->model == m, HC_ERR_INVALID, "hc_prefill: bad model/kv");
    HC_CHECK(seq >= 0 && seq < kv->n_seqs, HC_ERR_INVALID, "hc_prefill: seq %d out of range", seq);
    HC_CHECK(T >= 0 && (T == 0 || ids), HC_ERR_INVALID, "hc_prefill: bad ids");
    HC_CUDA(cudaSetDevice(m->device));
    const hc_config& c = m->cfg;
    HC_TRY(sync_pos(kv));
    const int p0 = kv->pos_host[seq];
    HC_CHECK((size_t)p0 + (size_t)T <= (size_t)kv->max_pos, HC_ERR_STATE, "hc_prefill: %d + %d positions exceed the cache (%d)",
             p0, T, kv->max_pos);
    for (int t = 0; t < T; t++)
        HC_CHECK(ids[t] < c.vocab_size, HC_ERR_INVALID, "hc_prefill: token id %u >= vocab %llu", ids[t],
                 (unsigned long long)c.vocab_size);
    if (T == 0) {  // turbo.rs:255-258
        if (logits_out) std::memset(logits_out, 0, c.vocab_size * sizeof(float));
        return HC_OK;
    }
    Scratch& s = m->sc;
    HC_TRY(ensure_scratch(m, (size_t)T, 1));
    HC_CUDA(cudaMemcpyAsync(s.ids, ids, T * sizeof(uint32_t), cudaMemcpyHostToDevice, m->stream));
    HC_TRY(hc::launch_embed(m->embed, s.ids, (size_t)T, s.hidden, c.hidden_size, m->stream));
    HC_TRY(run_layers(m, kv, (size_t)T, true, seq, p0));
    kv->pos_host[seq] = p0 + T;
    HC_CUDA(cudaMemcpyAsync(kv->pos_dev + seq, &kv->pos_host[seq], sizeof(int), cudaMemcpyHostToDevice, m->stream));
    const float* last = s.hidden + (size_t)(T - 1) * c.hidden_size;
    HC_TRY(hc::launch_rmsnorm(last, c.hidden_size, m->final_norm, s.xn, c.hidden_size, 1, c.hidden_size,
                              c.rms_norm_eps, m->stream));
    HC_TRY(lm_head_logits(m, s.xn, 1, s.logits));
    if (logits_out)
        HC_CUDA(cudaMemcpyAsync(logits_out, s.logits, c.vocab_size * sizeof(float), cudaMemcpyDeviceToHost, m->stream));
    HC_TRY(model_wait(m));
    return hc::gemm_check(m->gemm_ws);
}

static int decode_graphed(hc_model* m, hc_kv* kv, const int* seqs_dev, const uint32_t* ids_dev, int B,
                          float* logits_dev, uint32_t* argmax_dev);

static int sync_pos(hc_kv* kv) {
    if (!kv->host_stale) return HC_OK;
    HC_CUDA(cudaMemcpyAsync(kv->pos_host.data(), kv->pos_dev, kv->n_seqs * sizeof(int), cudaMemcpyDeviceToHost,
                            kv->model->stream));
    HC_CUDA(cudaStreamSynchronize(kv->model->stream));
    kv->host_stale = false;
    return HC_OK;
}

static int check_decode_args(hc_model* m, hc_kv* kv, const int* seqs, int B) {
    HC_TRY(sync_pos(kv));
    for (int b = 0; b < B; b++) {
        HC_CHECK(seqs[b] >= 0 && seqs[b] < kv->n_seqs, HC_ERR_INVALID, "decode: seq %d out of range", seqs[b]);
        HC_CHECK(kv->pos_host[seqs[b]] < kv->max_pos, HC_ERR_STATE, "decode: sequence %d is full (%d positions)",
                 seqs[b], kv->max_pos);
        for (int j = 0; j < b; j++)
            HC_CHECK(seqs[j] != seqs[b], HC_ERR_INVALID, "decode: sequence %d appears twice in one step", seqs[b]);
    }
    return HC_OK;
}

HC_EXPORT int hc_decode_step(hc_model* m, hc_kv* kv, const int* seqs, const uint32_t* ids, int B, float* logits_out,
                             uint32_t* argmax_out) {
    cudaGetLastError();  // a stale error of an earlier unrelated call is not ours
    HC_CHECK(m && kv && kv->model == m, HC_ERR_INVALID, "hc_decode_step: bad model/kv");
    HC_CHECK(B > 0 && seqs && ids, HC_ERR_INVALID, "hc_decode_step: bad batch");
    HC_CUDA(cudaSetDevice(m->device));
    HC_TRY(check_decode_args(m, kv, seqs, B));
    for (int b = 0; b < B; b++)
        HC_CHECK(ids[b] < m->cfg.vocab_size, HC_ERR_INVALID, "decode: token id %u >= vocab", ids[b]);
    Scratch& s = m->sc;
    HC_TRY(ensure_scratch(m, (size_t)B, (size_t)B));
    HC_CUDA(cudaMemcpyAsync(s.seqs, seqs, B * sizeof(int), cudaMemcpyHostToDevice, m->stream));
    HC_CUDA(cudaMemcpyAsync(s.ids, ids, B * sizeof(uint32_t), cudaMemcpyHostToDevice, m->stream));
    HC_TRY(decode_graphed(m, kv, s.seqs, s.ids, B, s.logits, argmax_out ? s.argmax : nullptr));
    for (int b = 0; b < B; b++) kv->pos_host[seqs[b]] += 1;
    const size_t V = m->cfg.vocab_size;
    if (logits_out)
        HC_CUDA(cudaMemcpyAsync(logits_out, s.logits, (size_t)B * V * sizeof(float), cudaMemcpyDeviceToHost, m->stream));
    if (argmax_out)
        HC_CUDA(cudaMemcpyAsync(argmax_out, s.argmax, B * sizeof(uint32_t), cudaMemcpyDeviceToHost, m->stream));
    HC_TRY(model_wait(m));
    return hc::gemm_check(m->gemm_ws);
}

static uint64_t model_generation(hc_model* m) { return m->sc.generation * 1000003ull + hc::gemm_generation(m->gemm_ws); }

// One decode step on the model's stream, replayed from a CUDA graph after the
// first call with the same key.  The first call runs eagerly (sizing every
// workspace), then captures the same launch sequence for later replays.
static int decode_graphed(hc_model* m, hc_kv* kv, const int* seqs_dev, const uint32_t* ids_dev, int B,
                          float* logits_dev, uint32_t* argmax_dev) {
    uint64_t gen = model_generation(m);
    for (auto& g : kv->graphs) {
        if (g.B == B && g.seqs == seqs_dev && g.ids == ids_dev && g.logits == logits_dev && g.argmax == argmax_dev &&
            g.gen == gen && g.exec) {
            HC_CUDA(cudaGraphLaunch(g.exec, m->stream));
            hc_count_launches(g.kernels);
            return HC_OK;
        }
    }
    HC_TRY(decode_dev_impl(m, kv, seqs_dev, ids_dev, B, logits_dev, argmax_dev));
    gen = model_generation(m);  // the eager run may have grown a workspace
    cudaGraph_t graph = nullptr;
    HC_CUDA(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
    int r = decode_dev_impl(m, kv, seqs_dev, ids_dev, B, logits_dev, argmax_dev);
    cudaError_t e = cudaStreamEndCapture(m->stream, &graph);
    if (r != HC_OK || e != cudaSuccess || model_generation(m) != gen) {
        if (graph) cudaGraphDestroy(graph);
        cudaGetLastError();
        return r != HC_OK ? r : HC_OK;  // the eager step already ran; stay uncaptured
    }
    size_t kernels = 0;
    {
        size_t nn = 0;
        if (cudaGraphGetNodes(graph, nullptr, &nn) == cudaSuccess && nn) {
            std::vector<cudaGraphNode_t> nodes(nn);
            if (cudaGraphGetNodes(graph, nodes.data(), &nn) == cudaSuccess)
                for (auto nd : nodes) {
                    cudaGraphNodeType t;
                    if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) kernels++;
                }
        }
    }
    cudaGraphExec_t exec = nullptr;
    e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return HC_OK;
    }
    // Replace a stale entry with the same pointers, or add one.
    for (auto& g : kv->graphs) {
        if (g.B == B && g.seqs == seqs_dev && g.ids == ids_dev && g.logits == logits_dev && g.argmax == argmax_dev) {
            if (g.exec) cudaGraphExecDestroy(g.exec);
            g.exec = exec;
            g.gen = gen;
            g.kernels = kernels;
            return HC_OK;
        }
    }
    DecodeGraph g;
    g.B = B;
    g.seqs = seqs_dev;
    g.ids = ids_dev;
    g.logits = logits_dev;
    g.argmax = argmax_dev;
    g.gen = gen;
    g.kernels = kernels;
    g.exec = exec;
    kv->graphs.push_back(g);
    return HC_OK;
}

HC_EXPORT int hc_decode_step_dev(hc_model* m, hc_kv* kv, const int* seqs_dev, const uint32_t* ids_dev, int B,
                                 float* logits_dev, uint32_t* argmax_dev) {
    HC_CHECK(m && kv && kv->model == m, HC_ERR_INVALID, "hc_decode_step_dev: bad model/kv");
    HC_CHECK(B > 0 && seqs_dev && ids_dev, HC_ERR_INVALID, "hc_decode_step_dev: bad batch");
    HC_CUDA(cudaSetDevice(m->device));
    // No host round trip: positions live on the device.  The kernels skip
    // stores past the cache capacity; hc_kv_seq_len reports the positions.
    HC_TRY(decode_graphed(m, kv, seqs_dev, ids_dev, B, logits_dev, argmax_dev));
    kv->host_stale = true;
    return HC_OK;
}

// One decode step like hc_decode_step_dev, launched eagerly with an event
// between phases; waits for it and adds each phase's device time to
// phase_ms[i] (hc_phase_count() entries, names from hc_phase_name).
HC_EXPORT int hc_decode_step_phases(hc_model* m, hc_kv* kv, const int* seqs_dev, const uint32_t* ids_dev, int B,
                                    uint32_t* argmax_dev, float* phase_ms) {
    HC_CHECK(m && kv && kv->model == m, HC_ERR_INVALID, "hc_decode_step_phases: bad model/kv");
    HC_CHECK(B > 0 && seqs_dev && ids_dev && phase_ms, HC_ERR_INVALID, "hc_decode_step_phases: bad arguments");
    HC_CUDA(cudaSetDevice(m->device));
    PhaseProf prof;
    m->prof = &prof;
    const int r = decode_dev_impl(m, kv, seqs_dev, ids_dev, B, nullptr, argmax_dev);
    m->prof = nullptr;
    HC_TRY(r);
    HC_TRY(model_wait(m));
    kv->host_stale = true;
    for (size_t i = 0; i + 1 < prof.n; i++) {
        float ms = 0.0f;
        HC_CUDA(cudaEventElapsedTime(&ms, prof.ev[i], prof.ev[i + 1]));
        if (prof.ph[i] < PH_COUNT) phase_ms[prof.ph[i]] += ms;
    }
    return HC_OK;
}

HC_EXPORT int hc_phase_count(void) { return PH_COUNT; }

HC_EXPORT const char* hc_phase_name(int i) { return (i >= 0 && i < PH_COUNT) ? kPhaseNames[i] : ""; }

// ============================================================ C ABI: tensor parallel

HC_EXPORT int hc_comm_unique_id(uint8_t* out128) {
    HC_CHECK(out128, HC_ERR_INVALID, "hc_comm_unique_id: NULL out");
    return hc::comm_unique_id(out128);
}

HC_EXPORT int hc_comm_init(hc_model* m, const uint8_t* id128, int rank, int size, double timeout_s) {
    HC_CHECK(m && id128, HC_ERR_INVALID, "hc_comm_init: NULL argument");
    HC_CHECK(size == m->cfg.tp_size && rank == m->cfg.tp_rank, HC_ERR_INVALID,
             "hc_comm_init: rank/size %d/%d differ from the model's shard %d/%d", rank, size, m->cfg.tp_rank,
             m->cfg.tp_size);
    HC_CUDA(cudaSetDevice(m->device));
    if (m->par) {
        hc::peer_ar_free(m->par, rank, size);
        m->par = nullptr;
    }
    if (m->comm) {
        hc::comm_free(m->comm);
        m->comm = nullptr;
    }
    if (timeout_s > 0) m->comm_timeout_s = timeout_s;
    HC_TRY(hc::comm_init(&m->comm, id128, rank, size, m->comm_timeout_s));
    // decode-sized all-reduces over mapped peer memory (up to 256 rows); NCCL
    // stays for larger ones and whenever peer mappings are unavailable
    const char* env = getenv("HC_PEER_ALLREDUCE");
    if (!(env && env[0] == '0'))
        HC_TRY(hc::peer_ar_init(m->comm, rank, size, 256, m->cfg.hidden_size, &m->par));
    return HC_OK;
}
