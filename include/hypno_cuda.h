/*
 * hypno_cuda.h — C ABI of the sm_100a backend for hypno's Q4_0 inference path.
 *
 * The library (hypno_b200/libhypno_cuda.so) replaces the CPU SIMD kernels
 * and the forward passes of the hypno engine (HypnotizerAI/hypno, Rust) with
 * one B200 backend.  Every entry point below names the reference interface
 * it replaces (paths relative to crates/hypno/src/ of the reference).
 *
 * Conventions
 *  - Every function returns an int status: HC_OK (0) or a negative HC_ERR_*.
 *    The message of the last failure on the calling thread is returned by
 *    hc_last_error().  No C++ exception crosses this boundary.
 *  - Handles are opaque.  Model-level calls are ordered on the model's own
 *    CUDA stream; calls that take or return HOST buffers synchronize before
 *    returning.  The *_dev variants take device pointers and a stream and do
 *    not synchronize.
 *  - dtype codes are the reference's DType discriminants (dtype.rs:6-15):
 *    0 = FP32, 1 = FP16, 2 = Q8_0, 3 = Q4_0.
 *  - There is no CPU fallback: without a usable CUDA device every compute
 *    entry point fails with HC_ERR_CUDA.
 */
#ifndef HYPNO_CUDA_H
#define HYPNO_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HC_OK 0
#define HC_ERR_INVALID (-1)     /* bad argument, shape or size */
#define HC_ERR_CUDA (-2)        /* CUDA runtime/driver error or no device */
#define HC_ERR_UNSUPPORTED (-3) /* dtype or shape the backend does not implement */
#define HC_ERR_FORMAT (-4)      /* malformed .hypno image */
#define HC_ERR_OOM (-5)         /* device allocation failed */
#define HC_ERR_TIMEOUT (-6)     /* a bounded device wait ran out */
#define HC_ERR_STATE (-7)       /* e.g. KV cache full, position out of range */

#define HC_DTYPE_FP32 0u
#define HC_DTYPE_FP16 1u
#define HC_DTYPE_Q8_0 2u
#define HC_DTYPE_Q4_0 3u

#define HC_KV_FP32 0
#define HC_KV_FP16 1

/* ---- library ---------------------------------------------------------- */

/* Message of the last failure on this thread ("" when none). */
const char* hc_last_error(void);
/* ABI version (major*10000 + minor*100 + patch). */
int hc_version(void);
/* Selects the CUDA device for subsequent calls on this thread. */
int hc_set_device(int device);
/* Number of CUDA kernels this library has launched in this process (all
 * threads).  Instrumentation for benchmarks; no reference counterpart. */
uint64_t hc_kernel_launches(void);

/* ---- op level: host slices in/out (drop-in for ops.rs) ----------------- */

/* ops::matmul_vec_auto, ops.rs:25-38 (and kernels::matmul_q4_0,
 * kernels.rs:256-265): y[n] = W[n x m] . x[m] (+ bias).  w/w_len is the raw
 * weight payload exactly as stored in a .hypno file (Q4_0: 18-byte blocks
 * over the flattened row-major tensor).  bias may be NULL.  dtype 2 (Q8_0)
 * returns HC_ERR_UNSUPPORTED. */
int hc_matmul_vec_auto(float* y, const uint8_t* w, size_t w_len, uint32_t dtype,
                       const float* x, const float* bias, size_t n, size_t m);

/* turbo::batch_matmul, turbo.rs:306-343: Y[batch x n] = X[batch x dim] . W^T. */
int hc_batch_matmul(float* y, const uint8_t* w, size_t w_len, uint32_t dtype,
                    const float* x, size_t n, size_t dim, size_t batch);

/* ops::rms_norm_in_place, ops.rs:59-61 (kernels::rms_norm_fused, kernels.rs:592). */
int hc_rms_norm_in_place(float* x, const float* w, size_t n, float eps);
/* ops::softmax_in_place, ops.rs:71-73 (kernels::softmax_fast, kernels.rs:631;
 * the exp(v/8) Taylor polynomial on the first floor(n/8)*8 entries). */
int hc_softmax_in_place(float* x, size_t n);
/* ops::silu_in_place, ops.rs:81-83. */
int hc_silu_in_place(float* x, size_t n);
/* ops::rope, ops.rs:86-99 (adjacent-pair rotation of one head of q and k). */
int hc_rope(float* q, float* k, size_t head_dim, size_t pos, float theta);

/* quant::quantize_f32_to_q4_0, quant.rs:108-117: floor(n/32) blocks of 18
 * bytes are written to out (bit-exact with the reference). */
int hc_q4_0_quantize(const float* x, size_t n, uint8_t* out);
/* quant::dequantize_q4_0, quant.rs:120-132: floor(nbytes/18) blocks -> out. */
int hc_q4_0_dequantize(const uint8_t* q, size_t nbytes, float* out);

/* ---- op level: device-resident ---------------------------------------- */

/* Same arithmetic as hc_q4_0_quantize / hc_q4_0_dequantize on device buffers
 * (AoS 18-byte blocks), stream-ordered, no synchronization. */
int hc_q4_0_quantize_dev(const float* x, size_t n, uint8_t* out, void* stream);
int hc_q4_0_dequantize_dev(const uint8_t* q, size_t nbytes, float* out, void* stream);

/* A Q4_0 weight matrix W[n x k] resident in HBM in the backend's layout
 * (nibble plane of 16-byte blocks + fp16 scale plane), built from the .hypno
 * payload.  Replaces the mmap'd &[u8] view of loader.rs:139-148 for the
 * device path. */
typedef struct hc_q4_matrix hc_q4_matrix;
int hc_q4_matrix_upload(const uint8_t* w, size_t w_len, size_t n, size_t k, hc_q4_matrix** out);
int hc_q4_matrix_from_dev(const uint8_t* w_dev, size_t w_len, size_t n, size_t k, void* stream,
                          hc_q4_matrix** out);
int hc_q4_matrix_free(hc_q4_matrix* mat);
/* Y[mtok x n] = X[mtok x k] . W^T on device buffers; the batched form of
 * kernels::matmul_q4_0 (turbo::batch_matmul for mtok > 1). */
int hc_q4_matmul_dev(const hc_q4_matrix* w, const float* x, size_t mtok, float* y, void* stream);

/* The same product as hc_q4_matmul_dev for callers that cannot allocate
 * device memory while running (a serving process whose device memory is all
 * handed to its own pool at start-up, or code that may not call cudaMalloc,
 * which can synchronize the device, while other work is in flight).  This
 * entry point has no counterpart in the reference engine.  It allocates
 * nothing: tensor-core shapes (mtok >= 2, k % 256 == 0, n >= 128) keep their
 * scratch (the hi + lo fp16 rows of x, mtok * k * 4 bytes, and the kernel's
 * abort flag) in a fixed 8 MiB array inside the library's device image (held
 * by every GPU that loads the library until the process exits) and require
 * mtok * k * 4 <= 8 MiB - 256 bytes, else HC_ERR_INVALID; other shapes use the
 * CUDA-core matvec, which needs no scratch and does not synchronize.  On the
 * tensor-core path the call waits for the stream to finish the product so
 * that it can read the abort flag: HC_ERR_TIMEOUT when a bounded pipeline
 * wait ran out (y is then not written).  The first call on a device looks up
 * the array's device address (cudaGetSymbolAddress) and should come before
 * any stream capture; the cached address belongs to the device's primary
 * context, so it is stale after cudaDeviceReset.  Every call shares the
 * array: calls that overlap on the GPU (different streams, or different host
 * threads on one device) race, so order them on one stream. */
int hc_q4_matmul_noalloc(const hc_q4_matrix* w, const float* x, size_t mtok, float* y, void* stream);

/* ---- model level: the forward passes ---------------------------------- */

typedef struct hc_model hc_model;
typedef struct hc_kv hc_kv;

/* HypnoConfig, transformer.rs:27-63 (head_dim = hidden / heads). */
typedef struct hc_config {
    uint64_t hidden_size;
    uint64_t intermediate_size;
    uint64_t num_attention_heads;
    uint64_t num_key_value_heads;
    uint64_t num_hidden_layers;
    uint64_t vocab_size;
    uint64_t max_position_embeddings;
    uint64_t head_dim;
    float rms_norm_eps;
    float rope_theta;
    uint32_t embed_dtype;   /* dtype of model.embed_tokens.weight */
    uint32_t lm_head_dtype; /* dtype of the LM head actually used */
    int32_t lm_head_tied;   /* 1 when the LM head is the embedding */
    int32_t tp_rank;
    int32_t tp_size;
    int32_t reserved;
} hc_config;

/* HypnoModel::open + HypnoConfig::from_model (loader.rs:39-133,
 * transformer.rs:42-63): parses a .hypno image held in host memory (the bytes
 * the reference mmaps), validates offsets, and uploads every weight once,
 * repacking Q4_0 into the device layout.  tp_size 1 = whole model; tp_size > 1
 * keeps the tp_rank shard of the attention heads and FFN columns. */
int hc_model_load(const uint8_t* image, size_t len, int tp_rank, int tp_size, hc_model** out);
int hc_model_config(const hc_model* model, hc_config* out);
int hc_model_free(hc_model* model);
/* Blocks until all work queued on the model's stream is done. */
int hc_sync(hc_model* model);
/* The model's CUDA stream (cudaStream_t) for callers that interleave work. */
void* hc_model_stream(hc_model* model);

/* FlatKVCache, transformer.rs:89-184: n_seqs independent caches of max_pos
 * positions each (kv_dtype HC_KV_FP32 = the reference's layout; HC_KV_FP16
 * halves the bytes).  All positions start at 0. */
int hc_kv_alloc(hc_model* model, int n_seqs, int max_pos, int kv_dtype, hc_kv** out);
int hc_kv_free(hc_kv* kv);
/* FlatKVCache::seq_len / set_pos / clear, transformer.rs:118-121,157-176. */
int hc_kv_seq_len(const hc_kv* kv, int seq, int* out);
int hc_kv_set_pos(hc_kv* kv, int seq, int pos);

/* turbo::batch_forward, turbo.rs:22-281: runs the T prompt tokens of
 * sequence `seq` through all layers, stores their K/V at positions
 * [pos, pos+T) and advances the position.  logits_out (vocab floats, host)
 * receives the last token's logits (zeros when T == 0); may be NULL. */
int hc_prefill(hc_model* model, hc_kv* kv, int seq, const uint32_t* ids, int T, float* logits_out);

/* transformer::model_forward (use_kv_cache = true), transformer.rs:465-528,
 * batched over B sequences: seqs[b] decodes token ids[b] at its current
 * position, then advances.  logits_out (B x vocab, host) and argmax_out
 * (B ids, host; greedy = last maximal index, the tie rule of Rust's max_by
 * used by run.rs:234-238) may each be NULL. */
int hc_decode_step(hc_model* model, hc_kv* kv, const int* seqs, const uint32_t* ids, int B,
                   float* logits_out, uint32_t* argmax_out);

/* Device-resident form of hc_decode_step: seqs/ids are device arrays of B
 * entries, logits_out (B x vocab) and argmax_out (B) are device buffers (each
 * may be NULL).  Ordered on the model's stream, no synchronization. */
int hc_decode_step_dev(hc_model* model, hc_kv* kv, const int* seqs_dev, const uint32_t* ids_dev,
                       int B, float* logits_dev, uint32_t* argmax_dev);

/* Instrumentation for benchmarks (no reference counterpart): one decode step
 * as hc_decode_step_dev (argmax only), launched without a CUDA graph and with
 * a CUDA event between phases; waits for the step and ADDS each phase's
 * device milliseconds to phase_ms[0 .. hc_phase_count()).  Phase i is named
 * by hc_phase_name(i) (embedding, norms, each projection GEMM, RoPE + KV
 * store, attention, the reduction + residual + norm after o/down, LM head,
 * logits exchange, argmax). */
int hc_decode_step_phases(hc_model* model, hc_kv* kv, const int* seqs_dev, const uint32_t* ids_dev, int B,
                          uint32_t* argmax_dev, float* phase_ms);
int hc_phase_count(void);
const char* hc_phase_name(int i);

/* ---- sampling ---------------------------------------------------------- */

/* run.rs:203-278 (sample_token with XorShift64::next_f32) for B rows of device
 * logits (row stride ld floats, V entries each), one token per row, on the
 * device: per-row temperature (exp(l / T) when T > 0, raw logits otherwise),
 * top_k (0 = off) and top_p (1 = off) as device arrays of B, and a device
 * array of B XorShift64 states (the caller seeds state = max(seed, 1)); a row
 * that draws advances its state by one step.  Every sum is added in f32 in
 * the reference's order, one term at a time (about one add latency per logit
 * and pass: a few hundred microseconds per row at V = 128256); exp is CUDA's
 * expf, so only a draw within a few ulp of a boundary can differ from the
 * reference.  Stream-ordered, no synchronization. */
int hc_sample_dev(const float* logits_dev, size_t ld, int B, int V, const float* temperature_dev,
                  const float* top_p_dev, const int* top_k_dev, uint64_t* rng_state_dev, uint32_t* out_dev,
                  void* stream);

/* run.rs:234-238, 249 and serve.rs:300, 304 (the greedy pick,
 * Iterator::max_by with partial_cmp(..).unwrap_or(Equal)) for B rows of
 * device logits (row stride ld floats, V entries each): out_dev[b] = the last
 * maximal index after the row's last NaN, or that NaN's index when it ends
 * the row (a NaN compares Equal, so the fold takes it and then the element
 * after it); the last maximal index when there is no NaN.  shards > 1 splits
 * every row into that many equal vocabulary slices (V % shards == 0), picks
 * per slice and folds the slices' picks in order, the kernels a
 * tensor-parallel LM head runs across its ranks; pairs_dev is then device
 * scratch of 2 * shards * B floats (may be NULL for shards == 1).
 * Stream-ordered, no synchronization. */
int hc_argmax_dev(const float* logits_dev, size_t ld, int B, int V, int shards, float* pairs_dev, uint32_t* out_dev,
                  void* stream);

/* ---- tensor parallelism (new in this backend; the reference is single-CPU) */

/* Writes a fresh 128-byte NCCL unique id (rank 0 creates it and shares it
 * with the other ranks by any host channel). */
int hc_comm_unique_id(uint8_t* out128);
/* Joins the tensor-parallel group of a model loaded with
 * hc_model_load(..., rank, size, ...).  The all-reduce after o_proj and
 * down_proj and the all-gather of the vocabulary-sharded logits then run on
 * the model's stream.  Decode-sized all-reduces (up to 256 rows) read the
 * peers' partial sums over CUDA-IPC-mapped device memory, fused with the
 * residual add and the next RMSNorm; NCCL carries larger ones, and all of
 * them when the environment sets HC_PEER_ALLREDUCE=0 or a peer cannot be
 * mapped.  Host waits of the model (hc_sync, hc_prefill,
 * hc_decode_step) are watched: a collective that does not finish within
 * timeout_s seconds (<= 0: 60) aborts the communicator and returns
 * HC_ERR_TIMEOUT. */
int hc_comm_init(hc_model* model, const uint8_t* id128, int rank, int size, double timeout_s);

/* ---- synthetic inputs (seeded; identical bytes on host and device) ----- */

/* Fills out[i] (i < n) with element offset+i of the seeded stream
 * (seed, stream): a 12-term Irwin-Hall sum of 16-bit uniforms, centred and
 * scaled by std/65536 — mean 0, variance std^2 — built from integer steps
 * and one IEEE multiply so host and device produce identical floats. */
int hc_synth_normal_host(uint64_t seed, uint64_t stream, uint64_t offset, uint64_t n, float std,
                         float* out);
int hc_synth_normal_dev(uint64_t seed, uint64_t stream, uint64_t offset, uint64_t n, float std,
                        float* out, void* cuda_stream);

#ifdef __cplusplus
}
#endif

#endif /* HYPNO_CUDA_H */
