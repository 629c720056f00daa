// Internal declarations shared by the translation units of libhypno_cuda.so.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stddef.h>
#include <string>
#include <vector>

#include "../../include/hypno_cuda.h"

#define HC_EXPORT extern "C" __attribute__((visibility("default")))

// ---------------------------------------------------------------- errors
void hc_set_error(const char* fmt, ...);
int hc_cuda_fail(cudaError_t e, const char* what, const char* file, int line);

#define HC_CUDA(call)                                                              \
    do {                                                                           \
        cudaError_t _e = (call);                                                   \
        if (_e != cudaSuccess) return hc_cuda_fail(_e, #call, __FILE__, __LINE__); \
    } while (0)

#define HC_CHECK(cond, code, ...)         \
    do {                                  \
        if (!(cond)) {                    \
            hc_set_error(__VA_ARGS__);    \
            return (code);                \
        }                                 \
    } while (0)

#define HC_TRY(expr)             \
    do {                         \
        int _r = (expr);         \
        if (_r != HC_OK) return _r; \
    } while (0)

// Launch-error check after a kernel launch; also counts the launch (every
// kernel launch of the library is followed by this macro).
void hc_count_launch();
void hc_count_launches(size_t n);
#define HC_LAUNCH_CHECK()          \
    do {                           \
        hc_count_launch();         \
        HC_CUDA(cudaGetLastError()); \
    } while (0)

// ---------------------------------------------------------------- Q4_0 matrix
// Device layout of a Q4_0 tensor.  The .hypno payload is a sequence of
// 18-byte blocks (f16 scale + 16 nibble bytes) over the flattened row-major
// tensor (quant.rs:10-18, kernels.rs:273-283).  On the device the blocks are
// split into two planes so every load is aligned and coalesced:
//   qs[b]  : 16 nibble bytes of block b (uint4, 16-byte aligned)
//   sc[b]  : fp16 scale of block b
// Block order is unchanged (flattened row-major), so for k % 32 == 0 row r
// owns blocks [r*k/32, (r+1)*k/32).  The split is exactly invertible.
struct hc_q4_matrix {
    size_t n = 0, k = 0, nblocks = 0;
    uint4* qs = nullptr;
    __half* sc = nullptr;
    bool owns = true;
};

// Dense weight of any supported dtype resident in HBM.
struct DevWeight {
    uint32_t dtype = 0;  // HC_DTYPE_*
    size_t n = 0, k = 0;
    hc_q4_matrix q4;     // dtype == Q4_0
    void* dense = nullptr;  // FP32 / FP16 payload
    bool present = false;
};

// ---------------------------------------------------------------- kernels
namespace hc {

enum Epi : int { EPI_STORE = 0, EPI_ADD = 1, EPI_SILU = 2 };  // EPI_SILU: tensor-core GEMM only
// Rows of the fused gate/up weight alternate in blocks of GU_BLOCK gate rows
// then the matching GU_BLOCK up rows (when the intermediate size allows), so
// one 128-row GEMM tile holds both halves of 64 SiLU-gate outputs.
constexpr int GU_BLOCK = 64;

// Q4_0 pack / unpack / repack (bit-exact with quant.rs).
int launch_q4_quantize(const float* x, size_t nblocks, uint8_t* out, cudaStream_t s);
int launch_q4_dequantize(const uint8_t* q, size_t nblocks, float* out, cudaStream_t s);
int launch_q4_split(const uint8_t* aos, size_t nblocks, uint4* qs, __half* sc, cudaStream_t s);

// Y[m][n] (+)= X[m][:] . W[n][:]  for m < mtok.  ldx/ldy in floats.
// res (may alias y, may be null) is added when epi == EPI_ADD: y = acc + res.
int launch_matmul(const DevWeight& w, const float* x, size_t ldx, size_t mtok, float* y, size_t ldy,
                  int epi, const float* res, size_t ldres, cudaStream_t s);

// Row-wise RMSNorm (kernels.rs:592-625): out[r] = x[r] * inv_rms(x[r]) * w.
// out16 (may be null): the same rows in fp16, in the tensor-core GEMM's K order.
// hidden[r] += sum of the split slabs part[i][r] (slab order; slab i at
// part + i * rows * n), then, when w is given, xn[r] = RMSNorm(hidden[r]) * w
// and its fp16 copy in GEMM K order (xn16 may be null).
bool residual_splits_norm_ok(size_t n, size_t ldh, size_t ldxn);
int launch_residual_splits_norm(const float* part, int splits, size_t rows, size_t n, float* hidden, size_t ldh,
                                const float* w, float eps, float* xn, size_t ldxn, __half* xn16, cudaStream_t s);
// Single-token Q4_0 matvec y = W . RMSNorm(x) * norm_w (x one row of w.k
// floats), with the norm computed inside the kernel; silu: W is a blocked
// fused gate/up weight and y gets its w.n / 2 SiLU-gated outputs.  Only where
// gemv1_fusable holds (Q4_0, k % 32 == 0, k <= 24576, 16-byte aligned x and
// norm_w, whole gate/up blocks).
bool gemv1_fusable(const DevWeight& w, const float* x, const float* norm_w, bool silu);
int launch_gemv1_fused(const DevWeight& w, const float* x, float* y, const float* norm_w, float eps, bool silu,
                       cudaStream_t s);
// Launches kfn as a programmatic dependent of the stream's previous kernel:
// its CTAs may become resident while that kernel still runs, which hides the
// launch gap of short dependent kernels (the single-token decode chain).
// kfn must call pdl_wait() before its first global memory access.
template <typename... KArgs, typename... Args>
inline int launch_pdl(void (*kfn)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    HC_CUDA(cudaLaunchKernelEx(&cfg, kfn, args...));
    return HC_OK;
}

int launch_rmsnorm(const float* x, size_t ldx, const float* w, float* out, size_t ldo, size_t rows,
                   size_t n, float eps, cudaStream_t s, __half* out16 = nullptr);
int launch_softmax_rows(float* x, size_t rows, size_t n, cudaStream_t s);
int launch_silu(float* x, size_t n, cudaStream_t s);
// act[r][i] = silu(gu[r][i]) * gu[r][im + i] (blocked: gate/up alternate in
// blocks of GU_BLOCK columns); splits > 1: gu holds that many split-K slabs of
// [rows][ldgu] (slab i at gu + i * rows * ldgu), added in slab order first
int launch_silu_mul(const float* gu, size_t ldgu, float* act, size_t ldact, size_t rows, size_t im,
                    cudaStream_t s, __half* act16 = nullptr, bool blocked = false, int splits = 1);
// x[row] = sum of the split slabs part[i][row] (slab order; slab i at part +
// i * rows * width, `width` elements per row), the first `heads` heads then
// rotated as launch_rope_rows does.
// kv (optional): also store the row's k and v elements (the nk elements at
// nq, then the nk at nq + nk) into the cache as launch_kv_store does.
struct KvStoreArgs {
    void* kc = nullptr;  // null: no store
    void* vc = nullptr;
    int kv_fp16 = 0;
    size_t seq_stride = 0, head_stride = 0;
    int max_pos = 0;
    const int* seqs = nullptr;  // row -> sequence (decode); null: fixed_seq, position pos0 + row
    const int* pos = nullptr;   // sequence -> cached positions
    int fixed_seq = 0, pos0 = 0;
    int nq = 0, nk = 0;         // k block at element nq, v block at nq + nk (nk = kv heads x head_dim)
};
int launch_rope_rows_slabs(const float* part, int splits, float* x, size_t ldx, size_t rows, size_t width,
                           size_t heads, size_t hd, const float2* cs, size_t cs_rows, const int* pos_dev, int pos0,
                           cudaStream_t s, const KvStoreArgs* kv = nullptr);
// Rotation of `heads` adjacent-pair heads per row at position pos0 + row
// using a (max_pos x hd/2) cos/sin table.
int launch_rope_rows(float* x, size_t ldx, size_t rows, size_t heads, size_t hd, const float2* cs, size_t cs_rows,
                     const int* pos_dev, int pos0, cudaStream_t s);

// Embedding gather for B ids (FP32 / FP16 / Q4_0 rows of width hidden).
int launch_embed(const DevWeight& emb, const uint32_t* ids, size_t B, float* out, size_t hidden,
                 cudaStream_t s);
int launch_argmax(const float* logits, size_t rows, size_t n, uint32_t* out, cudaStream_t s);
int launch_argmax(const float* logits, size_t rows, size_t n, size_t ld, uint32_t* out, cudaStream_t s);
// pairs[row] = (max of the row, bits of idx0 + its last maximal index)
int launch_argmax_pairs(const float* logits, size_t rows, size_t n, size_t ld, uint32_t idx0, float2* pairs,
                        cudaStream_t s);
// Greedy ids from [tp][rows] shard pairs (launch_argmax_pairs), shards in
// vocabulary order.
int launch_pick_pairs(const float2* pairs, size_t rows, int tp, uint32_t* out, cudaStream_t s);

// Synthetic normal stream (host and device versions agree bit for bit).
int launch_synth_normal(uint64_t seed, uint64_t stream, uint64_t offset, uint64_t n, float std,
                        float* out, cudaStream_t s);

}  // namespace hc

// RoPE angle table computed on the host with the C library's powf/cosf/sinf
// (the functions Rust's f32 methods call on Linux), transformer.rs:317-343.
std::vector<float2> hc_rope_table(size_t max_pos, size_t hd, float theta);

// Host-side f16 helpers.
uint16_t hc_f32_to_f16_host(float f);
float hc_f16_to_f32_host(uint16_t h);
