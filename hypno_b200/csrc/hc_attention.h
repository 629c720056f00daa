// Attention / KV-cache launch interface (see hc_attention.cu).
#pragma once
#include "hc_internal.h"

namespace hc {

struct AttnParams {
    const float* q;       // query rows; head h at q + row*ldq + h*hd
    size_t ldq;
    float* out;           // output rows; head h at out + row*ldo + h*hd
    size_t ldo;
    const float* vself;   // f32 V of the row's own token; kv head at + kvh*hd
    size_t ldself;
    int nh, nkv, hd;
    float scale;          // 1/sqrt(hd)
    int smem_n;           // capacity of the score buffer (>= max positions attended)
    int mode_prefill;     // 1: K/V rows come from kp/vp (prompt-relative)
    // decode source: cache[seq][layer][kvh][max_pos][hd], already offset to the layer
    const void* kc;
    const void* vc;
    size_t seq_stride, head_stride;
    const int* seqs;      // row -> sequence
    const int* pos;       // sequence -> cached positions before this step
    // prefill source: f32 K/V rows of the prompt with row stride ldkv
    const float* kp;
    const float* vp;
    size_t ldkv;
    __half* out16 = nullptr;  // optional fp16 copy of out (rows of nh*hd, GEMM K order)
    // prefill scratch (may be null): 4 planes of [T][nkv*hd] fp16 (K hi, K lo,
    // V hi, V lo), filled by launch_prefill_attention for the tensor-core kernel
    __half* kv16 = nullptr;
    int cluster = 1;          // > 1: that many CTAs of a cluster share a (sequence, KV head), chunk positions each
};

int launch_attention(const AttnParams& P, int rows, int kv_fp16, cudaStream_t s);
int launch_kv_store(const float* k, const float* v, size_t ld, int rows, int nkv, int hd, void* kc, void* vc,
                    int kv_fp16, size_t seq_stride, size_t head_stride, int max_pos, const int* seqs,
                    const int* pos, int fixed_seq, int pos0, cudaStream_t s);
int launch_advance(const int* seqs, int* pos, int B, cudaStream_t s);

// Grouped (GQA) decode attention, see hc_attention.cu.  cluster > 1 runs one
// pass per (sequence, KV head) split over a thread-block cluster; otherwise
// nsplit == 1 runs one fused pass per pair (chunk must equal max_pos) and
// nsplit > 1 runs scores / weighted-V / combine over splits of chunk positions.
constexpr int DA_REDUCE_WARPS = 8;  // warps per attention CTA
struct DecAttnParams {
    const float* q;       // query rows, head h at q + row*ldq + h*hd
    size_t ldq;
    float* out;
    size_t ldo;
    const float* vself;   // own f32 V of each row, kv head at + kvh*hd
    size_t ldself;
    int nh, nkv, hd;
    float scale;
    const void* kc;       // cache for this layer: [seq][.][kvh][max_pos][hd]
    const void* vc;
    size_t seq_stride, head_stride;
    const int* seqs;
    const int* pos;
    int max_pos;
    int chunk;            // positions per split
    int nsplit;           // splits launched (>= ceil(max n / chunk))
    float* S;             // scores [rows][nkv][max_pos][G] (G = nh / nkv)
    float* smax;          // [rows][nh][nsplit]
    float* opart;         // [rows][nh][nsplit][hd]
    float* spart;         // [rows][nh][nsplit]
    __half* out16 = nullptr;  // optional fp16 copy of out (rows of nh*hd, GEMM K order)
    // prefill scratch (may be null): 4 planes of [T][nkv*hd] fp16 (K hi, K lo,
    // V hi, V lo), filled by launch_prefill_attention for the tensor-core kernel
    __half* kv16 = nullptr;
    int cluster = 1;          // > 1: that many CTAs of a cluster share a (sequence, KV head), chunk positions each
    int wide = 0;             // whole context (nsplit 1): one 16-warp CTA per SM (see dattn_wide_ok)
};
bool dattn_supported(int nh, int nkv, int hd);
// The whole-context pass with one 16-warp CTA per (sequence, KV head) is
// available (fp16 cache, 1, 2 or 4 heads per KV head, head_dim 64 or 128,
// scores of max_pos positions in shared memory).
bool dattn_wide_ok(int nh, int nkv, int hd, int max_pos, int kv_fp16);
// Tiled f32 prefill attention over the prompt's own K/V rows (mode_prefill).
bool pattn_supported(int hd);
int launch_prefill_attention(const AttnParams& P, int T, cudaStream_t s);
int launch_decode_attention(const DecAttnParams& P, int rows, int kv_fp16, cudaStream_t s);

}  // namespace hc
