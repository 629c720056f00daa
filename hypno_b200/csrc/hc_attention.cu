// GQA attention over the HBM-resident KV cache with the reference's exact
// visibility rule and softmax weight function.
//
// Decode (transformer.rs:346-413): a token at position p (p tokens already
// cached) stores its K/V at p but attends only to cached positions [0, p);
// for p <= 1 the output is its own V (softmax of one element == 1.0).
// Prefill (turbo.rs:144-185): prompt token t attends to prompt tokens
// [0, t) for t >= 2, to its own V for t < 2; the K/V used are the prompt's
// own (f32) projections, never older cache entries.
// Softmax (kernels.rs:631-697): max, then the exp(v/8) Taylor polynomial on
// entries below floor(n/8)*8 and libm exp on the rest, normalised by the sum.
// Because the polynomial is not an exponential, weights cannot be rescaled
// online: scores are materialised first (shared memory), then weighted.
#include "hc_internal.h"
#include "hc_common.cuh"
#include "hc_attention.h"

namespace hc {

template <typename KT>
__device__ __forceinline__ float ldkv(const KT* p);
template <>
__device__ __forceinline__ float ldkv<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ldkv<__half>(const __half* p) { return __half2float(*p); }

// One CTA (4 warps) per (query row, query head).
template <typename KT>
__global__ void __launch_bounds__(128) k_attention(AttnParams P) {
    extern __shared__ float smem[];
    const int row = blockIdx.x, h = blockIdx.y;
    const int hd = P.hd;
    const int kvh = h / (P.nh / P.nkv);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __shared__ float red[32];

    const float* q = P.q + (size_t)row * P.ldq + (size_t)h * hd;
    float* out = P.out + (size_t)row * P.ldo + (size_t)h * hd;
    const float* vself = P.vself + (size_t)row * P.ldself + (size_t)kvh * hd;

    int n;
    const KT* kbase;
    const KT* vbase;
    size_t kstride;
    if (P.mode_prefill) {
        n = row;  // prompt-relative position
        kbase = reinterpret_cast<const KT*>(P.kp) + (size_t)kvh * hd;
        vbase = reinterpret_cast<const KT*>(P.vp) + (size_t)kvh * hd;
        kstride = P.ldkv;
    } else {
        int seq = P.seqs[row];
        n = min(P.pos[seq], P.smem_n);
        size_t off = (size_t)seq * P.seq_stride + (size_t)kvh * P.head_stride;
        kbase = reinterpret_cast<const KT*>(P.kc) + off;
        vbase = reinterpret_cast<const KT*>(P.vc) + off;
        kstride = hd;
    }

    if (n <= 1) {
        for (int d = threadIdx.x; d < hd; d += blockDim.x) out[d] = vself[d];
        return;
    }

    float* scores = smem;             // n floats
    float* part = smem + P.smem_n;    // 4 * hd floats

    // scores[p] = (q . k_p) * scale
    for (int p = warp; p < n; p += 4) {
        const KT* kp = kbase + (size_t)p * kstride;
        float dot = 0.0f;
        for (int d = lane; d < hd; d += 32) dot = fmaf(q[d], ldkv<KT>(kp + d), dot);
        dot = warp_sum(dot);
        if (lane == 0) scores[p] = __fmul_rn(dot, P.scale);
    }
    __syncthreads();
    float mx = -INFINITY;
    for (int p = threadIdx.x; p < n; p += blockDim.x) mx = fmaxf(mx, scores[p]);
    mx = block_max(mx, red);
    const int n8 = n - (n % 8);
    float sum = 0.0f;
    for (int p = threadIdx.x; p < n; p += blockDim.x) {
        float e = softmax_weight(scores[p], mx, p, n8);
        scores[p] = e;
        sum += e;
    }
    float total = block_sum(sum, red);
    float inv = __fdiv_rn(1.0f, total);
    for (int p = threadIdx.x; p < n; p += blockDim.x)
        scores[p] = (p < n8) ? __fmul_rn(scores[p], inv) : __fdiv_rn(scores[p], total);
    __syncthreads();

    // out[d] = sum_p w_p v_p[d]; warp w takes positions w, w+4, ...
    for (int d = lane; d < hd; d += 32) {
        float acc = 0.0f;
        for (int p = warp; p < n; p += 4) acc = fmaf(scores[p], ldkv<KT>(vbase + (size_t)p * kstride + d), acc);
        part[warp * hd + d] = acc;
    }
    __syncthreads();
    for (int d = threadIdx.x; d < hd; d += blockDim.x)
        out[d] = (part[d] + part[hd + d]) + (part[2 * hd + d] + part[3 * hd + d]);
}

int launch_attention(const AttnParams& P, int rows, int kv_fp16, cudaStream_t s) {
    if (rows == 0) return HC_OK;
    size_t smem = ((size_t)P.smem_n + 4 * (size_t)P.hd) * sizeof(float);
    if (smem > 200 * 1024) {
        hc_set_error("attention: context %d too long for the shared-memory score buffer", P.smem_n);
        return HC_ERR_UNSUPPORTED;
    }
    dim3 grid((unsigned)rows, (unsigned)P.nh);
    if (kv_fp16) {
        if (smem > 48 * 1024) HC_CUDA(cudaFuncSetAttribute(k_attention<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        k_attention<__half><<<grid, 128, smem, s>>>(P);
    } else {
        if (smem > 48 * 1024) HC_CUDA(cudaFuncSetAttribute(k_attention<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        k_attention<float><<<grid, 128, smem, s>>>(P);
    }
    HC_LAUNCH_CHECK();
    return HC_OK;
}

// Stores the (rotated) K and V of each row into the cache:
// cache[seq][layer][kvh][pos][hd] (FlatKVCache::store / store_at,
// transformer.rs:124-139, 161-173).  decode: seq = seqs[row], pos = pos[seq];
// prefill: seq = fixed_seq, pos = pos0 + row.
template <typename KT>
__global__ void k_kv_store(const float* __restrict__ k, const float* __restrict__ v, size_t ld, int nkv, int hd,
                           KT* __restrict__ kc, KT* __restrict__ vc, size_t seq_stride, size_t head_stride,
                           int max_pos, const int* __restrict__ seqs, const int* __restrict__ pos, int fixed_seq,
                           int pos0) {
    int row = blockIdx.y;
    int seq = seqs ? seqs[row] : fixed_seq;
    int p = seqs ? pos[seq] : pos0 + row;
    if (p < 0 || p >= max_pos) return;  // capacity guard: never write past the sequence's region
    int total = nkv * hd;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        int h = i / hd, d = i % hd;
        size_t off = (size_t)seq * seq_stride + (size_t)h * head_stride + (size_t)p * hd + d;
        float kv = k[(size_t)row * ld + i], vv = v[(size_t)row * ld + i];
        if constexpr (sizeof(KT) == 2) {
            kc[off] = __float2half_rn(kv);
            vc[off] = __float2half_rn(vv);
        } else {
            kc[off] = kv;
            vc[off] = vv;
        }
    }
}

int launch_kv_store(const float* k, const float* v, size_t ld, int rows, int nkv, int hd, void* kc, void* vc,
                    int kv_fp16, size_t seq_stride, size_t head_stride, int max_pos, const int* seqs, const int* pos,
                    int fixed_seq, int pos0, cudaStream_t s) {
    if (rows == 0) return HC_OK;
    unsigned gx = (unsigned)((nkv * hd + 255) / 256);
    if (gx > 16) gx = 16;
    dim3 grid(gx, (unsigned)rows);
    if (kv_fp16)
        k_kv_store<__half><<<grid, 256, 0, s>>>(k, v, ld, nkv, hd, (__half*)kc, (__half*)vc, seq_stride, head_stride,
                                                 max_pos, seqs, pos, fixed_seq, pos0);
    else
        k_kv_store<float><<<grid, 256, 0, s>>>(k, v, ld, nkv, hd, (float*)kc, (float*)vc, seq_stride, head_stride,
                                                max_pos, seqs, pos, fixed_seq, pos0);
    HC_LAUNCH_CHECK();
    return HC_OK;
}

// pos[seqs[b]] += 1 after a decode step (FlatKVCache::advance,
// transformer.rs:158, 508-510).
__global__ void k_advance(const int* __restrict__ seqs, int* __restrict__ pos, int B) {
    int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < B) pos[seqs[b]] += 1;
}

int launch_advance(const int* seqs, int* pos, int B, cudaStream_t s) {
    if (B == 0) return HC_OK;
    k_advance<<<(B + 127) / 128, 128, 0, s>>>(seqs, pos, B);
    HC_LAUNCH_CHECK();
    return HC_OK;
}

}  // namespace hc
