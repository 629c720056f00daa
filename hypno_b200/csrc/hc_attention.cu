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
#include "hc_gemm.h"

namespace hc {

template <typename KT>
__device__ __forceinline__ float ldkv(const KT* p);
template <>
__device__ __forceinline__ float ldkv<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ldkv<__half>(const __half* p) { return __half2float(*p); }

// Four consecutive K/V elements as f32 (16-byte / 8-byte aligned loads).
template <typename KT>
__device__ __forceinline__ float4 ld4(const KT* p);
template <>
__device__ __forceinline__ float4 ld4<float>(const float* p) { return *reinterpret_cast<const float4*>(p); }
template <>
__device__ __forceinline__ float4 ld4<__half>(const __half* p) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
}

// One CTA (4 warps) per (query row, query head): the path for head sizes and
// group sizes the tiled kernels do not take (e.g. 9 query heads over 3 KV
// heads).  Scores: one thread per position (its whole dot product, 4
// elements per load); weighted V: thread (position group, column quad) adds
// the weights times 4 columns over its group's positions, and the groups'
// sums are added in group order (4 elements per load when head_dim is a
// multiple of 4).  HD > 0 fixes head_dim at compile time (64, 128), so a
// score's loads are all in flight at once and the weighted-V loop keeps
// eight rows in flight; HD = 0 takes it from P.
template <typename KT, int HD>
__global__ void __launch_bounds__(128) k_attention(AttnParams P) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ float smem[];
    const int row = blockIdx.x, h = blockIdx.y;
    const int hd = HD > 0 ? HD : P.hd;
    const int kvh = h / (P.nh / P.nkv);
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
        for (int d = threadIdx.x; d < hd; d += blockDim.x) {
            out[d] = vself[d];
            if (P.out16) store_x16(P.out16 + (size_t)row * 2 * P.nh * hd, P.nh * hd, h * hd + d, vself[d]);
        }
        return;
    }

    // scores (smem_n floats, padded to a multiple of 4 so the float4 partial
    // sums below stay 16-byte aligned), q (hd floats), the groups' partials
    float* scores = smem;
    float* qs = smem + ((P.smem_n + 3) & ~3);
    float* part = qs + hd;  // [groups][hd]
    for (int d = threadIdx.x; d < hd; d += blockDim.x) qs[d] = q[d];
    __syncthreads();

    const bool vec = (hd & 3) == 0;  // 4 elements per load (every row start is then aligned)
    // scores[p] = (q . k_p) * scale, in element order
    for (int p = threadIdx.x; p < n; p += blockDim.x) {
        const KT* kp = kbase + (size_t)p * kstride;
        float dot = 0.0f;
        if (vec) {
#pragma unroll
            for (int d = 0; d < hd; d += 4) {
                const float4 k4 = ld4<KT>(kp + d);
                dot = fmaf(qs[d], k4.x, dot);
                dot = fmaf(qs[d + 1], k4.y, dot);
                dot = fmaf(qs[d + 2], k4.z, dot);
                dot = fmaf(qs[d + 3], k4.w, dot);
            }
        } else {
            for (int d = 0; d < hd; d++) dot = fmaf(qs[d], ldkv<KT>(kp + d), dot);
        }
        scores[p] = __fmul_rn(dot, P.scale);
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

    // out[d] = sum_p w_p v_p[d]
    const int cols = vec ? hd / 4 : hd, groups = max(1, (int)blockDim.x / cols);
    for (int t = threadIdx.x; t < groups * cols; t += blockDim.x) {
        const int c = t % cols, grp = t / cols;
        if (vec) {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
            for (int p = grp; p < n; p += groups) {
                const float w = scores[p];
                const float4 v4 = ld4<KT>(vbase + (size_t)p * kstride + 4 * c);
                acc.x = fmaf(w, v4.x, acc.x);
                acc.y = fmaf(w, v4.y, acc.y);
                acc.z = fmaf(w, v4.z, acc.z);
                acc.w = fmaf(w, v4.w, acc.w);
            }
            *reinterpret_cast<float4*>(part + (size_t)grp * hd + 4 * c) = acc;
        } else {
            float acc = 0.0f;
            for (int p = grp; p < n; p += groups) acc = fmaf(scores[p], ldkv<KT>(vbase + (size_t)p * kstride + c), acc);
            part[(size_t)grp * hd + c] = acc;
        }
    }
    __syncthreads();
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float o = part[d];
        for (int g = 1; g < groups; g++) o = o + part[(size_t)g * hd + d];
        out[d] = o;
        if (P.out16) store_x16(P.out16 + (size_t)row * 2 * P.nh * hd, P.nh * hd, h * hd + d, o);
    }
}

int launch_attention(const AttnParams& P, int rows, int kv_fp16, cudaStream_t s) {
    if (rows == 0) return HC_OK;
    HC_CHECK(P.hd >= 1, HC_ERR_INVALID, "attention: head_dim %d", P.hd);
    // scores, q, and the weighted-V partial sums of the position groups
    const size_t cols = P.hd % 4 == 0 ? (size_t)P.hd / 4 : (size_t)P.hd;
    const size_t groups = std::max<size_t>(1, 128 / cols);
    size_t smem = ((((size_t)P.smem_n + 3) & ~(size_t)3) + (1 + groups) * (size_t)P.hd) * sizeof(float);
    if (smem > 200 * 1024) {
        hc_set_error("attention: context %d too long for the shared-memory score buffer", P.smem_n);
        return HC_ERR_UNSUPPORTED;
    }
    dim3 grid((unsigned)rows, (unsigned)P.nh);
    auto run = [&](auto kfn) -> int {
        if (smem > 48 * 1024) HC_CUDA(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        return launch_pdl(kfn, grid, dim3(128), smem, s, P);
    };
    if (kv_fp16) {
        if (P.hd == 64) return run(k_attention<__half, 64>);
        if (P.hd == 128) return run(k_attention<__half, 128>);
        return run(k_attention<__half, 0>);
    }
    if (P.hd == 64) return run(k_attention<float, 64>);
    if (P.hd == 128) return run(k_attention<float, 128>);
    return run(k_attention<float, 0>);
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
    pdl_trigger();
    pdl_wait();
    int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < B) pos[seqs[b]] += 1;
}

int launch_advance(const int* seqs, int* pos, int B, cudaStream_t s) {
    if (B == 0) return HC_OK;
    HC_TRY(launch_pdl(k_advance, dim3((B + 127) / 128), dim3(128), 0, s, seqs, pos, B));
    return HC_OK;
}



// ============================================================ grouped decode attention
//
// Decode attention for long contexts, grouped by KV head: one CTA per
// (sequence, kv head, position split) serves all G = nh/nkv query heads of
// the group, so each K/V row is read once per group instead of once per
// query head.  The reference's softmax weight depends on the row maximum
// through a polynomial (not an exponential), so partial results cannot be
// rescaled: pass 1 writes the scores and a per-split maximum, pass 2 takes
// the global maximum, forms the weights and the partial P.V, pass 3 (only
// with several splits) adds the partials and normalises.
namespace {

constexpr int DA_WARPS = DA_REDUCE_WARPS;
constexpr int DA_THREADS = DA_WARPS * 32;
constexpr int DA_MAXG = 8;

// Lane-group mapping for one (sequence, KV head): LPP lanes share a K or V
// row, each lane owning EPL consecutive elements of it (32 bytes, 16 bytes for
// groups of 4 or more heads), so a warp reads whole rows with coalesced
// 16-byte loads and keeps its slice of the G query vectors in registers.  U
// row groups are loaded before any arithmetic to keep enough bytes in flight.
// Scores and weights are stored position-major, [p][G], so the weighted-V
// pass reads a row's G weights with one vector load.
template <typename KT, int G, int HD>
struct DA {
    static constexpr int BPL = (G <= 2) ? 32 : 16;                  // bytes per lane per row
    static constexpr int EPL = BPL / (int)sizeof(KT);               // elements per lane
    static constexpr int LPP = HD * (int)sizeof(KT) / BPL;          // lanes per row
    static constexpr int PPW = 32 / LPP;                            // rows per warp per step
    static constexpr int NV = BPL / 16;                             // 16-byte loads per lane per row
    static constexpr int U = (BPL == 16 && G < 8) ? 8 : 4;          // row groups in flight
    // G <= LPP: the G partial dots of a row are reduce-scattered over the
    // lane group (lane sub ends with head sub / (LPP / G)); otherwise every
    // head is all-reduced.
    static constexpr bool SCATTER = G > 1 && G <= LPP;
    static constexpr int GSPAN = SCATTER ? LPP / G : LPP;           // lanes sharing one head's sum
    static_assert(LPP >= 1 && LPP <= 32 && (LPP & (LPP - 1)) == 0, "head_dim / lane mapping");
    static_assert(EPL % 2 == 0, "pairs of elements");
};

// 16-byte chunks of fp16 or f32 elements -> pairs of f32
template <typename KT, int EPL>
__device__ __forceinline__ void cvt_pairs(const uint4* raw, float2* out) {
    if constexpr (sizeof(KT) == 2) {
#pragma unroll
        for (int v = 0; v < EPL / 8; v++) {
            const __half2* h2 = reinterpret_cast<const __half2*>(&raw[v]);
#pragma unroll
            for (int i = 0; i < 4; i++) out[v * 4 + i] = __half22float2(h2[i]);
        }
    } else {
#pragma unroll
        for (int v = 0; v < EPL / 4; v++) {
            const float2* f = reinterpret_cast<const float2*>(&raw[v]);
            out[v * 2] = f[0];
            out[v * 2 + 1] = f[1];
        }
    }
}

// Reduce-scatter of v[0..C) over the lanes of a group (offsets OFF, OFF/2,
// ..): at each level a lane keeps the half of its values selected by its
// lane bit and adds the partner's copy of that half; once one value is left
// the remaining levels all-reduce it.
template <int C, int OFF>
struct Scatter {
    static __device__ __forceinline__ void run(float* v, int sub) {
        if constexpr (C > 1) {
            constexpr int H = C / 2;
            const bool up = (sub & OFF) != 0;
#pragma unroll
            for (int i = 0; i < H; i++) {
                const float send = up ? v[i] : v[H + i];
                const float keep = up ? v[H + i] : v[i];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, OFF);
            }
            Scatter<H, OFF / 2>::run(v, sub);
        } else if constexpr (OFF > 0) {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], OFF);
            Scatter<1, OFF / 2>::run(v, sub);
        }
    }
};

// Scores of positions [p0, p1) written to S[(p - sbase) * G + g]; mx gets
// the maximum of the scores this lane wrote (head g_own of the lane when
// scattering, every head otherwise).
template <typename KT, int G, int HD>
__device__ __forceinline__ void da_scores(const KT* __restrict__ kbase, const float2 (&qr)[G][DA<KT, G, HD>::EPL / 2],
                                          int p0, int p1, float scale, float* S, int sbase, float (&mx)[G]) {
    using C = DA<KT, G, HD>;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int slot = lane / C::LPP, sub = lane % C::LPP;
    const int g_own = sub / C::GSPAN;
    const bool writer = (sub % C::GSPAN) == 0;
    constexpr int STEP = C::U * C::PPW;
    for (int c0 = p0 + warp * STEP; c0 < p1; c0 += DA_WARPS * STEP) {
        uint4 raw[C::U][C::NV];
#pragma unroll
        for (int u = 0; u < C::U; u++) {
            int p = c0 + u * C::PPW + slot;
            const uint4* src = reinterpret_cast<const uint4*>(kbase + (size_t)p * HD + sub * C::EPL);
#pragma unroll
            for (int v = 0; v < C::NV; v++) raw[u][v] = (p < p1) ? __ldg(src + v) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < C::U; u++) {
            float2 k[C::EPL / 2];
            cvt_pairs<KT, C::EPL>(raw[u], k);
            float acc[G];
#pragma unroll
            for (int g = 0; g < G; g++) {
                float2 a2 = make_float2(0.0f, 0.0f);
#pragma unroll
                for (int e = 0; e < C::EPL / 2; e++) a2 = __ffma2_rn(qr[g][e], k[e], a2);
                acc[g] = a2.x + a2.y;
            }
            const int p = c0 + u * C::PPW + slot;
            if constexpr (C::SCATTER) {
                Scatter<G, C::LPP / 2>::run(acc, sub);
                if (writer && p < p1) {
                    float sc = __fmul_rn(acc[0], scale);
                    S[(size_t)(p - sbase) * G + g_own] = sc;
                    mx[0] = fmaxf(mx[0], sc);
                }
            } else {
#pragma unroll
                for (int g = 0; g < G; g++) Scatter<1, C::LPP / 2>::run(&acc[g], sub);
                if (sub == 0 && p < p1) {
#pragma unroll
                    for (int g = 0; g < G; g++) {
                        float sc = __fmul_rn(acc[g], scale);
                        S[(size_t)(p - sbase) * G + g] = sc;
                        mx[g] = fmaxf(mx[g], sc);
                    }
                }
            }
        }
    }
}

// The G weights of row p: W[(p - wbase) * G .. + G)
template <int G>
__device__ __forceinline__ void load_w(const float* W, int idx, float (&w)[G]) {
    if constexpr (G % 4 == 0) {
#pragma unroll
        for (int i = 0; i < G / 4; i++) {
            float4 f = reinterpret_cast<const float4*>(W + (size_t)idx * G)[i];
            w[4 * i] = f.x; w[4 * i + 1] = f.y; w[4 * i + 2] = f.z; w[4 * i + 3] = f.w;
        }
    } else if constexpr (G == 2) {
        float2 f = reinterpret_cast<const float2*>(W)[idx];
        w[0] = f.x; w[1] = f.y;
    } else {
        w[0] = W[idx];
    }
}

// o[g][e] += sum over positions [p0, p1) of W[(p - wbase) * G + g] * V[p][d0 + e]
// for this lane's slot and slice (not yet reduced across slots or warps).
template <typename KT, int G, int HD>
__device__ __forceinline__ void da_pv(const KT* __restrict__ vbase, const float* W, int wbase, int p0, int p1,
                                      float2 (&o)[G][DA<KT, G, HD>::EPL / 2]) {
    using C = DA<KT, G, HD>;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int slot = lane / C::LPP, sub = lane % C::LPP;
    constexpr int STEP = C::U * C::PPW;
    for (int c0 = p0 + warp * STEP; c0 < p1; c0 += DA_WARPS * STEP) {
        uint4 raw[C::U][C::NV];
#pragma unroll
        for (int u = 0; u < C::U; u++) {
            int p = c0 + u * C::PPW + slot;
            const uint4* src = reinterpret_cast<const uint4*>(vbase + (size_t)p * HD + sub * C::EPL);
#pragma unroll
            for (int v = 0; v < C::NV; v++) raw[u][v] = (p < p1) ? __ldg(src + v) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < C::U; u++) {
            int p = c0 + u * C::PPW + slot;
            if (p >= p1) continue;
            float2 v2[C::EPL / 2];
            cvt_pairs<KT, C::EPL>(raw[u], v2);
            float w[G];
            load_w<G>(W, p - wbase, w);
#pragma unroll
            for (int g = 0; g < G; g++) {
                const float2 w2 = make_float2(w[g], w[g]);
#pragma unroll
                for (int e = 0; e < C::EPL / 2; e++) o[g][e] = __ffma2_rn(w2, v2[e], o[g][e]);
            }
        }
    }
}

// ---- Staged variants (the whole-context kernel): each lane copies its own
// 16-byte chunks of the next row groups into a per-warp shared-memory ring
// with cp.async (no registers held while the copies are in flight), so two
// stages of U row groups are in flight per warp instead of one.  A lane only
// reads back what it copied itself, so its own cp.async.wait_group is the
// only synchronisation.
constexpr int DA_NS = 2;  // stages of the per-warp ring

__device__ __forceinline__ void cp_async16(void* dst, const void* src, int bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// uint4 slots of one warp's ring
template <typename KT, int G, int HD>
__host__ __device__ constexpr int da_ring_u4() { return DA_NS * DA<KT, G, HD>::U * DA<KT, G, HD>::NV * 32; }

// Copies (zero-filled past p1) the row groups of the stage starting at c0
// into ring slot `slot`, as one commit group.
template <typename KT, int G, int HD>
__device__ __forceinline__ void da_stage(const KT* __restrict__ base, int c0, int p1, uint4* ring, int slot) {
    using C = DA<KT, G, HD>;
    const int lane = threadIdx.x & 31;
    const int sl = lane / C::LPP, sub = lane % C::LPP;
#pragma unroll
    for (int u = 0; u < C::U; u++) {
        const int p = c0 + u * C::PPW + sl;
        const bool in = p < p1;
        const uint4* src = reinterpret_cast<const uint4*>(base + (size_t)(in ? p : 0) * HD + sub * C::EPL);
#pragma unroll
        for (int v = 0; v < C::NV; v++) cp_async16(ring + ((slot * C::U + u) * C::NV + v) * 32 + lane, src + v, in ? 16 : 0);
    }
    cp_async_commit();
}

template <typename KT, int G, int HD>
__device__ __forceinline__ void da_unstage(const uint4* ring, int slot, uint4 (&raw)[DA<KT, G, HD>::U][DA<KT, G, HD>::NV]) {
    using C = DA<KT, G, HD>;
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int u = 0; u < C::U; u++)
#pragma unroll
        for (int v = 0; v < C::NV; v++) raw[u][v] = ring[((slot * C::U + u) * C::NV + v) * 32 + lane];
}

// da_scores through the ring (ring: this CTA's DA_WARPS rings)
template <typename KT, int G, int HD>
__device__ __forceinline__ void da_scores_staged(const KT* __restrict__ kbase, const float2 (&qr)[G][DA<KT, G, HD>::EPL / 2],
                                                 int p0, int p1, float scale, float* S, int sbase, float (&mx)[G],
                                                 uint4* ring_all) {
    using C = DA<KT, G, HD>;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int slot = lane / C::LPP, sub = lane % C::LPP;
    const int g_own = sub / C::GSPAN;
    const bool writer = (sub % C::GSPAN) == 0;
    constexpr int STEP = C::U * C::PPW;
    constexpr int WSTEP = DA_WARPS * STEP;
    uint4* ring = ring_all + warp * da_ring_u4<KT, G, HD>();
    int c0 = p0 + warp * STEP;
    da_stage<KT, G, HD>(kbase, c0, p1, ring, 0);
    da_stage<KT, G, HD>(kbase, c0 + WSTEP, p1, ring, 1);
    for (int it = 0; c0 < p1; it++, c0 += WSTEP) {
        uint4 raw[C::U][C::NV];
        cp_async_wait<1>();  // this stage landed (the next may still be in flight)
        da_unstage<KT, G, HD>(ring, it & 1, raw);
#pragma unroll
        for (int u = 0; u < C::U; u++) {
            float2 k[C::EPL / 2];
            cvt_pairs<KT, C::EPL>(raw[u], k);
            float acc[G];
#pragma unroll
            for (int g = 0; g < G; g++) {
                float2 a2 = make_float2(0.0f, 0.0f);
#pragma unroll
                for (int e = 0; e < C::EPL / 2; e++) a2 = __ffma2_rn(qr[g][e], k[e], a2);
                acc[g] = a2.x + a2.y;
            }
            const int p = c0 + u * C::PPW + slot;
            if constexpr (C::SCATTER) {
                Scatter<G, C::LPP / 2>::run(acc, sub);
                if (writer && p < p1) {
                    float sc = __fmul_rn(acc[0], scale);
                    S[(size_t)(p - sbase) * G + g_own] = sc;
                    mx[0] = fmaxf(mx[0], sc);
                }
            } else {
#pragma unroll
                for (int g = 0; g < G; g++) Scatter<1, C::LPP / 2>::run(&acc[g], sub);
                if (sub == 0 && p < p1) {
#pragma unroll
                    for (int g = 0; g < G; g++) {
                        float sc = __fmul_rn(acc[g], scale);
                        S[(size_t)(p - sbase) * G + g] = sc;
                        mx[g] = fmaxf(mx[g], sc);
                    }
                }
            }
        }
        // the slot's data is in registers and used: refill it two stages ahead
        da_stage<KT, G, HD>(kbase, c0 + 2 * WSTEP, p1, ring, it & 1);
    }
    cp_async_wait<0>();
}

// da_pv through the ring
template <typename KT, int G, int HD>
__device__ __forceinline__ void da_pv_staged(const KT* __restrict__ vbase, const float* W, int wbase, int p0, int p1,
                                             float2 (&o)[G][DA<KT, G, HD>::EPL / 2], uint4* ring_all) {
    using C = DA<KT, G, HD>;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int slot = lane / C::LPP;
    constexpr int STEP = C::U * C::PPW;
    constexpr int WSTEP = DA_WARPS * STEP;
    uint4* ring = ring_all + warp * da_ring_u4<KT, G, HD>();
    int c0 = p0 + warp * STEP;
    da_stage<KT, G, HD>(vbase, c0, p1, ring, 0);
    da_stage<KT, G, HD>(vbase, c0 + WSTEP, p1, ring, 1);
    for (int it = 0; c0 < p1; it++, c0 += WSTEP) {
        uint4 raw[C::U][C::NV];
        cp_async_wait<1>();
        da_unstage<KT, G, HD>(ring, it & 1, raw);
#pragma unroll
        for (int u = 0; u < C::U; u++) {
            int p = c0 + u * C::PPW + slot;
            if (p >= p1) continue;
            float2 v2[C::EPL / 2];
            cvt_pairs<KT, C::EPL>(raw[u], v2);
            float w[G];
            load_w<G>(W, p - wbase, w);
#pragma unroll
            for (int g = 0; g < G; g++) {
                const float2 w2 = make_float2(w[g], w[g]);
#pragma unroll
                for (int e = 0; e < C::EPL / 2; e++) o[g][e] = __ffma2_rn(w2, v2[e], o[g][e]);
            }
        }
        da_stage<KT, G, HD>(vbase, c0 + 2 * WSTEP, p1, ring, it & 1);
    }
    cp_async_wait<0>();
}

// Sum o over the slots of a warp and over the warps; the result for head g,
// feature d lands in red[DA_WARPS * G * HD + g * HD + d] (red holds
// (DA_WARPS + 1) * G * HD floats).
template <typename KT, int G, int HD>
__device__ __forceinline__ void da_reduce_o(float2 (&o)[G][DA<KT, G, HD>::EPL / 2], float* red) {
    using C = DA<KT, G, HD>;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int sub = lane % C::LPP;
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int e = 0; e < C::EPL / 2; e++)
#pragma unroll
            for (int off = C::LPP; off < 32; off <<= 1) {
                o[g][e].x += __shfl_xor_sync(0xffffffffu, o[g][e].x, off);
                o[g][e].y += __shfl_xor_sync(0xffffffffu, o[g][e].y, off);
            }
    __syncthreads();
    if (lane < C::LPP) {
#pragma unroll
        for (int g = 0; g < G; g++)
#pragma unroll
            for (int e = 0; e < C::EPL / 2; e++)
                reinterpret_cast<float2*>(red + ((size_t)warp * G + g) * HD + sub * C::EPL)[e] = o[g][e];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < G * HD; i += DA_THREADS) {
        float t = 0.0f;
#pragma unroll
        for (int w = 0; w < DA_WARPS; w++) t += red[(size_t)w * G * HD + i];
        red[(size_t)DA_WARPS * G * HD + i] = t;
    }
    __syncthreads();
}

template <typename KT, int G, int HD>
__device__ __forceinline__ void da_load_q(const DecAttnParams& P, int row, int kvh,
                                          float2 (&qr)[G][DA<KT, G, HD>::EPL / 2]) {
    using C = DA<KT, G, HD>;
    const int sub = (threadIdx.x & 31) % C::LPP;
#pragma unroll
    for (int g = 0; g < G; g++) {
        const float2* q2 =
            reinterpret_cast<const float2*>(P.q + (size_t)row * P.ldq + (size_t)(kvh * G + g) * HD + sub * C::EPL);
#pragma unroll
        for (int e = 0; e < C::EPL / 2; e++) qr[g][e] = q2[e];
    }
}

__device__ __forceinline__ void da_write_out(const DecAttnParams& P, int row, int h, int d, float v) {
    P.out[(size_t)row * P.ldo + (size_t)h * P.hd + d] = v;
    if (P.out16) store_x16(P.out16 + (size_t)row * 2 * P.nh * P.hd, P.nh * P.hd, h * P.hd + d, v);
}

// Block maxima per head of the lanes' maxima (one head per lane when the
// scores were scattered).
template <typename KT, int G, int HD>
__device__ __forceinline__ void da_head_max(const float (&mx)[G], float (&gmax)[G], float* redv) {
    using C = DA<KT, G, HD>;
    if constexpr (C::SCATTER) {
        const int g_own = ((threadIdx.x & 31) % C::LPP) / C::GSPAN;
#pragma unroll
        for (int g = 0; g < G; g++) gmax[g] = block_max(g_own == g ? mx[0] : -INFINITY, redv);
    } else {
#pragma unroll
        for (int g = 0; g < G; g++) gmax[g] = block_max(mx[g], redv);
    }
}

// Floats before the reduction buffer that follows n score floats (kept a
// multiple of 4 so the buffer's vector accesses stay aligned).
__host__ __device__ __forceinline__ size_t red_offset(int n) { return ((size_t)n + 3) & ~(size_t)3; }

// Whole context in one CTA per (sequence, KV head): scores kept in shared
// memory, then weights, then P.V; K and V are each read once.
// ST: K and V stream through per-warp cp.async rings that share the
// reduction buffer's shared memory.
template <typename KT, int G, int HD, bool ST>
__global__ void __launch_bounds__(DA_THREADS, 2) k_dattn_fused(DecAttnParams P) {
    pdl_trigger();
    using C = DA<KT, G, HD>;
    extern __shared__ float smem[];
    __shared__ float redv[32];
    const int row = blockIdx.x, kvh = blockIdx.y;
    const int seq = P.seqs[row];
    const int n = min(P.pos[seq], P.max_pos);
    if (n <= 1) {
        for (int i = threadIdx.x; i < G * HD; i += DA_THREADS)
            da_write_out(P, row, kvh * G + i / HD, i % HD, P.vself[(size_t)row * P.ldself + (size_t)kvh * HD + i % HD]);
        return;
    }
    float* S = smem;                                // [max_pos][G]
    float* red = smem + red_offset(G * P.max_pos);  // [(DA_WARPS + 1) * G * HD], 16-byte aligned
    const size_t off = (size_t)seq * P.seq_stride + (size_t)kvh * P.head_stride;
    const KT* kbase = reinterpret_cast<const KT*>(P.kc) + off;
    const KT* vbase = reinterpret_cast<const KT*>(P.vc) + off;
    float2 qr[G][C::EPL / 2];
    da_load_q<KT, G, HD>(P, row, kvh, qr);
    float mx[G];
#pragma unroll
    for (int g = 0; g < G; g++) mx[g] = -INFINITY;
    if constexpr (ST)
        da_scores_staged<KT, G, HD>(kbase, qr, 0, n, P.scale, S, 0, mx, reinterpret_cast<uint4*>(red));
    else
        da_scores<KT, G, HD>(kbase, qr, 0, n, P.scale, S, 0, mx);
    float gmax[G];
    da_head_max<KT, G, HD>(mx, gmax, redv);  // also orders the S writes
    const int n8 = n - (n % 8);
    float lsum[G];
#pragma unroll
    for (int g = 0; g < G; g++) lsum[g] = 0.0f;
    for (int p = threadIdx.x; p < n; p += DA_THREADS) {
#pragma unroll
        for (int g = 0; g < G; g++) {
            float e = softmax_weight(S[(size_t)p * G + g], gmax[g], p, n8);
            S[(size_t)p * G + g] = e;
            lsum[g] += e;
        }
    }
    float total[G];
#pragma unroll
    for (int g = 0; g < G; g++) total[g] = block_sum(lsum[g], redv);  // also orders the weight writes
    float2 o[G][C::EPL / 2];
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int e = 0; e < C::EPL / 2; e++) o[g][e] = make_float2(0.0f, 0.0f);
    if constexpr (ST)
        da_pv_staged<KT, G, HD>(vbase, S, 0, 0, n, o, reinterpret_cast<uint4*>(red));
    else
        da_pv<KT, G, HD>(vbase, S, 0, 0, n, o);
    da_reduce_o<KT, G, HD>(o, red);  // its first barrier follows every warp's last ring read
    const float* fin = red + (size_t)DA_WARPS * G * HD;
    for (int i = threadIdx.x; i < G * HD; i += DA_THREADS) {
        int g = i / HD;
        da_write_out(P, row, kvh * G + g, i % HD, __fdiv_rn(fin[i], total[g]));
    }
}

// ---- Tensor-core variant of the whole-context kernel for fp16 caches with
// G <= 4 query heads per KV head (mma.sync m16n8k16, f16 in, f32 accumulate).
// Scores: A = 16 cached K rows x 16 features (exact fp16), B = 16 features x 8
// columns holding each query head rounded to fp16 (columns g) and its rounding
// remainder (columns 4 + g); hi and lo are accumulated separately in f32 and
// then added, which recovers the f32 query to ~2^-22 relative.  Weighted V:
// A = the weights split the same way (rows g: fp16 parts, rows 4 + g: the
// remainders, rows 8-15 zero) x 16 positions, B = 16 positions x 8 features of
// V (exact fp16).  K and V tiles of 16 rows stream through per-warp cp.async
// rings (rows of HD/8 16-byte chunks, chunk c of row r stored at c ^ (r & 7)
// so the ldmatrix reads are conflict-free); each warp takes every eighth tile.
namespace {
constexpr int DM_TILE = 16;  // positions per tile

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"((uint32_t)__cvta_generic_to_shared(p)));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"((uint32_t)__cvta_generic_to_shared(p)));
}

// fp16 pair (lo half = a) of the hi part (lo == false) or the rounding
// remainder (lo == true) of two f32 values
__device__ __forceinline__ uint32_t split_pair(float a, float b, bool lo) {
    const __half ah = __float2half_rn(a), bh = __float2half_rn(b);
    __half2 h = lo ? __halves2half2(__float2half_rn(a - __half2float(ah)), __float2half_rn(b - __half2float(bh)))
                   : __halves2half2(ah, bh);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Copies tile `tile` (rows [16 tile, 16 tile + 16), zero past n) into ring slot
// `slot` (16 B units), one commit group.
template <int HD>
__device__ __forceinline__ void dm_stage(const __half* __restrict__ base, int tile, int n, uint4* slot_base) {
    constexpr int CPR = HD / 8;  // 16-byte chunks per row
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int j = 0; j < DM_TILE * CPR / 32; j++) {
        const int i = lane + 32 * j, r = i / CPR, c = i % CPR;
        const int p = tile * DM_TILE + r;
        const bool in = p < n;
        cp_async16(slot_base + r * CPR + (c ^ (r & 7)), base + (size_t)(in ? p : 0) * HD + c * 8, in ? 16 : 0);
    }
    cp_async_commit();
}
}  // namespace

// NW warps per CTA: 8 (two CTAs per SM) when the pairs fill the GPU, 16 (one
// CTA per SM, twice the copies in flight) when there are only about as many
// pairs as SMs.
template <int G, int HD, int NW>
__global__ void __launch_bounds__(NW * 32, 16 / NW) k_dattn_mma(DecAttnParams P) {
    constexpr int NS = 2;  // ring stages per warp
    static_assert(G == 1 || G == 2 || G == 4, "hi and lo columns of G heads in 8");
    static_assert(HD == 64 || HD == 128, "feature tiles");
    constexpr int CPR = HD / 8;
    constexpr int SLOT = DM_TILE * CPR;  // uint4 per ring slot
    pdl_trigger();
    extern __shared__ float smem[];
    __shared__ float redv[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int t = lane & 3, q4 = lane >> 2;
    const int row = blockIdx.x, kvh = blockIdx.y;
    const int seq = P.seqs[row];
    const int n = min(P.pos[seq], P.max_pos);
    if (n <= 1) {
        for (int i = threadIdx.x; i < G * HD; i += NW * 32)
            da_write_out(P, row, kvh * G + i / HD, i % HD, P.vself[(size_t)row * P.ldself + (size_t)kvh * HD + i % HD]);
        return;
    }
    float* S = smem;                                // [max_pos][G]
    float* red = smem + red_offset(G * P.max_pos);  // rings, then the reduction buffer
    uint4* ring = reinterpret_cast<uint4*>(red) + (size_t)warp * NS * SLOT;
    const size_t off = (size_t)seq * P.seq_stride + (size_t)kvh * P.head_stride;
    const __half* kbase = reinterpret_cast<const __half*>(P.kc) + off;
    const __half* vbase = reinterpret_cast<const __half*>(P.vc) + off;
    const int ntiles = (n + DM_TILE - 1) / DM_TILE;

    // ---- query fragments: column q4 of B = head q4 % 4, hi (q4 < 4) or lo
    uint32_t qf[HD / 16][2];
    {
        const int g = q4 & 3;
        const bool lo = q4 >= 4, valid = g < G;
        const float* qrow = P.q + (size_t)row * P.ldq + (size_t)(kvh * G + (valid ? g : 0)) * HD;
#pragma unroll
        for (int ks = 0; ks < HD / 16; ks++)
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int k = ks * 16 + 2 * t + 8 * h;
                const float a = valid ? qrow[k] : 0.0f, b = valid ? qrow[k + 1] : 0.0f;
                qf[ks][h] = split_pair(a, b, lo);
            }
    }

    // ---- scores
    float mx0 = -INFINITY, mx1 = -INFINITY;  // heads 2t, 2t + 1 (lanes t < 2)
#pragma unroll
    for (int i = 0; i < NS; i++) dm_stage<HD>(kbase, warp + i * NW, n, ring + i * SLOT);
    for (int tile = warp, it = 0; tile < ntiles; tile += NW, it++) {
        cp_async_wait<NS - 1>();
        __syncwarp();  // every lane's copies of this tile landed
        const uint4* sl = ring + (it % NS) * SLOT;
        float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int ks = 0; ks < HD / 16; ks++) {
            const int mi = lane >> 3, r = (lane & 7) + 8 * (mi & 1);
            uint32_t a[4];
            ldsm_x4(a, sl + r * CPR + ((2 * ks + (mi >> 1)) ^ (r & 7)));
            mma16816(d, a, qf[ks][0], qf[ks][1]);
        }
        // columns 2t, 2t + 1: hi parts (t < 2) and lo parts (t >= 2) of heads 2(t & 1), 2(t & 1) + 1
        float e[4];
#pragma unroll
        for (int i = 0; i < 4; i++) e[i] = __shfl_xor_sync(0xffffffffu, d[i], 2);
        if (t < 2) {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int g = 2 * t + (i & 1);
                const int p = tile * DM_TILE + q4 + 8 * (i >> 1);
                if (g < G && p < n) {
                    const float sc = __fmul_rn(d[i] + e[i], P.scale);
                    S[(size_t)p * G + g] = sc;
                    if (i & 1) mx1 = fmaxf(mx1, sc);
                    else mx0 = fmaxf(mx0, sc);
                }
            }
        }
        __syncwarp();  // the slot is read: refill it NS tiles ahead
        dm_stage<HD>(kbase, tile + NS * NW, n, ring + (it % NS) * SLOT);
    }
    cp_async_wait<0>();
    float gmax[G];
#pragma unroll
    for (int g = 0; g < G; g++) gmax[g] = block_max(t == (g >> 1) ? ((g & 1) ? mx1 : mx0) : -INFINITY, redv);

    // The weights (the reference's polynomial softmax over the global
    // maximum) are formed from the scores tile by tile in the weighted-V
    // pass, which also sums them.
    const int n8 = n - (n % 8);

    // ---- weighted V: rows q4 of A = head q4 % 4, hi (q4 < 4) or lo
    float acc[HD / 8][4];
#pragma unroll
    for (int j = 0; j < HD / 8; j++) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
    const int ga = q4 & 3;
    const bool alo = q4 >= 4, avalid = ga < G;
    float gm = gmax[0];  // global maximum of head ga
#pragma unroll
    for (int g = 1; g < G; g++)
        if (ga == g) gm = gmax[g];
    float lsum = 0.0f;  // lanes 0-15 (the hi rows): this lane's share of head ga's weight sum
#pragma unroll
    for (int i = 0; i < NS; i++) dm_stage<HD>(vbase, warp + i * NW, n, ring + i * SLOT);
    for (int tile = warp, it = 0; tile < ntiles; tile += NW, it++) {
        const int p0 = tile * DM_TILE + 2 * t;
        cp_async_wait<NS - 1>();
        __syncwarp();
        const uint4* sl = ring + (it % NS) * SLOT;
        float w[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int p = p0 + (i & 1) + 8 * (i >> 1);
            w[i] = (avalid && p < n) ? softmax_weight(S[(size_t)p * G + ga], gm, p, n8) : 0.0f;
            if (!alo) lsum += w[i];
        }
        const uint32_t a[4] = {split_pair(w[0], w[1], alo), 0u, split_pair(w[2], w[3], alo), 0u};
#pragma unroll
        for (int j = 0; j < HD / 16; j++) {
            const int mi = lane >> 3, r = (lane & 7) + 8 * (mi & 1);
            uint32_t b[4];
            ldsm_x4_t(b, sl + r * CPR + ((2 * j + (mi >> 1)) ^ (r & 7)));
            mma16816(acc[2 * j], a, b[0], b[1]);
            mma16816(acc[2 * j + 1], a, b[2], b[3]);
        }
        __syncwarp();
        dm_stage<HD>(vbase, tile + NS * NW, n, ring + (it % NS) * SLOT);
    }
    cp_async_wait<0>();
    // rows q4 and q4 + 4 (lanes l and l + 16) are the hi and lo sums of head q4
#pragma unroll
    for (int j = 0; j < HD / 8; j++) {
        acc[j][0] += __shfl_down_sync(0xffffffffu, acc[j][0], 16);
        acc[j][1] += __shfl_down_sync(0xffffffffu, acc[j][1], 16);
    }
    float total[G];
#pragma unroll
    for (int g = 0; g < G; g++) total[g] = block_sum(lane < 16 && q4 == g ? lsum : 0.0f, redv);
    __syncthreads();  // every warp is done with its ring: the buffer becomes the reduction area
    if (lane < 16 && q4 < G) {
#pragma unroll
        for (int j = 0; j < HD / 8; j++)
            *reinterpret_cast<float2*>(red + ((size_t)warp * G + q4) * HD + 8 * j + 2 * t) =
                make_float2(acc[j][0], acc[j][1]);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < G * HD; i += NW * 32) {
        float o = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; w++) o += red[(size_t)w * G * HD + i];
        da_write_out(P, row, kvh * G + i / HD, i % HD, __fdiv_rn(o, total[i / HD]));
    }
}

// ---- Cluster split.  When the batch has too few (sequence, KV head) pairs
// to fill the GPU (tensor-parallel shards), the NCL CTAs of a thread-block
// cluster share one pair: CTA c scores positions [c len, (c+1) len), the CTAs
// exchange their per-head maxima through distributed shared memory (every CTA
// then holds the same global maxima), form their weights and partial P.V, and
// after a second exchange CTA c finishes the output features
// [c G HD / NCL, (c+1) G HD / NCL) by adding the partials in rank order.
__device__ __forceinline__ void cl_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cl_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ float cl_ld(const float* local, int rank) {
    uint32_t a = (uint32_t)__cvta_generic_to_shared(local), remote;
    float v;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(a), "r"(rank));
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
    return v;
}

template <typename KT, int G, int HD>
__global__ void __launch_bounds__(DA_THREADS, 2) k_dattn_cluster(DecAttnParams P) {
    pdl_trigger();
    using C = DA<KT, G, HD>;
    extern __shared__ float smem[];
    __shared__ float redv[32];
    __shared__ float xch[2 * DA_MAXG];  // this CTA's per-head maxima, then its weight sums
    const int row = blockIdx.x, kvh = blockIdx.y;
    const int ncl = (int)gridDim.z;
    const int rank = (int)cl_rank();
    const int seq = P.seqs[row];
    const int n = min(P.pos[seq], P.max_pos);
    if (n <= 1) {  // uniform over the cluster: no exchange
        if (rank == 0)
            for (int i = threadIdx.x; i < G * HD; i += DA_THREADS)
                da_write_out(P, row, kvh * G + i / HD, i % HD,
                             P.vself[(size_t)row * P.ldself + (size_t)kvh * HD + i % HD]);
        return;
    }
    const int len = (n + ncl - 1) / ncl;
    const int p0 = min(n, rank * len), p1 = min(n, p0 + len);
    float* S = smem;                              // [chunk][G] (chunk >= len)
    float* red = smem + red_offset(G * P.chunk);  // [(DA_WARPS + 1) * G * HD]
    const size_t off = (size_t)seq * P.seq_stride + (size_t)kvh * P.head_stride;
    const KT* kbase = reinterpret_cast<const KT*>(P.kc) + off;
    const KT* vbase = reinterpret_cast<const KT*>(P.vc) + off;
    float2 qr[G][C::EPL / 2];
    da_load_q<KT, G, HD>(P, row, kvh, qr);
    float mx[G];
#pragma unroll
    for (int g = 0; g < G; g++) mx[g] = -INFINITY;
    da_scores<KT, G, HD>(kbase, qr, p0, p1, P.scale, S, p0, mx);
    float lmax[G];
    da_head_max<KT, G, HD>(mx, lmax, redv);  // also orders the S writes
    if (threadIdx.x < G) {
#pragma unroll
        for (int g = 0; g < G; g++)
            if (threadIdx.x == g) xch[g] = lmax[g];
    }
    cl_sync();
    float gmax[G];
#pragma unroll
    for (int g = 0; g < G; g++) {
        float m = -INFINITY;
        for (int c = 0; c < ncl; c++) m = fmaxf(m, cl_ld(&xch[g], c));
        gmax[g] = m;
    }
    const int n8 = n - (n % 8);
    float lsum[G];
#pragma unroll
    for (int g = 0; g < G; g++) lsum[g] = 0.0f;
    for (int p = p0 + threadIdx.x; p < p1; p += DA_THREADS) {
#pragma unroll
        for (int g = 0; g < G; g++) {
            float e = softmax_weight(S[(size_t)(p - p0) * G + g], gmax[g], p, n8);
            S[(size_t)(p - p0) * G + g] = e;
            lsum[g] += e;
        }
    }
    float tsum[G];
#pragma unroll
    for (int g = 0; g < G; g++) tsum[g] = block_sum(lsum[g], redv);  // also orders the weight writes
    float2 o[G][C::EPL / 2];
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int e = 0; e < C::EPL / 2; e++) o[g][e] = make_float2(0.0f, 0.0f);
    da_pv<KT, G, HD>(vbase, S, p0, p0, p1, o);
    da_reduce_o<KT, G, HD>(o, red);  // this CTA's partial P.V in red[DA_WARPS * G * HD ..]
    if (threadIdx.x < G) {
#pragma unroll
        for (int g = 0; g < G; g++)
            if (threadIdx.x == g) xch[DA_MAXG + g] = tsum[g];
    }
    cl_sync();  // partials and sums of every CTA are visible
    const float* fin = red + (size_t)DA_WARPS * G * HD;
    const int f0 = (G * HD) * rank / ncl, f1 = (G * HD) * (rank + 1) / ncl;
    for (int i = f0 + (int)threadIdx.x; i < f1; i += DA_THREADS) {
        const int g = i / HD;
        float num = 0.0f, den = 0.0f;
        for (int c = 0; c < ncl; c++) {
            num += cl_ld(&fin[i], c);
            den += cl_ld(&xch[DA_MAXG + g], c);
        }
        da_write_out(P, row, kvh * G + g, i % HD, __fdiv_rn(num, den));
    }
    cl_sync();  // peers finished reading this CTA's shared memory
}

// Split path, pass 1: scores of one split to global S, split maximum.
template <typename KT, int G, int HD>
__global__ void __launch_bounds__(DA_THREADS, 2) k_dattn_scores(DecAttnParams P) {
    using C = DA<KT, G, HD>;
    __shared__ float redv[32];
    const int row = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
    const int seq = P.seqs[row];
    const int n = min(P.pos[seq], P.max_pos);
    const int p0 = split * P.chunk, p1 = min(n, p0 + P.chunk);
    if (n <= 1) return;
    const KT* kbase = reinterpret_cast<const KT*>(P.kc) + (size_t)seq * P.seq_stride + (size_t)kvh * P.head_stride;
    float2 qr[G][C::EPL / 2];
    da_load_q<KT, G, HD>(P, row, kvh, qr);
    float mx[G];
#pragma unroll
    for (int g = 0; g < G; g++) mx[g] = -INFINITY;
    float* S = P.S + ((size_t)row * P.nh + kvh * G) * P.max_pos;  // [max_pos][G] of this (row, kv head)
    da_scores<KT, G, HD>(kbase, qr, p0, p1, P.scale, S, 0, mx);
    float gmax[G];
    da_head_max<KT, G, HD>(mx, gmax, redv);
    if (threadIdx.x < G) {
#pragma unroll
        for (int g = 0; g < G; g++)
            if (threadIdx.x == g) P.smax[((size_t)row * P.nh + kvh * G + g) * P.nsplit + split] = gmax[g];
    }
}

// Split path, pass 2: weights with the global maximum, partial P.V of the split.
template <typename KT, int G, int HD>
__global__ void __launch_bounds__(DA_THREADS, 2) k_dattn_pv(DecAttnParams P) {
    using C = DA<KT, G, HD>;
    extern __shared__ float smem[];  // [chunk][G] weights, then the reduction buffer
    __shared__ float redv[32];
    __shared__ float gmax[DA_MAXG];
    const int row = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
    const int seq = P.seqs[row];
    const int n = min(P.pos[seq], P.max_pos);
    if (n <= 1) {
        if (split == 0)
            for (int i = threadIdx.x; i < G * HD; i += DA_THREADS)
                da_write_out(P, row, kvh * G + i / HD, i % HD,
                             P.vself[(size_t)row * P.ldself + (size_t)kvh * HD + i % HD]);
        return;
    }
    const int nsplit_eff = (n + P.chunk - 1) / P.chunk;
    if (split >= nsplit_eff) return;
    const int p0 = split * P.chunk, p1 = min(n, p0 + P.chunk), len = p1 - p0;
    if (threadIdx.x < G) {
        float m = -INFINITY;
        for (int s2 = 0; s2 < nsplit_eff; s2++)
            m = fmaxf(m, P.smax[((size_t)row * P.nh + kvh * G + threadIdx.x) * P.nsplit + s2]);
        gmax[threadIdx.x] = m;
    }
    __syncthreads();
    float* W = smem;
    float* red = smem + red_offset(G * P.chunk);
    const int n8 = n - (n % 8);
    const float* Sg = P.S + ((size_t)row * P.nh + kvh * G) * P.max_pos;
    float lsum[G];
#pragma unroll
    for (int g = 0; g < G; g++) lsum[g] = 0.0f;
    for (int i = threadIdx.x; i < len; i += DA_THREADS) {
#pragma unroll
        for (int g = 0; g < G; g++) {
            float e = softmax_weight(Sg[(size_t)(p0 + i) * G + g], gmax[g], p0 + i, n8);
            W[(size_t)i * G + g] = e;
            lsum[g] += e;
        }
    }
    float total[G];
#pragma unroll
    for (int g = 0; g < G; g++) total[g] = block_sum(lsum[g], redv);
    const KT* vbase = reinterpret_cast<const KT*>(P.vc) + (size_t)seq * P.seq_stride + (size_t)kvh * P.head_stride;
    float2 o[G][C::EPL / 2];
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int e = 0; e < C::EPL / 2; e++) o[g][e] = make_float2(0.0f, 0.0f);
    da_pv<KT, G, HD>(vbase, W, p0, p0, p1, o);
    da_reduce_o<KT, G, HD>(o, red);
    const float* fin = red + (size_t)DA_WARPS * G * HD;
    for (int i = threadIdx.x; i < G * HD; i += DA_THREADS) {
        int g = i / HD, d = i % HD;
        size_t hidx = (size_t)row * P.nh + kvh * G + g;
        if (nsplit_eff == 1) {
            da_write_out(P, row, kvh * G + g, d, __fdiv_rn(fin[i], total[g]));
        } else {
            P.opart[(hidx * P.nsplit + split) * HD + d] = fin[i];
            if (d == 0) P.spart[hidx * P.nsplit + split] = total[g];
        }
    }
}

// Split path, pass 3: out = sum of partial P.V / sum of partial weights.
__global__ void k_dattn_combine(DecAttnParams P) {
    pdl_trigger();
    const int row = blockIdx.x, h = blockIdx.y;
    const int seq = P.seqs[row];
    const int n = min(P.pos[seq], P.max_pos);
    if (n <= 1) return;
    const int nsplit_eff = (n + P.chunk - 1) / P.chunk;
    if (nsplit_eff == 1) return;
    size_t hidx = (size_t)row * P.nh + h;
    float total = 0.0f;
    for (int s2 = 0; s2 < nsplit_eff; s2++) total += P.spart[hidx * P.nsplit + s2];
    for (int d = threadIdx.x; d < P.hd; d += blockDim.x) {
        float o = 0.0f;
        for (int s2 = 0; s2 < nsplit_eff; s2++) o += P.opart[(hidx * P.nsplit + s2) * P.hd + d];
        da_write_out(P, row, h, d, __fdiv_rn(o, total));
    }
}

template <typename KT, int G, int HD>
int launch_dattn_ghd(const DecAttnParams& P, int rows, cudaStream_t s) {
    const size_t red_floats = (size_t)(DA_WARPS + 1) * G * HD;
    if (P.cluster > 1) {  // chunk = positions per CTA of the cluster
        HC_CHECK(P.cluster <= 8 && (size_t)P.chunk * P.cluster >= (size_t)P.max_pos, HC_ERR_INVALID,
                 "decode attention: cluster %d x chunk %d does not cover %d positions", P.cluster, P.chunk,
                 P.max_pos);
        size_t smem = (red_offset(G * P.chunk) + red_floats) * sizeof(float);
        HC_CHECK(smem <= 220 * 1024, HC_ERR_UNSUPPORTED, "decode attention: chunk %d too long", P.chunk);
        if (smem > 48 * 1024)
            HC_CUDA(cudaFuncSetAttribute(k_dattn_cluster<KT, G, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem));
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)rows, (unsigned)P.nkv, (unsigned)P.cluster);
        cfg.blockDim = dim3(DA_THREADS);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = (unsigned)P.cluster;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        HC_CUDA(cudaLaunchKernelEx(&cfg, k_dattn_cluster<KT, G, HD>, P));
        hc_count_launch();
        return HC_OK;
    }
    if (P.nsplit == 1) {
        size_t smem = (red_offset(G * P.max_pos) + red_floats) * sizeof(float);
        HC_CHECK(smem <= 220 * 1024, HC_ERR_UNSUPPORTED, "decode attention: context %d too long for one split",
                 P.max_pos);
        if constexpr (sizeof(KT) == 2 && (G == 1 || G == 2 || G == 4) && (HD == 64 || HD == 128)) {
            // tensor-core variant: two ring stages per warp; P.wide: 16 warps,
            // one CTA per SM, else 8 warps, two CTAs per SM
            const int nw = P.wide ? 16 : DA_WARPS;
            const size_t smem_m =
                (red_offset(G * P.max_pos) + std::max<size_t>((size_t)nw * G * HD, (size_t)nw * DM_TILE * HD)) *
                sizeof(float);
            if (P.wide && smem_m <= 220 * 1024) {
                HC_CUDA(cudaFuncSetAttribute(k_dattn_mma<G, HD, 16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem_m));
                k_dattn_mma<G, HD, 16><<<dim3((unsigned)rows, (unsigned)P.nkv), 16 * 32, smem_m, s>>>(P);
                HC_LAUNCH_CHECK();
                return HC_OK;
            }
            if (!P.wide && smem_m <= 112 * 1024) {
                if (smem_m > 48 * 1024)
                    HC_CUDA(cudaFuncSetAttribute(k_dattn_mma<G, HD, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)smem_m));
                k_dattn_mma<G, HD, 8><<<dim3((unsigned)rows, (unsigned)P.nkv), DA_THREADS, smem_m, s>>>(P);
                HC_LAUNCH_CHECK();
                return HC_OK;
            }
        }
        // the cp.async rings when they still leave two CTAs per SM
        const size_t ring_floats = (size_t)DA_WARPS * da_ring_u4<KT, G, HD>() * 4;
        const size_t smem_st = (red_offset(G * P.max_pos) + std::max<size_t>(red_floats, ring_floats)) * sizeof(float);
        if (smem_st <= 112 * 1024) {
            if (smem_st > 48 * 1024)
                HC_CUDA(cudaFuncSetAttribute(k_dattn_fused<KT, G, HD, true>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_st));
            k_dattn_fused<KT, G, HD, true><<<dim3((unsigned)rows, (unsigned)P.nkv), DA_THREADS, smem_st, s>>>(P);
        } else {
            if (smem > 48 * 1024)
                HC_CUDA(cudaFuncSetAttribute(k_dattn_fused<KT, G, HD, false>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            k_dattn_fused<KT, G, HD, false><<<dim3((unsigned)rows, (unsigned)P.nkv), DA_THREADS, smem, s>>>(P);
        }
        HC_LAUNCH_CHECK();
        return HC_OK;
    }
    dim3 grid((unsigned)rows, (unsigned)P.nkv, (unsigned)P.nsplit);
    k_dattn_scores<KT, G, HD><<<grid, DA_THREADS, 0, s>>>(P);
    HC_LAUNCH_CHECK();
    size_t smem2 = (red_offset(G * P.chunk) + red_floats) * sizeof(float);
    if (smem2 > 48 * 1024)
        HC_CUDA(cudaFuncSetAttribute(k_dattn_pv<KT, G, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem2));
    k_dattn_pv<KT, G, HD><<<grid, DA_THREADS, smem2, s>>>(P);
    HC_LAUNCH_CHECK();
    k_dattn_combine<<<dim3((unsigned)rows, (unsigned)P.nh), 128, 0, s>>>(P);
    HC_LAUNCH_CHECK();
    return HC_OK;
}

template <typename KT, int G>
int launch_dattn_g(const DecAttnParams& P, int rows, cudaStream_t s) {
    switch (P.hd) {
        case 16: return launch_dattn_ghd<KT, G, 16>(P, rows, s);
        case 32: return launch_dattn_ghd<KT, G, 32>(P, rows, s);
        case 64: return launch_dattn_ghd<KT, G, 64>(P, rows, s);
        case 128: return launch_dattn_ghd<KT, G, 128>(P, rows, s);
        default:
            hc_set_error("grouped decode attention: unsupported head_dim %d", P.hd);
            return HC_ERR_UNSUPPORTED;
    }
}

template <typename KT>
int launch_dattn_kt(const DecAttnParams& P, int rows, cudaStream_t s) {
    switch (P.nh / P.nkv) {
        case 1: return launch_dattn_g<KT, 1>(P, rows, s);
        case 2: return launch_dattn_g<KT, 2>(P, rows, s);
        case 4: return launch_dattn_g<KT, 4>(P, rows, s);
        case 8: return launch_dattn_g<KT, 8>(P, rows, s);
        default:
            hc_set_error("grouped decode attention: unsupported group size %d", P.nh / P.nkv);
            return HC_ERR_UNSUPPORTED;
    }
}

}  // namespace

bool dattn_wide_ok(int nh, int nkv, int hd, int max_pos, int kv_fp16) {
    const int g = nh / nkv;
    if (!kv_fp16 || !(g == 1 || g == 2 || g == 4) || !(hd == 64 || hd == 128)) return false;
    const size_t smem = (red_offset(g * max_pos) + std::max<size_t>((size_t)16 * g * hd, (size_t)16 * DM_TILE * hd)) *
                        sizeof(float);
    return smem <= 220 * 1024;
}

bool dattn_supported(int nh, int nkv, int hd) {
    int g = nh / nkv;
    return (hd == 16 || hd == 32 || hd == 64 || hd == 128) && (g == 1 || g == 2 || g == 4 || g == 8);
}

int launch_decode_attention(const DecAttnParams& P, int rows, int kv_fp16, cudaStream_t s) {
    if (rows == 0) return HC_OK;
    return kv_fp16 ? launch_dattn_kt<__half>(P, rows, s) : launch_dattn_kt<float>(P, rows, s);
}


// ============================================================ tiled prefill attention
//
// turbo.rs:144-185 for a whole prompt: query t (t >= 2) attends prompt
// positions [0, t); t < 2 takes its own V.  One CTA per (64-query block,
// query head).  S = Q K^T tiles are formed in shared memory with a 4x4
// micro-tile per thread (f32 FMA); pass 1 takes each row's maximum over all
// its keys, pass 2 recomputes the tiles, forms the polynomial / exp weights
// with that maximum and accumulates W V.
namespace {

constexpr int PA_BQ = 64, PA_BK = 64, PA_THREADS = 256, PA_KT_STRIDE = PA_BK + 4;

template <int HD>
__global__ void __launch_bounds__(PA_THREADS) k_pattn(AttnParams P, int T) {
    pdl_trigger();
    extern __shared__ float sm[];
    float* Qt = sm;                          // [HD][BQ]
    float* Kt = Qt + HD * PA_BQ;             // [HD][BK + 4]   (also V tile [BK][HD])
    float* W = Kt + HD * PA_KT_STRIDE;       // [BQ][BK]
    const int t0 = blockIdx.x * PA_BQ, h = blockIdx.y;
    const int kvh = h / (P.nh / P.nkv);
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    const int qend = min(t0 + PA_BQ, T);

    // Q tile, transposed
    for (int i = tid; i < PA_BQ * HD; i += PA_THREADS) {
        int r = i / HD, d = i % HD;
        int t = t0 + r;
        Qt[d * PA_BQ + r] = (t < T) ? P.q[(size_t)t * P.ldq + (size_t)h * HD + d] : 0.0f;
    }
    const float* kb = P.kp + (size_t)kvh * HD;
    const float* vb = P.vp + (size_t)kvh * HD;
    const int nkt = (qend - 1 + PA_BK - 1) / PA_BK;  // key tiles covering keys < qend - 1

    auto load_kt = [&](int s0) {
        for (int i = tid; i < PA_BK * HD; i += PA_THREADS) {
            int c = i / HD, d = i % HD;
            int sidx = s0 + c;
            Kt[d * PA_KT_STRIDE + c] = (sidx < T) ? kb[(size_t)sidx * P.ldkv + d] : 0.0f;
        }
    };
    auto tile_s = [&](float (&acc)[4][4]) {
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;
#pragma unroll 8
        for (int d = 0; d < HD; d++) {
            float4 q4 = *reinterpret_cast<const float4*>(Qt + d * PA_BQ + ty * 4);
            float4 k4 = *reinterpret_cast<const float4*>(Kt + d * PA_KT_STRIDE + tx * 4);
            float qv[4] = {q4.x, q4.y, q4.z, q4.w}, kv[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = fmaf(qv[i], kv[j], acc[i][j]);
        }
    };

    // ---- pass 1: row maxima over keys s < t
    float rmax[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    for (int kt = 0; kt < nkt; kt++) {
        __syncthreads();
        load_kt(kt * PA_BK);
        __syncthreads();
        float acc[4][4];
        tile_s(acc);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            int t = t0 + ty * 4 + i;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                int sidx = kt * PA_BK + tx * 4 + j;
                if (sidx < t) rmax[i] = fmaxf(rmax[i], __fmul_rn(acc[i][j], P.scale));
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) rmax[i] = fmaxf(rmax[i], __shfl_xor_sync(0xffffffffu, rmax[i], o));

    // ---- pass 2: weights and W V
    constexpr int DC = HD / 16;  // output columns per thread
    float o[4][DC];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < DC; j++) o[i][j] = 0.0f;
    float rsum[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int kt = 0; kt < nkt; kt++) {
        __syncthreads();
        load_kt(kt * PA_BK);
        __syncthreads();
        float acc[4][4];
        tile_s(acc);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            int t = t0 + ty * 4 + i;
            int n8 = t - (t % 8);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                int sidx = kt * PA_BK + tx * 4 + j;
                float w = 0.0f;
                if (sidx < t) w = softmax_weight(__fmul_rn(acc[i][j], P.scale), rmax[i], sidx, n8);
                rsum[i] += w;
                W[(ty * 4 + i) * PA_BK + tx * 4 + j] = w;
            }
        }
        __syncthreads();
        // V tile [BK][HD] into the K buffer
        float* Vs = Kt;
        for (int i = tid; i < PA_BK * HD; i += PA_THREADS) {
            int c = i / HD, d = i % HD;
            int sidx = kt * PA_BK + c;
            Vs[c * HD + d] = (sidx < T) ? vb[(size_t)sidx * P.ldkv + d] : 0.0f;
        }
        __syncthreads();
#pragma unroll 4
        for (int k = 0; k < PA_BK; k++) {
            float wv[4];
#pragma unroll
            for (int i = 0; i < 4; i++) wv[i] = W[(ty * 4 + i) * PA_BK + k];
            const float* vr = Vs + k * HD + tx * DC;
#pragma unroll
            for (int j = 0; j < DC; j++) {
                float v = vr[j];
#pragma unroll
                for (int i = 0; i < 4; i++) o[i][j] = fmaf(wv[i], v, o[i][j]);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) rsum[i] += __shfl_xor_sync(0xffffffffu, rsum[i], off);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        int t = t0 + ty * 4 + i;
        if (t >= T) continue;
        float* out = P.out + (size_t)t * P.ldo + (size_t)h * HD + tx * DC;
        __half* o16 = P.out16 ? P.out16 + (size_t)t * 2 * P.nh * HD : nullptr;
        const float* vs = P.vself + (size_t)t * P.ldself + (size_t)kvh * HD + tx * DC;
#pragma unroll
        for (int j = 0; j < DC; j++) {
            float r = (t < 2) ? vs[j] : __fdiv_rn(o[i][j], rsum[i]);
            out[j] = r;
            if (o16) store_x16(o16, P.nh * HD, h * HD + tx * DC + j, r);
        }
    }
}

// ---- Tensor-core form of the tiled prefill attention (head_dim 64 or 128).
// One CTA of four warps per (64-query block, query head); warp w owns queries
// t0 + 16 w .. + 15.  Q, K and V tiles are split into fp16 hi = fp16(x) and
// lo = fp16(x - hi) in shared memory (rows of HD halves, 16-byte chunk c of
// row r stored at c ^ (r & 7) for conflict-free ldmatrix); every score is
// Qh.Kh + Qh.Kl + Ql.Kh and every output Wh.Vh + Wh.Vl + Wl.Vh (mma.sync
// m16n8k16, f32 accumulate), which keeps the f32 products to ~2^-22.  The
// two passes are those of k_pattn: the row maxima over the visible keys
// (s < t) first, then the weights (the reference's polynomial / exp with that
// maximum) and W V; the score accumulators of two 8-key blocks are reused
// directly as the A fragment of the W V step.  Query blocks run longest first.
constexpr int PM_BQ = 64, PM_BK = 64, PM_THREADS = 128;

// f32 tile rows [r0, r0 + 64) of `src` (row stride ld, HD features; rows past
// nrows are zero) -> hi and lo fp16 tiles in the swizzled layout.
template <int HD>
__device__ __forceinline__ void pm_fill(const float* __restrict__ src, size_t ld, int r0, int nrows, __half* hi,
                                        __half* lo) {
    constexpr int Q4 = HD / 4;  // float4 per row
    for (int i = threadIdx.x; i < PM_BQ * Q4; i += PM_THREADS) {
        const int r = i / Q4, c4 = i % Q4;
        const int gr = r0 + r;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (gr < nrows) v = *reinterpret_cast<const float4*>(src + (size_t)gr * ld + 4 * c4);
        uint2 h, l;
        h.x = split_pair(v.x, v.y, false);
        h.y = split_pair(v.z, v.w, false);
        l.x = split_pair(v.x, v.y, true);
        l.y = split_pair(v.z, v.w, true);
        const int chunk = (c4 >> 1) ^ (r & 7);
        const size_t off = (size_t)r * HD + chunk * 8 + (c4 & 1) * 4;  // halves
        *reinterpret_cast<uint2*>(hi + off) = h;
        *reinterpret_cast<uint2*>(lo + off) = l;
    }
}

// Address (for this lane) of the 8x8 matrix `mi` of an ldmatrix.x4 over rows
// row0 + (row8 ? 8 : 0) + (lane & 7), 16-byte chunk `chunk`.
template <int HD>
__device__ __forceinline__ const __half* pm_addr(const __half* tile, int row, int chunk) {
    return tile + (size_t)row * HD + ((chunk ^ (row & 7)) * 8);
}

// The prompt's f32 K and V rows -> the four fp16 planes of kv16 (K hi, K lo,
// V hi, V lo; rows of nk = nkv * hd halves), once per layer, so that the
// attention CTAs copy ready tiles instead of converting every tile they read.
__global__ void k_split_kv(const float* __restrict__ kp, const float* __restrict__ vp, size_t ldkv, int T, int nk,
                           __half* __restrict__ kv16) {
    const size_t plane = (size_t)T * nk, n4 = plane / 4;
    const int q4 = nk / 4;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const size_t t = i / q4, c = 4 * (i % q4);
        const float4 k = *reinterpret_cast<const float4*>(kp + t * ldkv + c);
        const float4 v = *reinterpret_cast<const float4*>(vp + t * ldkv + c);
        const size_t o = t * nk + c;
        *reinterpret_cast<uint2*>(kv16 + o) = make_uint2(split_pair(k.x, k.y, false), split_pair(k.z, k.w, false));
        *reinterpret_cast<uint2*>(kv16 + plane + o) = make_uint2(split_pair(k.x, k.y, true), split_pair(k.z, k.w, true));
        *reinterpret_cast<uint2*>(kv16 + 2 * plane + o) = make_uint2(split_pair(v.x, v.y, false), split_pair(v.z, v.w, false));
        *reinterpret_cast<uint2*>(kv16 + 3 * plane + o) = make_uint2(split_pair(v.x, v.y, true), split_pair(v.z, v.w, true));
    }
}

// Rows [r0, r0 + 64) of one KV head's fp16 plane (row stride nk halves, rows
// past T zero) -> a swizzled tile, by cp.async (the caller commits and waits).
template <int HD>
__device__ __forceinline__ void pm_copy(const __half* __restrict__ plane, int nk, int r0, int T, __half* tile) {
    constexpr int CPR = HD / 8;
    for (int i = threadIdx.x; i < PM_BK * CPR; i += PM_THREADS) {
        const int r = i / CPR, c = i % CPR;
        const bool in = r0 + r < T;
        cp_async16(tile + (size_t)r * HD + ((c ^ (r & 7)) * 8), plane + (size_t)(in ? r0 + r : 0) * nk + c * 8,
                   in ? 16 : 0);
    }
}

template <int HD>
__global__ void __launch_bounds__(PM_THREADS, 2) k_pattn_mma(AttnParams P, int T) {
    constexpr int KS = HD / 16;  // 16-feature steps of a score
    constexpr int NB = HD / 8;   // 8-feature blocks of an output row
    pdl_trigger();
    extern __shared__ __align__(16) uint8_t pm_smem[];
    __half* Qh = reinterpret_cast<__half*>(pm_smem);
    __half* Ql = Qh + PM_BQ * HD;
    __half* Kh = Ql + PM_BQ * HD;
    __half* Kl = Kh + PM_BK * HD;
    __half* Vh = Kl + PM_BK * HD;
    __half* Vl = Vh + PM_BK * HD;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int t = lane & 3, q4 = lane >> 2;
    const int qb = (int)gridDim.x - 1 - (int)blockIdx.x;  // longest blocks first
    const int t0 = qb * PM_BQ, h = blockIdx.y;
    const int kvh = h / (P.nh / P.nkv);
    const int qend = min(t0 + PM_BQ, T);
    const int nkt = (qend - 1 + PM_BK - 1) / PM_BK;  // key tiles covering keys < qend - 1
    const int ra = t0 + warp * 16 + q4, rb = ra + 8;   // this thread's two query rows

    pm_fill<HD>(P.q + (size_t)h * HD, P.ldq, t0, T, Qh, Ql);
    const float* kb = P.kp + (size_t)kvh * HD;
    const float* vb = P.vp + (size_t)kvh * HD;
    const int mi = lane >> 3, mr = lane & 7;
    // this KV head's columns of the fp16 planes (when the caller made them)
    const int nk = P.nkv * HD;
    const size_t plane = (size_t)T * nk;
    const __half* k16 = P.kv16 ? P.kv16 + (size_t)kvh * HD : nullptr;
    auto load_k = [&](int kt) {
        if (k16) {
            pm_copy<HD>(k16, nk, kt * PM_BK, T, Kh);
            pm_copy<HD>(k16 + plane, nk, kt * PM_BK, T, Kl);
        } else {
            pm_fill<HD>(kb, P.ldkv, kt * PM_BK, T, Kh, Kl);
        }
    };
    auto load_v = [&](int kt) {
        if (k16) {
            pm_copy<HD>(k16 + 2 * plane, nk, kt * PM_BK, T, Vh);
            pm_copy<HD>(k16 + 3 * plane, nk, kt * PM_BK, T, Vl);
        } else {
            pm_fill<HD>(vb, P.ldkv, kt * PM_BK, T, Vh, Vl);
        }
    };

    // S = Q K^T of key tile kt for the warp's 16 rows (acc[nb][0..3]: rows ra
    // / rb, keys 64 kt + 8 nb + 2 t, + 1), scaled
    auto scores = [&](float (&acc)[8][4]) {
#pragma unroll
        for (int nb = 0; nb < 8; nb++)
#pragma unroll
            for (int e = 0; e < 4; e++) acc[nb][e] = 0.0f;
#pragma unroll
        for (int kk = 0; kk < KS; kk++) {
            uint32_t ah[4], al[4];
            const int arow = warp * 16 + (mi & 1) * 8 + mr, achunk = 2 * kk + (mi >> 1);
            ldsm_x4(ah, pm_addr<HD>(Qh, arow, achunk));
            ldsm_x4(al, pm_addr<HD>(Ql, arow, achunk));
#pragma unroll
            for (int nb = 0; nb < 8; nb += 2) {
                uint32_t bh[4], bl[4];
                const int brow = 8 * (nb + (mi >> 1)) + mr, bchunk = 2 * kk + (mi & 1);
                ldsm_x4(bh, pm_addr<HD>(Kh, brow, bchunk));
                ldsm_x4(bl, pm_addr<HD>(Kl, brow, bchunk));
                mma16816(acc[nb], ah, bh[0], bh[1]);
                mma16816(acc[nb], ah, bl[0], bl[1]);
                mma16816(acc[nb], al, bh[0], bh[1]);
                mma16816(acc[nb + 1], ah, bh[2], bh[3]);
                mma16816(acc[nb + 1], ah, bl[2], bl[3]);
                mma16816(acc[nb + 1], al, bh[2], bh[3]);
            }
        }
#pragma unroll
        for (int nb = 0; nb < 8; nb++)
#pragma unroll
            for (int e = 0; e < 4; e++) acc[nb][e] = __fmul_rn(acc[nb][e], P.scale);
    };

    // ---- pass 1: row maxima over keys s < t
    float mxa = -INFINITY, mxb = -INFINITY;
    for (int kt = 0; kt < nkt; kt++) {
        __syncthreads();
        load_k(kt);
        cp_async_commit();
        cp_async_wait<0>();
        __syncthreads();
        float acc[8][4];
        scores(acc);
#pragma unroll
        for (int nb = 0; nb < 8; nb++) {
            const int key = kt * PM_BK + 8 * nb + 2 * t;
            if (key < ra) mxa = fmaxf(mxa, acc[nb][0]);
            if (key + 1 < ra) mxa = fmaxf(mxa, acc[nb][1]);
            if (key < rb) mxb = fmaxf(mxb, acc[nb][2]);
            if (key + 1 < rb) mxb = fmaxf(mxb, acc[nb][3]);
        }
    }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
        mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, o));
        mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, o));
    }

    // ---- pass 2: weights and W V
    float o[NB][4];
#pragma unroll
    for (int nb = 0; nb < NB; nb++)
#pragma unroll
        for (int e = 0; e < 4; e++) o[nb][e] = 0.0f;
    float suma = 0.0f, sumb = 0.0f;
    const int n8a = ra - (ra % 8), n8b = rb - (rb % 8);
    for (int kt = 0; kt < nkt; kt++) {
        __syncthreads();
        load_k(kt);
        load_v(kt);
        cp_async_commit();
        cp_async_wait<0>();
        __syncthreads();
        float acc[8][4];
        scores(acc);
#pragma unroll
        for (int nb = 0; nb < 8; nb++) {
            const int key = kt * PM_BK + 8 * nb + 2 * t;
            const float w0 = key < ra ? softmax_weight(acc[nb][0], mxa, key, n8a) : 0.0f;
            const float w1 = key + 1 < ra ? softmax_weight(acc[nb][1], mxa, key + 1, n8a) : 0.0f;
            const float w2 = key < rb ? softmax_weight(acc[nb][2], mxb, key, n8b) : 0.0f;
            const float w3 = key + 1 < rb ? softmax_weight(acc[nb][3], mxb, key + 1, n8b) : 0.0f;
            suma += w0 + w1;
            sumb += w2 + w3;
            acc[nb][0] = w0;
            acc[nb][1] = w1;
            acc[nb][2] = w2;
            acc[nb][3] = w3;
        }
#pragma unroll
        for (int j = 0; j < 4; j++) {  // 16 keys: score blocks 2 j and 2 j + 1
            uint32_t wh[4], wl[4];
            wh[0] = split_pair(acc[2 * j][0], acc[2 * j][1], false);
            wh[1] = split_pair(acc[2 * j][2], acc[2 * j][3], false);
            wh[2] = split_pair(acc[2 * j + 1][0], acc[2 * j + 1][1], false);
            wh[3] = split_pair(acc[2 * j + 1][2], acc[2 * j + 1][3], false);
            wl[0] = split_pair(acc[2 * j][0], acc[2 * j][1], true);
            wl[1] = split_pair(acc[2 * j][2], acc[2 * j][3], true);
            wl[2] = split_pair(acc[2 * j + 1][0], acc[2 * j + 1][1], true);
            wl[3] = split_pair(acc[2 * j + 1][2], acc[2 * j + 1][3], true);
#pragma unroll
            for (int nb = 0; nb < NB; nb += 2) {
                uint32_t vh[4], vl[4];
                const int vrow = 16 * j + 8 * (mi & 1) + mr, vchunk = nb + (mi >> 1);
                ldsm_x4_t(vh, pm_addr<HD>(Vh, vrow, vchunk));
                ldsm_x4_t(vl, pm_addr<HD>(Vl, vrow, vchunk));
                mma16816(o[nb], wh, vh[0], vh[1]);
                mma16816(o[nb], wh, vl[0], vl[1]);
                mma16816(o[nb], wl, vh[0], vh[1]);
                mma16816(o[nb + 1], wh, vh[2], vh[3]);
                mma16816(o[nb + 1], wh, vl[2], vl[3]);
                mma16816(o[nb + 1], wl, vh[2], vh[3]);
            }
        }
    }
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
        suma += __shfl_xor_sync(0xffffffffu, suma, off);
        sumb += __shfl_xor_sync(0xffffffffu, sumb, off);
    }
#pragma unroll
    for (int half = 0; half < 2; half++) {
        const int tr = half ? rb : ra;
        if (tr >= T) continue;
        const float sum = half ? sumb : suma;
        float* out = P.out + (size_t)tr * P.ldo + (size_t)h * HD;
        __half* o16 = P.out16 ? P.out16 + (size_t)tr * 2 * P.nh * HD : nullptr;
        const float* vs = P.vself + (size_t)tr * P.ldself + (size_t)kvh * HD;
#pragma unroll
        for (int nb = 0; nb < NB; nb++) {
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int d = 8 * nb + 2 * t + e;
                const float r = (tr < 2) ? vs[d] : __fdiv_rn(o[nb][2 * half + e], sum);
                out[d] = r;
                if (o16) store_x16(o16, P.nh * HD, h * HD + d, r);
            }
        }
    }
}

template <int HD>
int launch_pattn_mma(const AttnParams& P, int T, cudaStream_t s) {
    const size_t smem = (size_t)6 * PM_BQ * HD * sizeof(__half);
    if (P.kv16) {
        const int nk = P.nkv * HD;
        HC_CHECK(P.ldkv % 4 == 0 && ((uintptr_t)P.kp & 15) == 0 && ((uintptr_t)P.vp & 15) == 0 &&
                     ((uintptr_t)P.kv16 & 15) == 0,
                 HC_ERR_INVALID, "prefill attention: K/V rows must be 16-byte aligned");
        const size_t n4 = (size_t)T * nk / 4;
        const unsigned g = (unsigned)std::min<size_t>((n4 + 255) / 256, 2048);
        k_split_kv<<<g, 256, 0, s>>>(P.kp, P.vp, P.ldkv, T, nk, P.kv16);
        HC_LAUNCH_CHECK();
    }
    if (smem > 48 * 1024)
        HC_CUDA(cudaFuncSetAttribute(k_pattn_mma<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid((unsigned)((T + PM_BQ - 1) / PM_BQ), (unsigned)P.nh);
    k_pattn_mma<HD><<<grid, PM_THREADS, smem, s>>>(P, T);
    HC_LAUNCH_CHECK();
    return HC_OK;
}

template <int HD>
int launch_pattn_hd(const AttnParams& P, int T, cudaStream_t s) {
    size_t smem = ((size_t)HD * PA_BQ + (size_t)HD * PA_KT_STRIDE + (size_t)PA_BQ * PA_BK) * sizeof(float);
    if (smem > 48 * 1024) HC_CUDA(cudaFuncSetAttribute(k_pattn<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid((unsigned)((T + PA_BQ - 1) / PA_BQ), (unsigned)P.nh);
    k_pattn<HD><<<grid, PA_THREADS, smem, s>>>(P, T);
    HC_LAUNCH_CHECK();
    return HC_OK;
}

}  // namespace

bool pattn_supported(int hd) { return hd == 16 || hd == 32 || hd == 64 || hd == 128; }

int launch_prefill_attention(const AttnParams& P, int T, cudaStream_t s) {
    if (T == 0) return HC_OK;
    switch (P.hd) {
        case 16: return launch_pattn_hd<16>(P, T, s);
        case 32: return launch_pattn_hd<32>(P, T, s);
        case 64: return launch_pattn_mma<64>(P, T, s);
        case 128: return launch_pattn_mma<128>(P, T, s);
        default:
            hc_set_error("tiled prefill attention: unsupported head_dim %d", P.hd);
            return HC_ERR_UNSUPPORTED;
    }
}

}  // namespace hc
