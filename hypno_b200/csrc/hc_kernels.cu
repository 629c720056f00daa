// CUDA kernels of the hypno sm_100a backend (CUDA-core part): Q4_0 pack /
// unpack / repack, the Q4_0 matvec for small token counts, RMSNorm, softmax,
// SiLU, RoPE, embedding gather, argmax and the seeded synthetic generator.
// The tensor-core GEMM lives in hc_gemm_tc.cu and attention in hc_attention.cu.
#include "hc_internal.h"
#include "hc_common.cuh"
#include "hc_gemm.h"

#include <algorithm>
#include <math.h>

namespace hc {

// ============================================================ Q4_0 pack/unpack

// Q4_0Block::quantize (quant.rs:49-71), one thread per 32-element block:
// scale = max|x|/7 in f32 (1.0 for an all-zero block), stored as f16 (RNE);
// q = clamp(round_half_away(x / scale_f32), -8, 7) + 8, low nibble = even
// element.  IEEE division and roundf keep it bit-exact.
__global__ void k_q4_quantize(const float* __restrict__ x, size_t nblocks, uint8_t* __restrict__ out) {
    size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    const float* src = x + b * 32;
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = src[i];
    float max_abs = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; i++) max_abs = fmaxf(max_abs, fabsf(v[i]));
    float scale = (max_abs > 0.0f) ? __fdiv_rn(max_abs, 7.0f) : 1.0f;
    uint32_t hb = (uint32_t)__half_as_ushort(__float2half_rn(scale));
    uint32_t packed[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int i = 0; i < 16; i++) {
        float r0 = roundf(__fdiv_rn(v[2 * i], scale));
        float r1 = roundf(__fdiv_rn(v[2 * i + 1], scale));
        int q0 = isnan(r0) ? 0 : (int)fminf(fmaxf(r0, -8.0f), 7.0f);
        int q1 = isnan(r1) ? 0 : (int)fminf(fmaxf(r1, -8.0f), 7.0f);
        uint32_t byte = (uint32_t)((q0 + 8) & 0x0F) | ((uint32_t)((q1 + 8) & 0x0F) << 4);
        packed[i >> 2] |= byte << (8 * (i & 3));
    }
    // 18-byte block at an address that is only 2-byte aligned: scale first,
    // then the 16 nibble bytes, written as 16-bit halves.
    uint16_t* o16 = reinterpret_cast<uint16_t*>(out + b * 18);
    o16[0] = (uint16_t)hb;
#pragma unroll
    for (int i = 0; i < 8; i++) o16[1 + i] = (uint16_t)(packed[i >> 1] >> (16 * (i & 1)));
}

// Q4_0Block::dequantize (quant.rs:25-34): (nibble - 8) * scale, exact in f32.
__global__ void k_q4_dequantize(const uint8_t* __restrict__ q, size_t nblocks, float* __restrict__ out) {
    size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    const uint8_t* blk = q + b * 18;
    float scale = __half2float(__ushort_as_half((uint16_t)(blk[0] | (blk[1] << 8))));
    float* dst = out + b * 32;
#pragma unroll
    for (int i = 0; i < 16; i++) {
        uint8_t byte = blk[2 + i];
        dst[2 * i] = (float)((int)(byte & 0x0F) - 8) * scale;
        dst[2 * i + 1] = (float)((int)(byte >> 4) - 8) * scale;
    }
}

// AoS 18-byte blocks -> nibble plane (uint4 per block) + scale plane.
__global__ void k_q4_split(const uint8_t* __restrict__ aos, size_t nblocks, uint4* __restrict__ qs,
                           __half* __restrict__ sc) {
    size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    const uint8_t* blk = aos + b * 18;
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; i++)
        w[i] = (uint32_t)blk[2 + 4 * i] | ((uint32_t)blk[3 + 4 * i] << 8) | ((uint32_t)blk[4 + 4 * i] << 16) |
               ((uint32_t)blk[5 + 4 * i] << 24);
    qs[b] = make_uint4(w[0], w[1], w[2], w[3]);
    sc[b] = __ushort_as_half((uint16_t)(blk[0] | (blk[1] << 8)));
}

static inline unsigned grid_for(size_t n, unsigned threads) {
    return (unsigned)((n + threads - 1) / threads);
}

int launch_q4_quantize(const float* x, size_t nblocks, uint8_t* out, cudaStream_t s) {
    if (nblocks == 0) return HC_OK;
    k_q4_quantize<<<grid_for(nblocks, 128), 128, 0, s>>>(x, nblocks, out);
    HC_LAUNCH_CHECK();
    return HC_OK;
}
int launch_q4_dequantize(const uint8_t* q, size_t nblocks, float* out, cudaStream_t s) {
    if (nblocks == 0) return HC_OK;
    k_q4_dequantize<<<grid_for(nblocks, 128), 128, 0, s>>>(q, nblocks, out);
    HC_LAUNCH_CHECK();
    return HC_OK;
}
// Launched after the plane split, as an ordinary (not programmatic) launch:
// the single-token matvec requests its weights before it waits for the
// previous kernel, which is only safe when that kernel did not write them;
// with this empty kernel in between, the split has completed and its stores
// are visible before any matvec that follows on the stream can start.
__global__ void k_weights_settled() {}

int launch_q4_split(const uint8_t* aos, size_t nblocks, uint4* qs, __half* sc, cudaStream_t s) {
    if (nblocks == 0) return HC_OK;
    k_q4_split<<<grid_for(nblocks, 256), 256, 0, s>>>(aos, nblocks, qs, sc);
    HC_LAUNCH_CHECK();
    k_weights_settled<<<1, 32, 0, s>>>();
    HC_LAUNCH_CHECK();
    return HC_OK;
}

// ============================================================ Q4_0 matvec
//
// y[m][row] = sum_b scale[row,b] * sum_j (nib[row,b,j] - 8) * x[m][32b + j]
// for k % 32 == 0 (blocks aligned with rows).  Up to MT tokens are handled
// per pass.  The per-block dot is formed exactly on integers-as-floats and
// folded in with one fma by the f32 scale.

__device__ __forceinline__ float nib_f(uint32_t w, int j) {
    // (nibble j of w) - 8 as an exact float: 2^23 + nib built by bit-or, then
    // 2^23 + 8 subtracted.
    return __int_as_float(0x4B000000 | ((w >> (4 * j)) & 0xF)) - 8388616.0f;
}

__device__ __forceinline__ float q4_block_dot(uint4 q, const float* xv) {
    float d0 = 0.0f, d1 = 0.0f, d2 = 0.0f, d3 = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        d0 = fmaf(nib_f(q.x, j), xv[j], d0);
        d1 = fmaf(nib_f(q.y, j), xv[8 + j], d1);
        d2 = fmaf(nib_f(q.z, j), xv[16 + j], d2);
        d3 = fmaf(nib_f(q.w, j), xv[24 + j], d3);
    }
    return (d0 + d1) + (d2 + d3);
}

// One CTA (GV_THREADS threads) per R rows.  Thread t takes blocks t,
// t + GV_THREADS, ... of every row (16-byte nibble loads, coalesced across the
// CTA), loads U such blocks of all R rows before any arithmetic (U x R x 16
// bytes in flight per thread), and loads each f32 x block once for the R rows
// (x traffic 128 B per R x 18 B of weights, so L1 stays below the DRAM rate).
// Each block's dot product is exact-order within the block and scaled once
// (fmaf by the f32 scale), as in kernels.rs:286-344; a thread sums its blocks
// in order, then the CTA reduces (warp tree, then warps in order), so the
// result does not depend on scheduling.
constexpr int GV_THREADS = 128;

template <int R, int U, int MT>
__global__ void __launch_bounds__(GV_THREADS) k_q4_gemv(const uint4* __restrict__ qs, const __half* __restrict__ sc,
                                                        const float* __restrict__ x, size_t ldx, int mtok,
                                                        float* __restrict__ y, size_t ldy, int epi,
                                                        const float* res, size_t ldres, int N, int KB) {
    __shared__ float red[GV_THREADS / 32][R * MT];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = blockIdx.x * R;
    int rows[R];
#pragma unroll
    for (int r = 0; r < R; r++) rows[r] = min(row0 + r, N - 1);
    for (int m0 = 0; m0 < mtok; m0 += MT) {
        float acc[R][MT];
#pragma unroll
        for (int r = 0; r < R; r++)
#pragma unroll
            for (int t = 0; t < MT; t++) acc[r][t] = 0.0f;
        for (int b0 = threadIdx.x; b0 < KB; b0 += GV_THREADS * U) {
            uint4 q[U][R];
            float s[U][R];
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int b = b0 + u * GV_THREADS;
#pragma unroll
                for (int r = 0; r < R; r++) {
                    if (b < KB) {
                        size_t bi = (size_t)rows[r] * KB + b;
                        q[u][r] = __ldg(qs + bi);
                        s[u][r] = __half2float(sc[bi]);
                    } else {
                        q[u][r] = make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);
                        s[u][r] = 0.0f;
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int b = b0 + u * GV_THREADS;
#pragma unroll
                for (int t = 0; t < MT; t++) {
                    if (b < KB && m0 + t < mtok) {
                        const float4* xp =
                            reinterpret_cast<const float4*>(x + (size_t)(m0 + t) * ldx + (size_t)b * 32);
                        float xv[32];
#pragma unroll
                        for (int i = 0; i < 8; i++) {
                            float4 f = __ldg(xp + i);
                            xv[4 * i] = f.x; xv[4 * i + 1] = f.y; xv[4 * i + 2] = f.z; xv[4 * i + 3] = f.w;
                        }
#pragma unroll
                        for (int r = 0; r < R; r++) acc[r][t] = fmaf(s[u][r], q4_block_dot(q[u][r], xv), acc[r][t]);
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < R; r++)
#pragma unroll
            for (int t = 0; t < MT; t++) {
                float v = warp_sum(acc[r][t]);
                if (lane == 0) red[warp][r * MT + t] = v;
            }
        __syncthreads();
        if (threadIdx.x < R * MT) {
            const int r = threadIdx.x / MT, t = threadIdx.x % MT;
            const int row = row0 + r, m = m0 + t;
            float v = 0.0f;
#pragma unroll
            for (int w = 0; w < GV_THREADS / 32; w++) v += red[w][threadIdx.x];
            if (row < N && m < mtok) {
                if (epi == EPI_ADD && res) v = v + res[(size_t)m * ldres + row];
                y[(size_t)m * ldy + row] = v;
            }
        }
        __syncthreads();
    }
}

// ---- Single-token matvec with a packed dot (k % 32 == 0, k <= 24576).
//
// Nibble p of a 32-bit word w (p = 0..4: bits 4p..4p+3, inside the f32
// mantissa) is isolated with one AND; the bits read as an f32 are the
// denormal nib * 2^(4p) * 2^-149.  One packed f32x2 fma with x 2^126 and
// + (-8 * 2^(4p-23)) gives (nib - 8) * 2^(4p-23) exactly (a power-of-two
// product, then an exact sum of small integers times one power of two;
// denormals are kept, the build does not flush them).  Nibbles 5..7 come from
// w >> 20 at positions 0..2.  x is staged once per CTA in shared memory
// scaled by 2^(23-4p) (exact), so a second packed fma accumulates
// (nib - 8) * x with an exact product and one rounding per add, as the scalar
// path does.  Position of element j (0..7) of a word: 0 1 2 3 4 | 0 1 2.
constexpr int G1_THREADS = 256;

__device__ __forceinline__ float2 nib_pair(uint32_t a, uint32_t ma, uint32_t b, uint32_t mb, float2 bias) {
    const float2 f = make_float2(__uint_as_float(a & ma), __uint_as_float(b & mb));
    const float2 up = make_float2(__uint_as_float(0x7E800000u), __uint_as_float(0x7E800000u));  // 2^126
    return __ffma2_rn(f, up, bias);
}

// Adds word w's 8 products (nib_j - 8) * x_j to the two pair accumulators;
// xa / xb are the word's scaled x elements 0..3 / 4..7.
__device__ __forceinline__ void word_dot_packed(uint32_t w, float4 xa, float4 xb, float2& a0, float2& a1) {
    const float b0 = -9.5367431640625e-07f, b1 = -1.52587890625e-05f, b2 = -0.000244140625f;  // -8 * 2^(4p-23)
    const float b3 = -0.00390625f, b4 = -0.0625f;
    const uint32_t hi = w >> 20;
    a0 = __ffma2_rn(nib_pair(w, 0xFu, w, 0xF0u, make_float2(b0, b1)), make_float2(xa.x, xa.y), a0);
    a1 = __ffma2_rn(nib_pair(w, 0xF00u, w, 0xF000u, make_float2(b2, b3)), make_float2(xa.z, xa.w), a1);
    a0 = __ffma2_rn(nib_pair(w, 0xF0000u, hi, 0xFu, make_float2(b4, b0)), make_float2(xb.x, xb.y), a0);
    a1 = __ffma2_rn(nib_pair(hi, 0xF0u, hi, 0xF00u, make_float2(b1, b2)), make_float2(xb.z, xb.w), a1);
}

// Scaled x of block b starts at float4 G1_XS * b: 8 float4 of data plus one of
// padding, so lanes reading consecutive blocks hit distinct shared-memory banks.
constexpr int G1_XS = 9;

// One warp per group of R rows at a time (grid-stride over the groups); lane
// l takes blocks l, l + 32, ... of the R rows, U blocks of loads before any
// arithmetic; each x chunk (one word's 8 elements) is read once for the R
// rows; the warp then sums its lanes in a fixed tree.
// Elements 4i..4i+3 of x (word positions (4i & 7) + 0..3) times 2^(23-4p)
// for nibble position p: 2^23, 2^19, 2^15, 2^11, 2^7 (exact).
__device__ __forceinline__ float4 g1_prescale(float4 v, int i) {
    if ((i & 1) == 0) {  // word elements 0..3: positions 0 1 2 3
        v.x = __fmul_rn(v.x, 8388608.0f);
        v.y = __fmul_rn(v.y, 524288.0f);
        v.z = __fmul_rn(v.z, 32768.0f);
        v.w = __fmul_rn(v.w, 2048.0f);
    } else {             // word elements 4..7: positions 4 0 1 2
        v.x = __fmul_rn(v.x, 128.0f);
        v.y = __fmul_rn(v.y, 8388608.0f);
        v.z = __fmul_rn(v.z, 524288.0f);
        v.w = __fmul_rn(v.w, 32768.0f);
    }
    return v;
}

// nw (may be null): x is first replaced by RMSNorm(x) * nw, computed by
// every CTA with k_rmsnorm_v4's arithmetic (the single-token forward then
// needs no separate norm kernel).  silu: the weight is a fused gate/up
// weight in blocks of GU_BLOCK gate rows and their GU_BLOCK up rows; a
// warp takes a gate row and its up row and writes y[i] = silu(gate) * up
// (k_silu_mul's arithmetic) for the N / 2 outputs.  PRE (every warp has at
// most one row group): the warp's weights are requested before the wait for
// the previous kernel; with several groups per warp that hoisting slows the
// loop (128256 x 4096: 81 against 74 µs), so it is left out there.
template <int R, int U, bool PRE>
__global__ void __launch_bounds__(G1_THREADS, 3) k_q4_gemv1(const uint4* __restrict__ qs, const __half* __restrict__ sc,
                                                         const float* __restrict__ x, float* __restrict__ y, int epi,
                                                         const float* res, int N, int KB,
                                                         const float* __restrict__ nw, float eps, int silu) {
    pdl_trigger();
    extern __shared__ float4 xs4[];  // x' = x scaled per nibble position, KB x G1_XS float4
    __shared__ float red[32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int groups = silu ? N / 2 : (N + R - 1) / R;
    auto row_of = [&](int g, int r) {
        return silu ? (g / GU_BLOCK) * (2 * GU_BLOCK) + g % GU_BLOCK + r * GU_BLOCK : min(g * R + r, N - 1);
    };
    // one batch of U blocks (lane + 32 u from b0) of the group's R rows
    uint4 q[U][R];
    float s[U][R];
    auto load_batch = [&](int g, int b0) {
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int b = b0 + u * 32;
#pragma unroll
            for (int r = 0; r < R; r++) {
                if (b < KB) {
                    const size_t bi = (size_t)row_of(g, r) * KB + b;
                    q[u][r] = __ldg(qs + bi);
                    s[u][r] = __half2float(sc[bi]);
                } else {
                    q[u][r] = make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);
                    s[u][r] = 0.0f;
                }
            }
        }
    };
    // the weights do not depend on the previous kernel: the warp's first
    // batch is in flight before the wait for it
    const int g0 = blockIdx.x * (G1_THREADS / 32) + warp;
    if (PRE && g0 < groups) load_batch(g0, lane);
    pdl_wait();
    // x, read once: staged raw while the sum of squares accumulates, then
    // (with nw) normalized in place; each thread rewrites only its own
    // elements
    float ss = 0.0f;
    for (int i = threadIdx.x; i < KB * 8; i += G1_THREADS) {
        float4 v = __ldg(reinterpret_cast<const float4*>(x) + i);
        if (nw) {
            ss = fmaf(v.x, v.x, ss);
            ss = fmaf(v.y, v.y, ss);
            ss = fmaf(v.z, v.z, ss);
            ss = fmaf(v.w, v.w, ss);
        } else {
            v = g1_prescale(v, i);
        }
        xs4[(i >> 3) * G1_XS + (i & 7)] = v;
    }
    if (nw) {
        ss = block_sum(ss, red);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)(KB * 32)), eps)));
        for (int i = threadIdx.x; i < KB * 8; i += G1_THREADS) {
            float4 v = xs4[(i >> 3) * G1_XS + (i & 7)];
            const float4 ww = __ldg(reinterpret_cast<const float4*>(nw) + i);
            v.x = __fmul_rn(__fmul_rn(v.x, inv), ww.x);
            v.y = __fmul_rn(__fmul_rn(v.y, inv), ww.y);
            v.z = __fmul_rn(__fmul_rn(v.z, inv), ww.z);
            v.w = __fmul_rn(__fmul_rn(v.w, inv), ww.w);
            xs4[(i >> 3) * G1_XS + (i & 7)] = g1_prescale(v, i);
        }
    }
    __syncthreads();
    for (int g = g0; g < groups; g += gridDim.x * (G1_THREADS / 32)) {
        float acc[R];
#pragma unroll
        for (int r = 0; r < R; r++) acc[r] = 0.0f;
        for (int b0 = lane; b0 < KB; b0 += 32 * U) {
            if (!PRE || g != g0 || b0 != lane) load_batch(g, b0);
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int b = b0 + u * 32;
                if (b < KB) {
                    const float4* xb4 = xs4 + (size_t)b * G1_XS;
                    float2 a[R][2];
#pragma unroll
                    for (int r = 0; r < R; r++) a[r][0] = a[r][1] = make_float2(0.0f, 0.0f);
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const float4 xa = xb4[2 * i], xb = xb4[2 * i + 1];
#pragma unroll
                        for (int r = 0; r < R; r++) {
                            const uint32_t wd = i == 0 ? q[u][r].x : i == 1 ? q[u][r].y : i == 2 ? q[u][r].z : q[u][r].w;
                            word_dot_packed(wd, xa, xb, a[r][0], a[r][1]);
                        }
                    }
#pragma unroll
                    for (int r = 0; r < R; r++)
                        acc[r] = fmaf(s[u][r], (a[r][0].x + a[r][0].y) + (a[r][1].x + a[r][1].y), acc[r]);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < R; r++) acc[r] = warp_sum(acc[r]);
        if (lane == 0 && silu) {
            y[g] = __fmul_rn(silu_f(acc[0]), acc[1]);
        } else if (lane == 0) {
#pragma unroll
            for (int r = 0; r < R; r++) {
                const int row = g * R + r;
                if (row < N) {
                    float v = acc[r];
                    if (epi == EPI_ADD && res) v = v + res[row];
                    y[row] = v;
                }
            }
        }
    }
}

// General Q4_0 matvec for k % 32 != 0: blocks straddle row boundaries
// (kernels.rs:281-349).  One warp per (row, token); element e of the
// flattened tensor uses block e/32, nibble e%32.
__global__ void k_q4_gemv_general(const uint4* __restrict__ qs, const __half* __restrict__ sc, size_t nblocks,
                                  const float* __restrict__ x, size_t ldx, int mtok, float* __restrict__ y,
                                  size_t ldy, int epi, const float* res, size_t ldres, int N, int K) {
    int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= N * mtok) return;
    int row = warp % N, m = warp / N;
    const uint8_t* qb = reinterpret_cast<const uint8_t*>(qs);
    float acc = 0.0f;
    for (int i = lane; i < K; i += 32) {
        size_t e = (size_t)row * K + i;
        size_t b = e >> 5;
        if (b >= nblocks) break;
        int j = (int)(e & 31);
        uint8_t byte = qb[b * 16 + (j >> 1)];
        int nib = (j & 1) ? (byte >> 4) : (byte & 0xF);
        float deq = (float)(nib - 8) * __half2float(sc[b]);
        acc = fmaf(deq, x[(size_t)m * ldx + i], acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) {
        if (epi == EPI_ADD && res) acc = acc + res[(size_t)m * ldres + row];
        y[(size_t)m * ldy + row] = acc;
    }
}

// FP32 / FP16 weight matvec (kernels.rs:69-241, 537-586): one warp per
// (row, token).
template <typename T>
__device__ __forceinline__ float ld_as_f32(const T* p);
template <>
__device__ __forceinline__ float ld_as_f32<float>(const float* p) { return __ldg(p); }
template <>
__device__ __forceinline__ float ld_as_f32<__half>(const __half* p) { return __half2float(*p); }

template <typename T>
__global__ void k_dense_gemv(const T* __restrict__ w, const float* __restrict__ x, size_t ldx, int mtok,
                             float* __restrict__ y, size_t ldy, int epi, const float* res, size_t ldres, int N,
                             int K) {
    int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= N * mtok) return;
    int row = warp % N, m = warp / N;
    const T* wr = w + (size_t)row * K;
    const float* xr = x + (size_t)m * ldx;
    float acc = 0.0f;
    for (int i = lane; i < K; i += 32) acc = fmaf(ld_as_f32<T>(wr + i), xr[i], acc);
    acc = warp_sum(acc);
    if (lane == 0) {
        if (epi == EPI_ADD && res) acc = acc + res[(size_t)m * ldres + row];
        y[(size_t)m * ldy + row] = acc;
    }
}

template <int R, int U, int MT>
static void launch_gemv_t(const hc_q4_matrix& w, const float* x, size_t ldx, size_t mtok, float* y, size_t ldy,
                          int epi, const float* res, size_t ldres, cudaStream_t s) {
    unsigned grid = (unsigned)((w.n + R - 1) / R);
    k_q4_gemv<R, U, MT><<<grid, GV_THREADS, 0, s>>>(w.qs, w.sc, x, ldx, (int)mtok, y, ldy, epi, res, ldres,
                                                    (int)w.n, (int)(w.k / 32));
}

// 8 rows per CTA (x reused 8 times) when that still gives ~2 CTAs per SM,
// fewer for short matrices; U = 2 unrolled blocks per thread when the rows
// are longer than one block per thread.
template <int MT>
static void launch_gemv_mt(const hc_q4_matrix& w, const float* x, size_t ldx, size_t mtok, float* y, size_t ldy,
                           int epi, const float* res, size_t ldres, cudaStream_t s) {
    const size_t kb = w.k / 32;
    const bool u2 = kb > (size_t)GV_THREADS;
    if constexpr (MT > 1) {  // several tokens: their accumulators take the registers of extra rows
        if (u2) launch_gemv_t<2, 2, MT>(w, x, ldx, mtok, y, ldy, epi, res, ldres, s);
        else launch_gemv_t<2, 1, MT>(w, x, ldx, mtok, y, ldy, epi, res, ldres, s);
    } else {
        if (w.n >= 8 * 296) {
            if (u2) launch_gemv_t<8, 2, 1>(w, x, ldx, mtok, y, ldy, epi, res, ldres, s);
            else launch_gemv_t<8, 1, 1>(w, x, ldx, mtok, y, ldy, epi, res, ldres, s);
        } else if (w.n >= 4 * 296) {
            if (u2) launch_gemv_t<4, 2, 1>(w, x, ldx, mtok, y, ldy, epi, res, ldres, s);
            else launch_gemv_t<4, 1, 1>(w, x, ldx, mtok, y, ldy, epi, res, ldres, s);
        } else {
            if (u2) launch_gemv_t<2, 2, 1>(w, x, ldx, mtok, y, ldy, epi, res, ldres, s);
            else launch_gemv_t<2, 1, 1>(w, x, ldx, mtok, y, ldy, epi, res, ldres, s);
        }
    }
}

static int launch_gemv(const hc_q4_matrix& w, const float* x, size_t ldx, size_t mtok, float* y, size_t ldy,
                       int epi, const float* res, size_t ldres, cudaStream_t s) {
    const size_t kb = w.k / 32;
    if (mtok == 1 && kb <= 768) {
        // a few CTAs per SM, each staging x once and striding over row groups
        const size_t smem = kb * G1_XS * sizeof(float4);
        const size_t groups = (w.n + 1) / 2;  // 2 rows per warp
        const size_t per_cta = G1_THREADS / 32;
        unsigned grid = (unsigned)std::min<size_t>((groups + per_cta - 1) / per_cta, 148 * 3);
        auto kfn = groups <= (size_t)grid * per_cta ? k_q4_gemv1<2, 4, true> : k_q4_gemv1<2, 4, false>;
        if (smem > 48 * 1024) cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        return launch_pdl(kfn, dim3(grid), dim3(G1_THREADS), smem, s, w.qs, w.sc, x, y, epi, res, (int)w.n, (int)kb,
                          (const float*)nullptr, 0.0f, 0);
    }
    if (mtok == 1) launch_gemv_mt<1>(w, x, ldx, mtok, y, ldy, epi, res, ldres, s);
    else if (mtok <= 4) launch_gemv_mt<4>(w, x, ldx, mtok, y, ldy, epi, res, ldres, s);
    else launch_gemv_mt<8>(w, x, ldx, mtok, y, ldy, epi, res, ldres, s);
    return HC_OK;
}

bool gemv1_fusable(const DevWeight& w, const float* x, const float* norm_w, bool silu) {
    if (w.dtype != HC_DTYPE_Q4_0) return false;
    const hc_q4_matrix& q = w.q4;
    return q.k % 32 == 0 && q.k / 32 <= 768 && q.nblocks >= q.n * (q.k / 32) && ((uintptr_t)x & 15) == 0 &&
           ((uintptr_t)norm_w & 15) == 0 && (!silu || q.n % (2 * GU_BLOCK) == 0);
}

int launch_gemv1_fused(const DevWeight& w, const float* x, float* y, const float* norm_w, float eps, bool silu,
                       cudaStream_t s) {
    HC_CHECK(gemv1_fusable(w, x, norm_w, silu), HC_ERR_INVALID, "fused single-token matvec: unsupported weight");
    const hc_q4_matrix& q = w.q4;
    const size_t kb = q.k / 32;
    const size_t smem = kb * G1_XS * sizeof(float4);
    const size_t groups = silu ? q.n / 2 : (q.n + 1) / 2;
    const size_t per_cta = G1_THREADS / 32;
    const unsigned grid = (unsigned)std::min<size_t>((groups + per_cta - 1) / per_cta, 148 * 3);
    auto kfn = groups <= (size_t)grid * per_cta ? k_q4_gemv1<2, 4, true> : k_q4_gemv1<2, 4, false>;
    if (smem > 48 * 1024) HC_CUDA(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    return launch_pdl(kfn, dim3(grid), dim3(G1_THREADS), smem, s, q.qs, q.sc, x, y, (int)EPI_STORE,
                      (const float*)nullptr, (int)q.n, (int)kb, norm_w, eps, silu ? 1 : 0);
}

int launch_matmul(const DevWeight& w, const float* x, size_t ldx, size_t mtok, float* y, size_t ldy, int epi,
                  const float* res, size_t ldres, cudaStream_t s) {
    if (mtok == 0 || w.n == 0) return HC_OK;
    if (w.dtype == HC_DTYPE_Q4_0) {
        const hc_q4_matrix& q = w.q4;
        bool aligned = (q.k % 32 == 0) && (((uintptr_t)x & 15) == 0) && (ldx % 4 == 0) &&
                       (q.nblocks >= q.n * (q.k / 32));
        if (aligned) {
            HC_TRY(launch_gemv(q, x, ldx, mtok, y, ldy, epi, res, ldres, s));
        } else {
            size_t warps = q.n * mtok;
            k_q4_gemv_general<<<grid_for(warps * 32, 256), 256, 0, s>>>(q.qs, q.sc, q.nblocks, x, ldx, (int)mtok, y,
                                                                        ldy, epi, res, ldres, (int)q.n, (int)q.k);
        }
    } else if (w.dtype == HC_DTYPE_FP32) {
        size_t warps = w.n * mtok;
        k_dense_gemv<float><<<grid_for(warps * 32, 256), 256, 0, s>>>((const float*)w.dense, x, ldx, (int)mtok, y,
                                                                      ldy, epi, res, ldres, (int)w.n, (int)w.k);
    } else if (w.dtype == HC_DTYPE_FP16) {
        size_t warps = w.n * mtok;
        k_dense_gemv<__half><<<grid_for(warps * 32, 256), 256, 0, s>>>((const __half*)w.dense, x, ldx, (int)mtok,
                                                                       y, ldy, epi, res, ldres, (int)w.n, (int)w.k);
    } else {
        hc_set_error("matmul: unsupported weight dtype %u", w.dtype);
        return HC_ERR_UNSUPPORTED;
    }
    HC_LAUNCH_CHECK();
    return HC_OK;
}

// ============================================================ RMSNorm
// kernels.rs:592-625: ms = sum(x^2)/n, inv = 1/sqrt(ms + eps), y = (x*inv)*w.
__global__ void k_rmsnorm(const float* __restrict__ x, size_t ldx, const float* __restrict__ w,
                          float* __restrict__ out, size_t ldo, int n, float eps, __half* __restrict__ out16) {
    pdl_trigger();
    __shared__ float red[32];
    const float* xr = x + (size_t)blockIdx.x * ldx;
    float* orow = out + (size_t)blockIdx.x * ldo;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
    ss = block_sum(ss, red);
    float ms = __fdiv_rn(ss, (float)n);
    float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float o = __fmul_rn(__fmul_rn(xr[i], inv), w[i]);
        orow[i] = o;
        if (out16) store_x16(out16 + (size_t)blockIdx.x * 2 * n, n, i, o);
    }
}

// Same arithmetic with 16-byte accesses (n % 4 == 0, 16-byte aligned rows):
// one float4 per thread per pass, the row held in registers between passes.
template <int VPT>
__global__ void k_rmsnorm_v4(const float* __restrict__ x, size_t ldx, const float* __restrict__ w,
                             float* __restrict__ out, size_t ldo, int n, float eps, __half* __restrict__ out16) {
    pdl_trigger();
    __shared__ float red[32];
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)blockIdx.x * ldx);
    const float4* wr = reinterpret_cast<const float4*>(w);
    float4* orow = reinterpret_cast<float4*>(out + (size_t)blockIdx.x * ldo);
    const int n4 = n / 4;
    float4 v[VPT];
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < VPT; j++) {
        int i = threadIdx.x + j * blockDim.x;
        v[j] = i < n4 ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        ss = fmaf(v[j].x, v[j].x, ss);
        ss = fmaf(v[j].y, v[j].y, ss);
        ss = fmaf(v[j].z, v[j].z, ss);
        ss = fmaf(v[j].w, v[j].w, ss);
    }
    ss = block_sum(ss, red);
    float ms = __fdiv_rn(ss, (float)n);
    float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
#pragma unroll
    for (int j = 0; j < VPT; j++) {
        int i = threadIdx.x + j * blockDim.x;
        if (i < n4) {
            float4 ww = wr[i], o;
            o.x = __fmul_rn(__fmul_rn(v[j].x, inv), ww.x);
            o.y = __fmul_rn(__fmul_rn(v[j].y, inv), ww.y);
            o.z = __fmul_rn(__fmul_rn(v[j].z, inv), ww.z);
            o.w = __fmul_rn(__fmul_rn(v[j].w, inv), ww.w);
            orow[i] = o;
            if (out16) {
                __half* r16 = out16 + (size_t)blockIdx.x * (2 * (size_t)n);
                store_x16(r16, n, 4 * i, o.x);
                store_x16(r16, n, 4 * i + 1, o.y);
                store_x16(r16, n, 4 * i + 2, o.z);
                store_x16(r16, n, 4 * i + 3, o.w);
            }
        }
    }
}

int launch_rmsnorm(const float* x, size_t ldx, const float* w, float* out, size_t ldo, size_t rows, size_t n,
                   float eps, cudaStream_t s, __half* out16) {
    if (rows == 0) return HC_OK;
    bool vec = n % 4 == 0 && ldx % 4 == 0 && ldo % 4 == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)w & 15) == 0 &&
               ((uintptr_t)out & 15) == 0 && n <= 4 * 1024 * 4;
    if (vec) {
        size_t n4 = n / 4;
        unsigned threads = (unsigned)std::min<size_t>(1024, ((n4 + 31) / 32) * 32);
        size_t vpt = (n4 + threads - 1) / threads;
        if (vpt <= 1) k_rmsnorm_v4<1><<<(unsigned)rows, threads, 0, s>>>(x, ldx, w, out, ldo, (int)n, eps, out16);
        else if (vpt <= 2) k_rmsnorm_v4<2><<<(unsigned)rows, threads, 0, s>>>(x, ldx, w, out, ldo, (int)n, eps, out16);
        else k_rmsnorm_v4<4><<<(unsigned)rows, threads, 0, s>>>(x, ldx, w, out, ldo, (int)n, eps, out16);
    } else {
        k_rmsnorm<<<(unsigned)rows, 256, 0, s>>>(x, ldx, w, out, ldo, (int)n, eps, out16);
    }
    HC_LAUNCH_CHECK();
    return HC_OK;
}

// ============================================================ split-K slabs + residual + RMSNorm
// hidden[row] += (part[0][row] + part[1][row] + ... + part[S-1][row]) (slab
// order, then the residual: the reference's `hidden[i] = residual[i] +
// proj[i]`, transformer.rs:561-563, 595-598), then, when w is given,
// xn[row] = RMSNorm(hidden[row]) * w and its fp16 copy in GEMM K order
// (rms_norm_fused, kernels.rs:592-625).  One CTA per row.
constexpr int RSN_MAX_SPLITS = 8;  // most slabs a projection writes (the model's kPartSplits)

template <int VPT>
__global__ void k_residual_splits_norm(const float* __restrict__ part, int splits, size_t slab, float* hidden,
                                       size_t ldh, const float* __restrict__ w, float* __restrict__ xn, size_t ldxn,
                                       __half* __restrict__ xn16, int n, float eps) {
    pdl_trigger();
    __shared__ float red[32];
    const size_t row = blockIdx.x;
    const int n4 = n / 4;
    float4* hrow = reinterpret_cast<float4*>(hidden + row * ldh);
    const float4* prow = reinterpret_cast<const float4*>(part + row * (size_t)n);
    float4 v[VPT];
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < VPT; j++) {
        const int i = threadIdx.x + j * blockDim.x;
        if (i < n4) {
            // every slab and the residual are loaded before the first add
            // (one memory round trip); the sum keeps slab order
            float4 q[RSN_MAX_SPLITS];
#pragma unroll
            for (int sp = 0; sp < RSN_MAX_SPLITS; sp++)
                if (sp < splits) q[sp] = prow[(size_t)sp * (slab / 4) + i];
            float4 r = hrow[i];
            float4 acc = q[0];
#pragma unroll
            for (int sp = 1; sp < RSN_MAX_SPLITS; sp++) {
                if (sp < splits) {
                    acc.x = acc.x + q[sp].x;
                    acc.y = acc.y + q[sp].y;
                    acc.z = acc.z + q[sp].z;
                    acc.w = acc.w + q[sp].w;
                }
            }
            r.x = acc.x + r.x;
            r.y = acc.y + r.y;
            r.z = acc.z + r.z;
            r.w = acc.w + r.w;
            hrow[i] = r;
            v[j] = r;
        } else {
            v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        ss = fmaf(v[j].x, v[j].x, ss);
        ss = fmaf(v[j].y, v[j].y, ss);
        ss = fmaf(v[j].z, v[j].z, ss);
        ss = fmaf(v[j].w, v[j].w, ss);
    }
    if (!w) return;  // uniform over the grid
    const float4* wr = reinterpret_cast<const float4*>(w);
    float4 wv[VPT];  // the norm weights travel while the block reduces
#pragma unroll
    for (int j = 0; j < VPT; j++) {
        const int i = threadIdx.x + j * blockDim.x;
        wv[j] = i < n4 ? wr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    ss = block_sum(ss, red);
    const float ms = __fdiv_rn(ss, (float)n);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
    float4* orow = reinterpret_cast<float4*>(xn + row * ldxn);
#pragma unroll
    for (int j = 0; j < VPT; j++) {
        const int i = threadIdx.x + j * blockDim.x;
        if (i < n4) {
            float4 ww = wv[j], o;
            o.x = __fmul_rn(__fmul_rn(v[j].x, inv), ww.x);
            o.y = __fmul_rn(__fmul_rn(v[j].y, inv), ww.y);
            o.z = __fmul_rn(__fmul_rn(v[j].z, inv), ww.z);
            o.w = __fmul_rn(__fmul_rn(v[j].w, inv), ww.w);
            orow[i] = o;
            if (xn16) {
                __half* r16 = xn16 + row * (size_t)(2 * n);
                store_x16(r16, n, 4 * i, o.x);
                store_x16(r16, n, 4 * i + 1, o.y);
                store_x16(r16, n, 4 * i + 2, o.z);
                store_x16(r16, n, 4 * i + 3, o.w);
            }
        }
    }
}

bool residual_splits_norm_ok(size_t n, size_t ldh, size_t ldxn) {
    return n % 4 == 0 && ldh % 4 == 0 && ldxn % 4 == 0 && n <= 2 * 1024 * 4;
}

int launch_residual_splits_norm(const float* part, int splits, size_t rows, size_t n, float* hidden, size_t ldh,
                                const float* w, float eps, float* xn, size_t ldxn, __half* xn16, cudaStream_t s) {
    if (rows == 0) return HC_OK;
    HC_CHECK(splits >= 1 && splits <= RSN_MAX_SPLITS && residual_splits_norm_ok(n, ldh, ldxn) && ((uintptr_t)part & 15) == 0 &&
                 ((uintptr_t)hidden & 15) == 0 && (!w || ((uintptr_t)w & 15) == 0) && (!w || ((uintptr_t)xn & 15) == 0),
             HC_ERR_INVALID, "residual_splits_norm: unsupported layout (n %zu)", n);
    const size_t n4 = n / 4;
    const unsigned threads = (unsigned)std::min<size_t>(1024, ((n4 + 31) / 32) * 32);
    const size_t vpt = (n4 + threads - 1) / threads;
    const size_t slab = rows * n;
    if (vpt <= 1)
        k_residual_splits_norm<1><<<(unsigned)rows, threads, 0, s>>>(part, splits, slab, hidden, ldh, w, xn, ldxn, xn16,
                                                                     (int)n, eps);
    else
        k_residual_splits_norm<2><<<(unsigned)rows, threads, 0, s>>>(part, splits, slab, hidden, ldh, w, xn, ldxn, xn16,
                                                                     (int)n, eps);
    HC_LAUNCH_CHECK();
    return HC_OK;
}

// ============================================================ softmax rows
// softmax_fast (kernels.rs:631-668), one CTA per row.
__global__ void k_softmax_rows(float* __restrict__ x, int n) {
    __shared__ float red[32];
    float* xr = x + (size_t)blockIdx.x * n;
    float mx = -INFINITY;
    for (int i = threadIdx.x; i < n; i += blockDim.x) mx = fmaxf(mx, xr[i]);
    mx = block_max(mx, red);
    int n8 = n - (n % 8);
    float sum = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float e = softmax_weight(xr[i], mx, i, n8);
        xr[i] = e;
        sum += e;
    }
    float total = block_sum(sum, red);
    float inv = __fdiv_rn(1.0f, total);
    for (int i = threadIdx.x; i < n; i += blockDim.x) xr[i] = (i < n8) ? __fmul_rn(xr[i], inv) : __fdiv_rn(xr[i], total);
}

int launch_softmax_rows(float* x, size_t rows, size_t n, cudaStream_t s) {
    if (rows == 0 || n == 0) return HC_OK;
    k_softmax_rows<<<(unsigned)rows, 256, 0, s>>>(x, (int)n);
    HC_LAUNCH_CHECK();
    return HC_OK;
}

// ============================================================ SiLU

__global__ void k_silu(float* __restrict__ x, size_t n) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] = silu_f(x[i]);
}

int launch_silu(float* x, size_t n, cudaStream_t s) {
    if (n == 0) return HC_OK;
    k_silu<<<grid_for(n, 256), 256, 0, s>>>(x, n);
    HC_LAUNCH_CHECK();
    return HC_OK;
}

// transformer.rs:446-449 / turbo.rs:235-237: silu(gate) * up.  With
// `blocked`, gate and up rows alternate in blocks of GU_BLOCK (the fused
// weight's row order): gate i sits at column (i / B) * 2B + i % B, its up at
// + B; otherwise gate i at i and up at im + i.
// With splits > 1 the gate/up product arrives as split-K slabs (slab i at
// gu + i * slab), added in slab order first.
__global__ void k_silu_mul(const float* __restrict__ gu, size_t ldgu, float* __restrict__ act, size_t ldact,
                           int im, __half* __restrict__ act16, int blocked, int splits, size_t slab) {
    pdl_trigger();
    const float* g = gu + (size_t)blockIdx.y * ldgu;
    float* a = act + (size_t)blockIdx.y * ldact;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < im; i += gridDim.x * blockDim.x) {
        const int gi = blocked ? (i / GU_BLOCK) * (2 * GU_BLOCK) + i % GU_BLOCK : i;
        const int ui = blocked ? gi + GU_BLOCK : im + i;
        float gq[RSN_MAX_SPLITS], uq[RSN_MAX_SPLITS];  // every slab requested before the first add
#pragma unroll
        for (int sp = 0; sp < RSN_MAX_SPLITS; sp++) {
            if (sp < splits) {
                gq[sp] = g[(size_t)sp * slab + gi];
                uq[sp] = g[(size_t)sp * slab + ui];
            }
        }
        float gv = gq[0], uv = uq[0];
#pragma unroll
        for (int sp = 1; sp < RSN_MAX_SPLITS; sp++) {
            if (sp < splits) {
                gv = gv + gq[sp];
                uv = uv + uq[sp];
            }
        }
        float o = __fmul_rn(silu_f(gv), uv);
        a[i] = o;
        if (act16) store_x16(act16 + (size_t)blockIdx.y * 2 * im, im, i, o);
    }
}

int launch_silu_mul(const float* gu, size_t ldgu, float* act, size_t ldact, size_t rows, size_t im,
                    cudaStream_t s, __half* act16, bool blocked, int splits) {
    if (rows == 0) return HC_OK;
    HC_CHECK(!blocked || im % GU_BLOCK == 0, HC_ERR_INVALID, "silu_mul: blocked layout needs im %% %d == 0", GU_BLOCK);
    HC_CHECK(splits >= 1 && splits <= RSN_MAX_SPLITS, HC_ERR_INVALID, "silu_mul: %d slabs", splits);
    unsigned gx = (unsigned)std::min<size_t>((im + 255) / 256, 64);
    k_silu_mul<<<dim3(gx, (unsigned)rows), 256, 0, s>>>(gu, ldgu, act, ldact, (int)im, act16, blocked ? 1 : 0, splits,
                                                        rows * ldgu);
    HC_LAUNCH_CHECK();
    return HC_OK;
}

// ============================================================ RoPE
// Adjacent-pair rotation (ops.rs:86-99, transformer.rs:317-343,
// turbo.rs:113-142) with the (cos, sin) of (pos as f32) * freq_i taken from a
// table built by the host C library; the rotation itself is done with
// separately rounded products (no fma), as in the reference.
__global__ void k_rope_rows(float* __restrict__ x, size_t ldx, int heads, int hd, const float2* __restrict__ cs,
                            int cs_rows, const int* __restrict__ pos_dev, int pos0) {
    int row = blockIdx.y;
    int pos = pos_dev ? pos_dev[row] : pos0 + row;
    if (pos < 0 || pos >= cs_rows) return;  // beyond the cache: the position is rejected elsewhere
    int half = hd / 2;
    float* xr = x + (size_t)row * ldx;
    for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < heads * half; p += gridDim.x * blockDim.x) {
        int h = p / half, i = p % half;
        float2 c = cs[(size_t)pos * half + i];
        float* e = xr + (size_t)h * hd + 2 * i;
        float a = e[0], b = e[1];
        e[0] = __fsub_rn(__fmul_rn(a, c.x), __fmul_rn(b, c.y));
        e[1] = __fadd_rn(__fmul_rn(a, c.y), __fmul_rn(b, c.x));
    }
}

int launch_rope_rows(float* x, size_t ldx, size_t rows, size_t heads, size_t hd, const float2* cs, size_t cs_rows,
                     const int* pos_dev, int pos0, cudaStream_t s) {
    if (rows == 0 || heads == 0) return HC_OK;
    size_t pairs = heads * hd / 2;
    unsigned gx = (unsigned)std::min<size_t>((pairs + 127) / 128, 64);
    k_rope_rows<<<dim3(gx, (unsigned)rows), 128, 0, s>>>(x, ldx, (int)heads, (int)hd, cs, (int)cs_rows, pos_dev,
                                                         pos0);
    HC_LAUNCH_CHECK();
    return HC_OK;
}

// The same rotation applied while adding the split-K slabs of the qkv
// projection: x[row][e] = sum over slabs (slab order) of part[i][row][e] for
// the row's `width` elements, rotated for the first `heads` heads (q and k;
// v is only summed).  Slab i starts at part + i * rows * width.  With kv.kc
// set, the row's (rotated) k and v elements are also stored into the cache
// exactly as launch_kv_store does.
template <typename KT>
__global__ void k_rope_rows_slabs(const float* __restrict__ part, int splits, size_t slab, float* __restrict__ x,
                                  size_t ldx, int width, int heads, int hd, const float2* __restrict__ cs, int cs_rows,
                                  const int* __restrict__ pos_dev, int pos0, KvStoreArgs kv) {
    pdl_trigger();
    pdl_wait();
    const int row = blockIdx.y;
    const int pos = pos_dev ? pos_dev[row] : pos0 + row;
    const bool rot_ok = pos >= 0 && pos < cs_rows;  // else the position is rejected elsewhere
    const int half = hd / 2;
    int kseq = 0, kpos = -1;
    if (kv.kc) {
        kseq = kv.seqs ? kv.seqs[row] : kv.fixed_seq;
        kpos = kv.seqs ? kv.pos[kseq] : kv.pos0 + row;
    }
    const bool store = kv.kc && kpos >= 0 && kpos < kv.max_pos;  // capacity guard of launch_kv_store
    const float2* pr = reinterpret_cast<const float2*>(part + (size_t)row * width);
    float2* xr = reinterpret_cast<float2*>(x + (size_t)row * ldx);
    for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < width / 2; p += gridDim.x * blockDim.x) {
        // every slab is loaded before the first add (one memory round trip);
        // the sum keeps slab order
        float2 q[RSN_MAX_SPLITS];
#pragma unroll
        for (int sp = 0; sp < RSN_MAX_SPLITS; sp++)
            if (sp < splits) q[sp] = pr[(size_t)sp * (slab / 2) + p];
        float2 v = q[0];
#pragma unroll
        for (int sp = 1; sp < RSN_MAX_SPLITS; sp++) {
            if (sp < splits) {
                v.x = v.x + q[sp].x;
                v.y = v.y + q[sp].y;
            }
        }
        const int h = p / half, i = p % half;
        if (h < heads && rot_ok) {
            const float2 c = cs[(size_t)pos * half + i];
            const float a = v.x, b = v.y;
            v.x = __fsub_rn(__fmul_rn(a, c.x), __fmul_rn(b, c.y));
            v.y = __fadd_rn(__fmul_rn(a, c.y), __fmul_rn(b, c.x));
        }
        xr[p] = v;
        const int e = 2 * p - kv.nq;  // element within the k (then v) block
        if (store && e >= 0) {
            const bool is_v = e >= kv.nk;
            const int ev = is_v ? e - kv.nk : e;
            const size_t off = (size_t)kseq * kv.seq_stride + (size_t)(ev / hd) * kv.head_stride + (size_t)kpos * hd +
                               (size_t)(ev % hd);
            KT* dst = reinterpret_cast<KT*>(is_v ? kv.vc : kv.kc) + off;
            if constexpr (sizeof(KT) == 2) {
                dst[0] = __float2half_rn(v.x);
                dst[1] = __float2half_rn(v.y);
            } else {
                dst[0] = v.x;
                dst[1] = v.y;
            }
        }
    }
}

int launch_rope_rows_slabs(const float* part, int splits, float* x, size_t ldx, size_t rows, size_t width,
                           size_t heads, size_t hd, const float2* cs, size_t cs_rows, const int* pos_dev, int pos0,
                           cudaStream_t s, const KvStoreArgs* kv) {
    if (rows == 0) return HC_OK;
    HC_CHECK(splits >= 1 && splits <= RSN_MAX_SPLITS && width % 2 == 0 && hd % 2 == 0 && ldx % 2 == 0 && heads * hd <= width &&
                 ((uintptr_t)part & 7) == 0 && ((uintptr_t)x & 7) == 0,
             HC_ERR_INVALID, "rope_rows_slabs: unsupported layout");
    KvStoreArgs k{};
    if (kv) {
        k = *kv;
        HC_CHECK(k.nq >= 0 && (size_t)(k.nq + 2 * k.nk) <= width && k.nq % 2 == 0 && k.nk % (int)hd == 0,
                 HC_ERR_INVALID, "rope_rows_slabs: k/v block outside the row");
    }
    const size_t pairs = width / 2;
    const unsigned gx = (unsigned)std::min<size_t>((pairs + 127) / 128, 64);
    if (kv && k.kv_fp16)
        return launch_pdl(k_rope_rows_slabs<__half>, dim3(gx, (unsigned)rows), dim3(128), 0, s, part, splits,
                          rows * width, x, ldx, (int)width, (int)heads, (int)hd, cs, (int)cs_rows, pos_dev, pos0, k);
    return launch_pdl(k_rope_rows_slabs<float>, dim3(gx, (unsigned)rows), dim3(128), 0, s, part, splits, rows * width,
                      x, ldx, (int)width, (int)heads, (int)hd, cs, (int)cs_rows, pos_dev, pos0, k);
}

// ============================================================ embedding
// transformer.rs:477-500 / turbo.rs:40-66 / quant.rs:139-153.
__global__ void k_embed(uint32_t dtype, const void* __restrict__ dense, const uint4* __restrict__ qs,
                        const __half* __restrict__ sc, const uint32_t* __restrict__ ids, float* __restrict__ out,
                        int hidden) {
    pdl_trigger();
    pdl_wait();
    int b = blockIdx.y;
    size_t id = ids[b];
    float* o = out + (size_t)b * hidden;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < hidden; i += gridDim.x * blockDim.x) {
        float v;
        if (dtype == HC_DTYPE_FP32) {
            v = reinterpret_cast<const float*>(dense)[id * hidden + i];
        } else if (dtype == HC_DTYPE_FP16) {
            v = __half2float(reinterpret_cast<const __half*>(dense)[id * hidden + i]);
        } else {
            size_t blk = id * (hidden / 32) + (i >> 5);
            int j = i & 31;
            const uint8_t* qb = reinterpret_cast<const uint8_t*>(qs + blk);
            uint8_t byte = qb[j >> 1];
            int nib = (j & 1) ? (byte >> 4) : (byte & 0xF);
            v = (float)(nib - 8) * __half2float(sc[blk]);
        }
        o[i] = v;
    }
}

int launch_embed(const DevWeight& emb, const uint32_t* ids, size_t B, float* out, size_t hidden, cudaStream_t s) {
    if (B == 0) return HC_OK;
    if (!emb.present) {
        HC_CUDA(cudaMemsetAsync(out, 0, B * hidden * sizeof(float), s));
        return HC_OK;
    }
    if (emb.dtype == HC_DTYPE_Q4_0 && hidden % 32 != 0) {
        hc_set_error("Q4_0 embedding needs hidden %% 32 == 0 (quant.rs:139-153)");
        return HC_ERR_UNSUPPORTED;
    }
    unsigned gx = (unsigned)std::min<size_t>((hidden + 255) / 256, 32);
    return launch_pdl(k_embed, dim3(gx, (unsigned)B), dim3(256), 0, s, emb.dtype, emb.dense, emb.q4.qs, emb.q4.sc, ids,
                      out, (int)hidden);
}

// ============================================================ argmax
// Greedy pick: Iterator::max_by with partial_cmp(..).unwrap_or(Equal)
// (run.rs:234-238, serve.rs:300).  The fold keeps its accumulator only while
// it is strictly greater than the next element, so the LAST maximal index
// wins, and a NaN (Equal to everything) is taken and then replaced by the
// element after it: the pick is the last maximal index after the row's last
// NaN, or that NaN's index when it ends the row.

// (best, bi) <- (ov, oi) when oi is the larger value or the same value at a
// larger index (non-NaN values; bi < 0: nothing yet)
__device__ __forceinline__ void am_take(float& best, int& bi, float ov, int oi) {
    if (oi >= 0 && (bi < 0 || ov > best || (ov == best && oi > bi))) {
        best = ov;
        bi = oi;
    }
}

// Block-wide am_take and max of nan_i; the result is in every thread.
__device__ __forceinline__ void am_reduce(float& best, int& bi, int& nan_i, float* sv, int* si, int* sn) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        am_take(best, bi, __shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, bi, o));
        nan_i = max(nan_i, __shfl_xor_sync(0xffffffffu, nan_i, o));
    }
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();  // (sv / si / sn may still be read by an earlier reduction)
    if (lane == 0) {
        sv[w] = best;
        si[w] = bi;
        sn[w] = nan_i;
    }
    __syncthreads();
    best = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : -1;
    nan_i = lane < nw ? sn[lane] : -1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        am_take(best, bi, __shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, bi, o));
        nan_i = max(nan_i, __shfl_xor_sync(0xffffffffu, nan_i, o));
    }
}

// One CTA per row of n logits (row stride ld): out[row] = the pick; with
// pairs, pairs[row] = (its value, bits of idx0 + pick, bit 31 set when the
// row held a NaN; all bits set for an empty row) for the vocabulary-sharded
// exchange of tensor parallelism (k_pick_pairs).
__global__ void k_argmax(const float* __restrict__ logits, int n, size_t ld, uint32_t* __restrict__ out,
                         float2* __restrict__ pairs = nullptr, uint32_t idx0 = 0) {
    pdl_trigger();
    pdl_wait();
    __shared__ float sv[32];
    __shared__ int si[32], sn[32];
    const float* l = logits + (size_t)blockIdx.x * ld;
    float best = -INFINITY;
    int bi = -1, nan_i = -1;
    // Each thread visits its indices in increasing order, so ">=" keeps its
    // last maximum and nan_i its last NaN; the reductions break ties toward
    // the larger index.
    auto visit = [&](float e, int i) {
        if (e != e)
            nan_i = i;
        else if (bi < 0 || e >= best) {
            best = e;
            bi = i;
        }
    };
    if ((n & 3) == 0 && ((uintptr_t)l & 15) == 0) {
        constexpr int U = 4;  // float4 loads in flight per thread
        const float4* l4 = reinterpret_cast<const float4*>(l);
        const int n4 = n >> 2;
        for (int i0 = threadIdx.x; i0 < n4; i0 += U * blockDim.x) {
            float4 v[U];
#pragma unroll
            for (int u = 0; u < U; u++) {
                int i = i0 + u * blockDim.x;
                if (i < n4) v[u] = __ldg(l4 + i);
            }
#pragma unroll
            for (int u = 0; u < U; u++) {
                int i = i0 + u * blockDim.x;
                if (i < n4) {
                    visit(v[u].x, 4 * i);
                    visit(v[u].y, 4 * i + 1);
                    visit(v[u].z, 4 * i + 2);
                    visit(v[u].w, 4 * i + 3);
                }
            }
        }
    } else {
        for (int i = threadIdx.x; i < n; i += blockDim.x) visit(l[i], i);
    }
    am_reduce(best, bi, nan_i, sv, si, sn);
    const int last_nan = nan_i;
    if (last_nan >= 0) {  // rare: the last maximum after the last NaN
        best = -INFINITY;
        bi = -1;
        nan_i = -1;
        for (int i = last_nan + 1 + threadIdx.x; i < n; i += blockDim.x) visit(l[i], i);
        am_reduce(best, bi, nan_i, sv, si, sn);
        if (bi < 0) {  // the NaN ends the row
            bi = last_nan;
            best = l[last_nan];
        }
    }
    if (threadIdx.x == 0) {
        if (pairs)
            pairs[blockIdx.x] = make_float2(
                best, __uint_as_float(bi < 0 ? 0xFFFFFFFFu : (idx0 + (uint32_t)bi) | (last_nan >= 0 ? 0x80000000u : 0u)));
        else
            out[blockIdx.x] = (uint32_t)(bi < 0 ? 0 : bi);
    }
}

// Greedy ids from the shards' pairs ([tp][rows], shard order = vocabulary
// order): the fold of max_by over the shards' picks, restarted at a shard
// that held a NaN (everything before its last NaN is irrelevant); 0 for no
// logits.
__global__ void k_pick_pairs(const float2* __restrict__ pairs, int rows, int tp, uint32_t* __restrict__ out) {
    pdl_trigger();
    pdl_wait();
    const int row = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= rows) return;
    float best = 0.0f;
    int bi = -1;
    for (int r = 0; r < tp; r++) {
        const float2 p = pairs[(size_t)r * rows + row];
        const uint32_t bits = __float_as_uint(p.y);
        if (bits == 0xFFFFFFFFu) continue;  // an empty shard
        const int oi = (int)(bits & 0x7FFFFFFFu);
        // a shard with a NaN restarts the fold; otherwise its pick (the last
        // maximum of NaN-free logits) replaces the accumulator unless that is
        // strictly greater (a NaN accumulator is replaced)
        if ((bits >> 31) || bi < 0 || !(best > p.x)) {
            best = p.x;
            bi = oi;
        }
    }
    out[row] = (uint32_t)(bi < 0 ? 0 : bi);
}

int launch_argmax_pairs(const float* logits, size_t rows, size_t n, size_t ld, uint32_t idx0, float2* pairs,
                        cudaStream_t s) {
    if (rows == 0) return HC_OK;
    return launch_pdl(k_argmax, dim3((unsigned)rows), dim3(1024), 0, s, logits, (int)n, ld, (uint32_t*)nullptr, pairs,
                      idx0);
}

int launch_pick_pairs(const float2* pairs, size_t rows, int tp, uint32_t* out, cudaStream_t s) {
    if (rows == 0) return HC_OK;
    return launch_pdl(k_pick_pairs, dim3((unsigned)((rows + 127) / 128)), dim3(128), 0, s, pairs, (int)rows, tp, out);
}

int launch_argmax(const float* logits, size_t rows, size_t n, size_t ld, uint32_t* out, cudaStream_t s) {
    if (rows == 0) return HC_OK;
    return launch_pdl(k_argmax, dim3((unsigned)rows), dim3(1024), 0, s, logits, (int)n, ld, out, (float2*)nullptr,
                      (uint32_t)0);
}

int launch_argmax(const float* logits, size_t rows, size_t n, uint32_t* out, cudaStream_t s) {
    return launch_argmax(logits, rows, n, n, out, s);
}

// ============================================================ synthetic data
__global__ void k_synth_normal(uint64_t key, uint64_t offset, uint64_t n, float scale, float* __restrict__ out) {
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (; i < n; i += stride) out[i] = synth_normal(key, offset + i, scale);
}

int launch_synth_normal(uint64_t seed, uint64_t stream, uint64_t offset, uint64_t n, float std, float* out,
                        cudaStream_t s) {
    if (n == 0) return HC_OK;
    uint64_t key = synth_key(seed, stream);
    float scale = std / 65536.0f;
    unsigned grid = (unsigned)std::min<uint64_t>((n + 255) / 256, 148ull * 16);
    k_synth_normal<<<grid, 256, 0, s>>>(key, offset, n, scale, out);
    HC_LAUNCH_CHECK();
    return HC_OK;
}

}  // namespace hc
