// Tensor-core Q4_0 GEMM for sm_100a (tcgen05 + TMEM + TMA).
//
//   Y[t][n] (+)= sum_k X[t][k] * deq(W)[n][k]      (t < T tokens, n < N rows)
//
// It is the prefill projection of turbo::batch_matmul (turbo.rs:306-343) and
// the batched decode matvec of kernels::matmul_q4_0 (kernels.rs:256-359) when
// several tokens share the weights.  The MMA is issued "swap-AB": the weight
// tile is the M = 128 side and the tokens are the N side, so one CTA tile is
// 128 weight rows x TN tokens.
//
//   TMA (warps 0, 2)  the Q4_0 nibble tile of 128 rows x 128 K and its scales
//                     -> weight ring; X tile (fp16, K-major, 128B swizzle)
//                     -> X ring
//   dequant (warps 4-19 for prefill tiles, 4-11 for decode tiles; one
//                     weight row per thread) nibbles -> (nib - 8) * scale in
//                     fp16 -> tcgen05.st into tensor memory (the A operand
//                     never touches shared memory, so shared-memory bandwidth
//                     is left to the TMA traffic and the B operand)
//   MMA (warp 1, and warp 3 for decode tiles)  tcgen05.mma.kind::f16, A from
//                     TMEM, B from the smem descriptor, f32 accumulator in
//                     TMEM; tcgen05.commit frees the X stage and the A slot
//   epilogue (warps 4-7)  tcgen05.ld of the accumulator -> Y (+ residual);
//                     with split K, the CTAs of a tile (one cluster) add their
//                     partial tiles in split order over distributed shared memory
//
// Every TMA load writes only the issuing CTA's own shared memory (the same
// code runs under tensor parallelism on several GPUs; split-K clusters share
// partial tiles through distributed shared memory loads, never through TMA).
// Every mbarrier wait is bounded by a clock
// deadline; on expiry the kernel records an error flag, skips its stores, and
// still frees its tensor memory before returning.
#include "hc_gemm.h"
#include "hc_tc.cuh"

#include <cudaTypedefs.h>

#include <mutex>
#include <map>
#include <tuple>

namespace hc {

namespace {

constexpr int BM = 128;      // weight rows per tile (MMA M)
constexpr int BK = 128;      // K per pipeline stage
// Instruction descriptor: f16 x f16 -> f32, A and B K-major, M = 128, N = tn.
__host__ __device__ constexpr uint32_t make_idesc(int tn) { return make_idesc_mn(BM, tn); }

constexpr int EPI_CH = 16;     // tokens per epilogue chunk (one tcgen05.ld x16)
constexpr int MAX_SPLITS = 8;  // split-K cluster size limit (portable cluster size)

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}


// Store v at shared-memory offset `local` (this CTA's address of it) in the
// CTA of the cluster with the given rank.
__device__ __forceinline__ void st_dsmem_f32(uint32_t local, int rank, float v) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(rank));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
}

// y[jj * ldy] = v[jj] (+ res[jj * ldres]) for jj < tl, one column of an
// EPI_CH-token chunk.  The residuals are all loaded before the first store
// (res may alias y element for element, so plain coherent loads are used).
__device__ __forceinline__ void store_chunk(float* y, size_t ldy, const uint32_t* v, int tl, const float* res,
                                            size_t ldres) {
    float r[EPI_CH];
#pragma unroll
    for (int jj = 0; jj < EPI_CH; jj++) r[jj] = (res && jj < tl) ? res[(size_t)jj * ldres] : 0.0f;
#pragma unroll
    for (int jj = 0; jj < EPI_CH; jj++) {
        if (jj < tl) {
            float o = __uint_as_float(v[jj]);
            if (res) o = o + r[jj];
            y[(size_t)jj * ldy] = o;
        }
    }
}

// K order inside a 32-element Q4_0 block.  Word i (4 bytes = elements
// 8i..8i+7, low nibble first) yields four fp16 pairs: pair k = (element
// 8i+k, element 8i+k+4), i.e. bits [4k, 4k+4) and [16+4k, 16+4k+4).  The A
// operand (the weights) is therefore laid out along K in the order
//   position 8i+2k <- element 8i+k,   position 8i+2k+1 <- element 8i+k+4,
// and the B operand (the activations) is written in the same order by
// k_rows_to_f16_perm, so every dot product sees matching pairs.
// Pairs 0 and 2 (the low nibble of a byte pair) become (nib + 1024) with one
// and/or, exact in fp16 (0x6400 | nib), minus 1032; pairs 1 and 3 are taken
// in place as (16 nib + 1024) and turned into nib - 8 by one fma with 1/16
// and -72, both exact.  One shift serves the word's upper bytes.
//
// The weight (nib - 8) * scale (the reference dequantizes in f32,
// quant.rs:25-34) needs up to 14 significant bits, more than fp16 holds, so
// it enters the MMAs as two exact fp16 terms: scale = s_hi + s_lo, s_hi the
// scale with the 3 low mantissa bits cleared (8 significant bits) and s_lo
// the rest (3 bits); |nib - 8| <= 8 has at most 3 significant bits, so
// (nib - 8) * s_hi (<= 11 bits) and (nib - 8) * s_lo (<= 6 bits) are both
// exact fp16 products, and their sum is the f32 weight.
__device__ __forceinline__ void split_scale(uint32_t s16, __half2& shi2, __half2& slo2) {
    const bool special = (s16 & 0x7C00u) == 0x7C00u;  // inf / NaN scale: kept whole, lo = 0
    const __half s = __ushort_as_half((unsigned short)s16);
    const __half sh = __ushort_as_half((unsigned short)(special ? s16 : (s16 & 0xFFF8u)));
    const __half sl = special ? __ushort_as_half((unsigned short)0) : __hsub(s, sh);  // exact
    shi2 = __half2half2(sh);
    slo2 = __half2half2(sl);
}

// The (hi, lo) weight pairs of one Q4_0 word: hi[k] = (nib - 8) * s_hi,
// lo[k] = (nib - 8) * s_lo for the four pairs of the word (see above).
__device__ __forceinline__ void deq_word_split(uint32_t w, __half2 shi2, __half2 slo2, uint32_t* hi_out,
                                               uint32_t* lo_out) {
    const uint32_t up = w >> 8;
    uint32_t v[4] = {(w & 0x000F000Fu) | 0x64006400u, (w & 0x00F000F0u) | 0x64006400u,
                     (up & 0x000F000Fu) | 0x64006400u, (up & 0x00F000F0u) | 0x64006400u};
#pragma unroll
    for (int k = 0; k < 4; k++) {
        __half2 h = *reinterpret_cast<__half2*>(&v[k]);
        h = (k & 1) ? __hfma2(h, __float2half2_rn(0.0625f), __float2half2_rn(-72.0f))
                    : __hsub2(h, __float2half2_rn(1032.0f));
        __half2 a = __hmul2(h, shi2), b = __hmul2(h, slo2);
        hi_out[k] = *reinterpret_cast<uint32_t*>(&a);
        lo_out[k] = *reinterpret_cast<uint32_t*>(&b);
    }
}

// Pipeline shapes.  Every tile is 128 weight rows x TN tokens (TN = 32, 64
// or 128) on one CTA per SM that owns all 512 tensor-memory columns.  The
// MMA's B operand is 2 TN rows, the fp16 hi rows of the tile's tokens and
// then their lo rows, so one instruction w_hi x [x_hi; x_lo] (N = 2 TN) and
// one w_lo x x_hi (N = TN) per 16-wide K step give every product the f32
// path needs (w_lo x x_lo is below 2^-20 of the result); the epilogue adds
// the accumulator's two column halves.  Decode tiles (TN = 32) are bound by
// the rate at which one thread can issue MMAs (every barrier wait, tcgen05
// fence and commit holds the issuing thread for hundreds of cycles), so two
// warps issue alternate stages, each into its own accumulator.
//
// Shared memory holds two rings.  The weight ring (nibble tile + scale box,
// S_W stages) is released by the dequant warps as soon as they have read a
// stage, so its depth is spent on DRAM latency alone; the X ring (S_X
// stages) is released by the MMA commit.  Tensor memory holds S_TM A slots of
// 128 columns (the hi weights of a 128-K stage, then its lo weights); S_TM
// divides S_X, so the commit that frees X stage j % S_X also frees A slot
// j % S_TM.
//
// Stream-K (SK, decode tiles of 32 tokens): a grid of G <= #SM CTAs, each
// taking an equal run of the (tile, stage) units [c U / G, (c + 1) U / G),
// U = tiles x stages per tile, instead of one tile per CTA: no second wave
// of CTAs when the tiles do not divide over the SMs.  A CTA's run falls into
// pieces, one per tile it touches; the stage counter j runs on across the
// pieces, so the rings and their barrier phases are those of one long tile.
// A fourth warpgroup drains the accumulators after every piece (the
// issuers wait for it before the next piece's first MMA).  The piece that
// holds a tile's first stage owns the tile: the CTAs holding its other
// pieces (their first, or only, piece) store their partial sums in a
// workspace slot and raise a per-warp flag, and the owner adds them in K
// order before its usual epilogue.
template <int TN, bool SK = false>
struct Cfg {
    static constexpr int TN_ = TN;
    static constexpr int NB = 2 * TN;                        // B rows of an MMA: hi tokens, then lo tokens
    static constexpr int COLS = 512;                         // tensor-memory columns (one CTA per SM)
    static constexpr int DEQ_WARPS = 16;
    static constexpr int EPI_WARP0 = 4 + DEQ_WARPS;          // SK: the epilogue warpgroup
    static constexpr int THREADS = 128 + 32 * DEQ_WARPS + (SK ? 128 : 0);
    static constexpr int MIN_BLOCKS = 1;
    static constexpr int X_STAGE = 2 * NB * 128;             // two 64-element K halves, 128 B per B row
    static constexpr int W_STAGE = BM * (BK / 2);            // 128 rows x 64 nibble bytes
    // fp16 block scales of the stage's 128 rows: the aligned 16-byte box of
    // 8 scales (this stage's 4 and its pair's) per row
    static constexpr int S_STAGE = BM * 16;
    static constexpr int S_X = TN <= 32 ? 6 : (TN <= 64 ? 4 : 2);  // X ring stages
    static constexpr int S_W = TN <= 64 ? 6 : 4;                    // weight ring stages
    // Issuing warps.  A warp's instructions after a batch of MMAs wait for
    // those MMAs to drain through the tensor pipe, so decode tiles (TN = 32,
    // short MMAs) use two issuing warps that take alternate stages, each into
    // its own accumulator D_i (summed by the epilogue): one warp's barrier
    // waits overlap the other's MMAs.  With one issuer and TN = 64 the
    // lo-weight products go to their own accumulator D_lo (TN columns after
    // D), so consecutive MMAs never wait on each other's accumulator; with
    // 128-token tiles every MMA is long enough for one accumulator.
    static constexpr int ISS = TN <= 32 ? 2 : 1;
    static constexpr bool DUALD = ISS == 1 && TN <= 64;
    static constexpr int D_COLS = NB + (DUALD ? TN : 0);       // per issuer
    static constexpr int A_COL = ISS * D_COLS <= 128 ? 128 : 256;  // D_i at [i D_COLS, ...); A slots from here
    static constexpr int A_SLOT = 128;                       // hi weights (64 columns), then lo weights
    static constexpr int S_TM = (COLS - A_COL) / A_SLOT;     // A slots
    static constexpr int MMA_BATCH = S_TM < 4 ? S_TM : 4;    // stages issued under one wait + fence
    // Two dequant groups take alternate stages (matching the two issuers'
    // stage parity), so one group's waits overlap the other's conversion;
    // each converts its whole share of a stage before it waits for the A slot,
    // so only the tensor-memory stores sit inside the slot's reuse cycle.
    static constexpr int RR = 2;                             // dequant groups working on different stages
    static constexpr int WG_PER = (DEQ_WARPS / 4) / RR;      // warpgroups per group, each 4 / WG_PER blocks
    // the dequant warps wait for the weight stage before the A slot (the
    // stage S_W back was this group's own, S_W % RR == 0)
    static constexpr bool PRELOAD = true;
    __host__ __device__ static constexpr int x_off(int s) { return s * X_STAGE; }
    __host__ __device__ static constexpr int w_off(int s) { return S_X * X_STAGE + s * W_STAGE; }
    __host__ __device__ static constexpr int s_off(int s) { return S_X * X_STAGE + S_W * W_STAGE + s * S_STAGE; }
    __host__ __device__ static constexpr int ring_bytes() { return S_X * X_STAGE + S_W * (W_STAGE + S_STAGE); }
    // SK: the epilogue's accumulator tile ([TN][BM] f32), apart from the busy rings
    static constexpr int XB_BYTES = SK ? TN * BM * 4 : 0;
    // SK register split (setmaxnreg): the launch gives every thread 80
    // registers (768 threads); the producer / issuer warpgroup and the
    // epilogue warpgroup hand theirs down so the four dequant warpgroups run
    // with as many as the 640-thread kernel: 128 x 48 + 128 x 48 + 512 x 96
    // = 768 x 80.
    static constexpr int REG_LAUNCH = 80, REG_CTRL = 48, REG_EPI = 48, REG_DEQ = 96;
    static_assert(!SK || 128 * REG_CTRL + 128 * REG_EPI + 32 * DEQ_WARPS * REG_DEQ <= THREADS * REG_LAUNCH,
                  "register split above the launch's registers");
    __host__ __device__ static constexpr int xb_off() { return ring_bytes(); }
    __host__ __device__ static constexpr int bar_off() { return ring_bytes() + XB_BYTES; }
    static constexpr int NBARS = 2 * S_W + 2 * S_X + S_TM + 1 + (SK ? 1 : 0);
    __host__ __device__ static constexpr int smem() { return bar_off() + NBARS * 8 + 16 + 1024; }
    static_assert(NB <= 256 && NB % 16 == 0, "MMA N of a 128-row tile");
    static_assert(S_TM >= 2 && A_COL + A_SLOT * S_TM <= COLS, "tensor memory budget");
    static_assert(ISS == 1 || ISS == 2, "one or two issuing warps");
    static_assert(MMA_BATCH >= 1 && MMA_BATCH <= S_TM, "batched stages each need their own A slot");
    // two issuers: issuer i takes the stages j % 2 == i; the phase arguments
    // of the issuer need the X ring to respect the stage parity
    static_assert(ISS == 1 || (S_X % 2 == 0 && S_W % S_TM == 0), "alternating issuers");
    static_assert(S_X % S_TM == 0, "an A slot is freed by the MMA commit that frees an X stage");
    static_assert(RR <= S_TM && RR <= S_W, "dequant groups must not run more than one barrier phase apart");
    static_assert(S_W >= S_TM && RR <= S_X && (ISS == 1 || S_W % S_TM == 0), "barrier phase ordering (see the dequant warps)");
    static_assert(WG_PER == 1 || WG_PER == 2 || WG_PER == 4, "dequant split: 4, 2 or 1 blocks per warpgroup");
    static_assert(!PRELOAD || S_W % RR == 0, "weight-first waits (see the dequant warps)");
    static_assert(!SK || (ISS == 2 && TN == 32), "stream-K runs decode tiles (two issuers)");
    static_assert(smem() <= 232448, "shared memory budget");
    static_assert((TN * 128) % 1024 == 0, "each X box starts on a 1024-byte swizzle atom");
    static constexpr int RED_PITCH = TN + 1;                  // floats per row of the split-K partial tiles
    static_assert((BM + MAX_SPLITS) * RED_PITCH * 4 <= ring_bytes(), "split-K partials fit in the rings");
};

// Tokens [c0, c0 + EPI_CH) of TMEM lane quarter q of the accumulator: the
// sum of its hi-token and lo-token column halves, of D_lo (the lo-weight
// products) when it has its own columns, and of D_1 when a second issuer
// wrote it.  Warp-collective.
template <typename C>
__device__ __forceinline__ void load_accumulators(uint32_t tmem, int q, int c0, int nk, uint32_t* v) {
    const uint32_t base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0;
    uint32_t a[EPI_CH], b[EPI_CH];
    tmem_ld_x16(base, v);
    tmem_ld_x16(base + (uint32_t)C::TN_, a);
    if (C::DUALD) tmem_ld_x16(base + (uint32_t)C::NB, b);
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int jj = 0; jj < EPI_CH; jj++) {
        float o = __uint_as_float(v[jj]) + __uint_as_float(a[jj]);
        if (C::DUALD) o = o + __uint_as_float(b[jj]);
        v[jj] = __float_as_uint(o);
    }
    if (C::ISS == 2 && nk > 1) {  // issuer 1 wrote D_1
        tmem_ld_x16(base + (uint32_t)C::D_COLS, a);
        tmem_ld_x16(base + (uint32_t)(C::D_COLS + C::TN_), b);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int jj = 0; jj < EPI_CH; jj++)
            v[jj] = __float_as_uint(__uint_as_float(v[jj]) + (__uint_as_float(a[jj]) + __uint_as_float(b[jj])));
    }
}

// Stream-K flags (one per contributing CTA and TMEM lane quarter): the whole
// warp polls with acquire loads, bounded like the barrier waits.
__device__ __forceinline__ bool sk_flag_wait(const int* flag, volatile int* abort_flag) {
    const long long start = clock64();
    for (uint32_t i = 0;; i++) {
        int v;
        asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
        if (__all_sync(0xffffffffu, v != 0)) return true;
        __nanosleep(128);
        if ((i & 63) == 63) {
            if (*abort_flag || clock64() - start > WAIT_CYCLES) {
                *abort_flag = 1;
                return false;
            }
        }
    }
}

__device__ __forceinline__ void sk_flag_set(int* flag, int v) {
    asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(flag), "r"(v) : "memory");
}

template <int TN, bool SK = false>
__global__ void __launch_bounds__(Cfg<TN, SK>::THREADS, Cfg<TN, SK>::MIN_BLOCKS)
    k_q4_gemm_tc(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                 const __grid_constant__ CUtensorMap smap, float* __restrict__ y, size_t ldy, const float* res, size_t ldres,
                 int epi, int N, int K, int T, int splits, size_t split_stride, __half* __restrict__ y16,
                 int* __restrict__ err, float* __restrict__ sk_part, int* __restrict__ sk_flag) {
    using C = Cfg<TN, SK>;
    constexpr int S_X = C::S_X, S_W = C::S_W, S_TM = C::S_TM;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* wfull = reinterpret_cast<uint64_t*>(smem + C::bar_off());  // [S_W] weight stage landed
    uint64_t* wempty = wfull + S_W;                                      // [S_W] weight stage read by dequant
    uint64_t* xfull = wempty + S_W;                                      // [S_X] X stage landed
    uint64_t* mdone = xfull + S_X;                                       // [S_X] MMAs of the stage done
    uint64_t* aready = mdone + S_X;                                      // [S_TM] A slot written
    uint64_t* dfull = aready + S_TM;                                     // accumulators complete (per SK piece)
    uint64_t* dempty = dfull + 1;                                        // SK: accumulators drained
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dfull + 1 + (SK ? 1 : 0));
    __shared__ int abort_flag;
    bool epi_ok = false;  // epilogue warpgroup: the accumulators are complete

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BM, t0 = blockIdx.y * TN, split = blockIdx.z;
    const int nk_all = K / BK;
    const int it0 = (int)((long long)nk_all * split / splits), it1 = (int)((long long)nk_all * (split + 1) / splits);
    // SK: this CTA's run [sk_b, sk_e) of the sk_u (tile, stage) units
    // (the host keeps sk_u x gridDim.x below 2^31)
    int sk_b = 0, sk_e = 0, sk_u = 0;
    if constexpr (SK) {
        sk_u = ((N + BM - 1) / BM) * nk_all;
        sk_b = (int)blockIdx.x * sk_u / (int)gridDim.x;
        sk_e = ((int)blockIdx.x + 1) * sk_u / (int)gridDim.x;
    }
    const int nk = SK ? sk_e - sk_b : it1 - it0;
    // first weight row and K stage of stage j
    auto stage_at = [&](int j, int& row0, int& kst) {
        if constexpr (SK) {
            const int u = sk_b + j;
            const int tile = u / nk_all;
            row0 = tile * BM;
            kst = u - tile * nk_all;
        } else {
            row0 = n0;
            kst = it0 + j;
        }
    };

    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int st = 0; st < S_W; st++) {
            mbar_init(&wfull[st], 1);
            mbar_init(&wempty[st], 4 * C::WG_PER);  // the warps of the converting group
        }
        for (int st = 0; st < S_X; st++) {
            mbar_init(&xfull[st], 1);
            mbar_init(&mdone[st], 1);  // the commit of the stage's issuer
        }
        for (int a = 0; a < S_TM; a++) mbar_init(&aready[a], 4 * C::WG_PER);
        mbar_init(dfull, C::ISS);
        if (SK) mbar_init(dempty, 4);  // the epilogue warps
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 2) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(C::COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    const uint32_t tmem = *tmem_slot;

    // Stage j (k range it0 + j) lives in weight stage j % S_W, X stage
    // j % S_X and tensor-memory A slot j % S_TM.  Phase parities below are
    // those of the j-th use of each barrier; every wait is at most one phase
    // away from the phase it observes (see the dequant note), which is what
    // parity waits require.
    // Roles by warpgroup (an SK register split applies to whole warpgroups
    // and must dominate only their code): warps 0-3 produce and issue,
    // 4 .. EPI_WARP0-1 dequantize, the SK epilogue warpgroup drains.
    if (warp < 4) {
        if constexpr (SK) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(C::REG_CTRL));
        if (warp == 0) {
            // ---------------- weight producer.  The weights do not depend on the
            // previous kernel, so (launched as a programmatic dependent) this CTA
            // streams them while the kernel producing X may still be running.
            if (lane == 0) {
                for (int j = 0; j < nk; j++) {
                    const int st = j % S_W;
                    if (j >= S_W && !mbar_wait(&wempty[st], ((uint32_t)(j / S_W) & 1u) ^ 1u, &abort_flag, 64)) break;
                    int row0, kst;
                    stage_at(j, row0, kst);
                    mbar_expect_tx(&wfull[st], (uint32_t)(C::W_STAGE + C::S_STAGE));
                    tma_load_2d(smem + C::w_off(st), &wmap, &wfull[st], kst * BK / 2, row0);
                    tma_load_2d(smem + C::s_off(st), &smap, &wfull[st], 8 * (kst >> 1), row0);
                }
            }
        } else if (warp == 2) {
            // ---------------- X producer (after the grid dependency)
            if (lane == 0) {
                grid_dependency_wait();
                for (int j = 0; j < nk; j++) {
                    const int st = j % S_X;
                    if (j >= S_X && !mbar_wait(&mdone[st], ((uint32_t)(j / S_X) & 1u) ^ 1u, &abort_flag, 64)) break;
                    mbar_expect_tx(&xfull[st], (uint32_t)C::X_STAGE);
                    uint8_t* xs = smem + C::x_off(st);
                    int row0, kst;
                    stage_at(j, row0, kst);
                    const int kk = kst * BK;
                    // K half h of the stage holds NB rows: the tile's hi rows
                    // (columns [0, K) of the activation rows), then its lo rows
                    // (columns [K, 2K)); rows past the last token read as zeros
    #pragma unroll
                    for (int h = 0; h < 2; h++)
    #pragma unroll
                        for (int p = 0; p < 2; p++)
                            tma_load_2d(xs + (h * C::NB + p * TN) * 128, &xmap, &xfull[st], p * K + kk + 64 * h, t0);
                }
            }
        } else if (warp == 1 || (C::ISS == 2 && warp == 3)) {
            // ---------------- MMA issuer(s): the whole warp runs the loop and its
            // waits; one elected lane issues each batch of MMAs (a converged issue
            // keeps the operands in uniform registers: ~40 cycles per MMA instead
            // of ~110 from a lone lane).  Issuer i takes the stages j = i, i + ISS,
            // ... into its accumulator D_i.  A single issuer takes every stage that
            // is already dequantized (and whose X has landed) when the oldest one
            // is, up to MMA_BATCH, under one wait + fence.  Per 16-wide K step:
            // hi weights x [x_hi; x_lo] into D_i, lo weights x x_hi into D_lo (or
            // into D_i's hi-token half).
            // Phases: an issuer's aready / xfull wait for stage j must find the
            // barrier's previous phase (stage j - S_TM, resp. j - S_X) complete.
            // With one issuer that stage was its own.  With two, stage j - S_X
            // (S_X even) is its own; stage j - S_TM may be the other issuer's, so
            // the issuer first waits for that stage's MMAs (mdone), which follow
            // its aready.  The next phases need this issuer's MMA of stage j.
            constexpr uint32_t idesc_hi = make_idesc(C::NB);  // hi weights x (hi, lo) tokens
            constexpr uint32_t idesc_lo = make_idesc(TN);     // lo weights x hi tokens
            constexpr int KSTEPS = BK / 16;
            const int iss = warp == 1 ? 0 : 1;
            const uint32_t d_hi = tmem + (uint32_t)(iss * C::D_COLS);
            const uint32_t d_lo = d_hi + (uint32_t)(C::DUALD ? C::NB : 0);
            bool ok = true;
            if constexpr (SK) {
                // one piece per tile of the run: the issuer's stages of the piece
                // (every other one, from its first, jf) accumulate from zero;
                // before a piece's first MMA the epilogue has read the last one
                const int tb = sk_b / nk_all, te = (sk_e - 1) / nk_all;
                for (int tp = tb; tp <= te && ok; tp++) {
                    const int p = tp - tb;
                    const int ps = max(sk_b, tp * nk_all) - sk_b;
                    const int pe = min(sk_e, (tp + 1) * nk_all) - sk_b;
                    if (p > 0 && !warp_wait(dempty, (uint32_t)(p - 1) & 1u, &abort_flag)) {
                        ok = false;
                        break;
                    }
                    const int jf = ps + ((ps ^ iss) & 1);
                    for (int j = jf; j < pe; j += 2) {
                        if (((S_TM & 1) && j >= S_TM &&
                             !warp_wait(&mdone[(j - S_TM) % S_X], (uint32_t)((j - S_TM) / S_X) & 1u, &abort_flag)) ||
                            !warp_wait(&xfull[j % S_X], (uint32_t)(j / S_X) & 1u, &abort_flag) ||
                            !warp_wait(&aready[j % S_TM], (uint32_t)(j / S_TM) & 1u, &abort_flag)) {
                            ok = false;
                            break;
                        }
                        __syncwarp();
                        tmem_fence_after();
                        if (elect_one()) {
                            const int st = j % S_X, a = j % S_TM;
                            const uint32_t xs = smem_u32(smem + C::x_off(st));
    #pragma unroll
                            for (int kk = 0; kk < KSTEPS; kk++) {
                                const uint32_t a_tmem = tmem + (uint32_t)(C::A_COL + a * C::A_SLOT + kk * 8);
                                const uint64_t bd = sw128_desc(xs + (uint32_t)((kk >> 2) * C::NB * 128 + (kk & 3) * 32));
                                const uint32_t acc = (j > jf || kk > 0) ? 1u : 0u;
                                mma_f16_ts(d_hi, a_tmem, bd, idesc_hi, acc);
                                mma_f16_ts(d_lo, a_tmem + 64u, bd, idesc_lo, 1u);
                            }
                            mma_commit(&mdone[st]);
                        }
                        __syncwarp();
                    }
                    if (ok && elect_one()) mma_commit(dfull);  // also when the piece had no stage of this issuer
                    __syncwarp();
                }
            } else
            for (int j = iss; j < nk;) {
                if ((C::ISS == 2 && (S_TM & 1) && j >= S_TM &&
                     !warp_wait(&mdone[(j - S_TM) % S_X], (uint32_t)((j - S_TM) / S_X) & 1u, &abort_flag)) ||
                    !warp_wait(&xfull[j % S_X], (uint32_t)(j / S_X) & 1u, &abort_flag) ||
                    !warp_wait(&aready[j % S_TM], (uint32_t)(j / S_TM) & 1u, &abort_flag)) {
                    ok = false;
                    break;
                }
                int cnt = 1;
                if (C::ISS == 1 && lane == 0) {
                    while (cnt < C::MMA_BATCH && j + cnt < nk &&
                           mbar_test_wait(&aready[(j + cnt) % S_TM], (uint32_t)((j + cnt) / S_TM) & 1u) &&
                           mbar_test_wait(&xfull[(j + cnt) % S_X], (uint32_t)((j + cnt) / S_X) & 1u))
                        cnt++;
                }
                cnt = __shfl_sync(0xffffffffu, cnt, 0);
                __syncwarp();
                tmem_fence_after();
                if (elect_one()) {
                    for (int b = 0; b < cnt; b++) {
                        const int jj = j + b * C::ISS, st = jj % S_X, a = jj % S_TM;
                        const uint32_t xs = smem_u32(smem + C::x_off(st));
    #pragma unroll
                        for (int kk = 0; kk < KSTEPS; kk++) {
                            const uint32_t a_tmem = tmem + (uint32_t)(C::A_COL + a * C::A_SLOT + kk * 8);
                            const uint64_t bd = sw128_desc(xs + (uint32_t)((kk >> 2) * C::NB * 128 + (kk & 3) * 32));
                            const uint32_t first = (jj > iss || kk > 0) ? 1u : 0u;
                            mma_f16_ts(d_hi, a_tmem, bd, idesc_hi, first);
                            mma_f16_ts(d_lo, a_tmem + 64u, bd, idesc_lo, C::DUALD ? first : 1u);
                        }
                        mma_commit(&mdone[st]);  // frees the X stage and (S_TM | S_X) the A slot
                    }
                }
                __syncwarp();
                j += cnt * C::ISS;
            }
            if (!SK && ok && elect_one()) mma_commit(dfull);  // also when this issuer had no stage
            __syncwarp();
        }
    } else if (warp < C::EPI_WARP0) {
        if constexpr (SK) asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(C::REG_DEQ));
        // ---------------- dequant: thread <-> weight row (TMEM lane).  The
        // dequant warpgroups form RR groups; group g converts the stages j
        // with j % RR == g (each of its WG_PER warpgroups 4 / WG_PER of the
        // stage's Q4_0 blocks), so RR stages are in flight at once.  Parity
        // waits cannot tell phases two apart, so each wait below must find its
        // barrier in the awaited phase or the one after it:
        // The dequant of stage j needs the MMA of j - S_TM, which needs the
        // dequant of j - S_TM: the dequant of j follows that of every stage
        // j - m S_TM.
        //  * mdone of stage j - S_TM: its previous phase (stage j - S_TM - S_X)
        //    completed before this group finished stage j - RR: that stage
        //    waited for the MMA of j - RR - S_TM, which the same issuer (one
        //    issuer, or S_X - RR even) issued after the earlier one;
        //    its next phase is the MMA of stage j - S_TM + S_X, which (S_TM
        //    divides S_X) follows the dequant of j.
        //  * wfull of stage j: with PRELOAD, stage j - S_W was this group's
        //    own (S_W % RR == 0) and its load was waited for; otherwise the
        //    mdone wait before it means the dequant of stage j - S_TM, hence
        //    (S_TM divides S_W, or one in-order issuer) that of j - S_W, is
        //    done, so the load of j - S_W landed.  Its next phase needs this
        //    group's release of stage j.
        const int wg = (warp - 4) >> 2;
        const int part = wg % C::WG_PER;
        const int q = warp & 3;          // TMEM lane quarter of this warp
        const int r = q * 32 + lane;
        const int n = n0 + r;
        const bool row_ok = n < N;
        bool ok = true;
        constexpr int BLK_PER = 4 / C::WG_PER;  // Q4_0 blocks of the stage per thread
        const int blk0 = part * BLK_PER;
        const int sw = (r >> 1) & 3;  // 16-byte chunk c of row r is stored at chunk c ^ sw
        const int g = wg / C::WG_PER;  // dequant group: stages j with j % RR == g
        for (int j = g; j < nk; j += C::RR) {
            const int st = j % S_W, a = j % S_TM;
            // A slot a was last read by the MMAs of stage j - S_TM, whose
            // completion is phase (j - S_TM) / S_X of mdone[(j - S_TM) % S_X].
            // The warps read and release the weight stage and convert their
            // blocks before they wait for the slot.
            const bool slot_wait = j >= S_TM;
            if (!warp_wait(&wfull[st], (uint32_t)(j / S_W) & 1u, &abort_flag)) {
                ok = false;
                break;
            }
            // the stage's 4 scales of row r (the scale box holds the stage pair's 8)
            // K stage parity (which half of the scale box): stages per tile
            // are even (K % 256 == 0), so the unit's parity in an SK run
            const int kpar = ((SK ? sk_b : it0) + j) & 1;
            const uint2 sc = *reinterpret_cast<const uint2*>(smem + C::s_off(st) + r * 16 + kpar * 8);
            const uint8_t* wrow = smem + C::w_off(st) + r * (BK / 2);  // 64-byte rows of nibbles
            // hi weights of block b at columns [16 b, 16 b + 16) of the slot, lo weights 64 further
            const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(C::A_COL + a * C::A_SLOT);
            uint4 q4[BLK_PER];
#pragma unroll
            for (int bb = 0; bb < BLK_PER; bb++) q4[bb] = *reinterpret_cast<const uint4*>(wrow + (((blk0 + bb) ^ sw) << 4));
            __syncwarp();
            if (lane == 0) mbar_arrive(&wempty[st]);  // the warp's last read of the weight stage
            uint32_t vh[BLK_PER][16], vl[BLK_PER][16];
#pragma unroll
            for (int bb = 0; bb < BLK_PER; bb++) {
                const int blk = blk0 + bb;
                const uint32_t s32 = (blk < 2) ? sc.x : sc.y;
                __half2 shi2, slo2;
                split_scale((blk & 1) ? (s32 >> 16) : (s32 & 0xFFFFu), shi2, slo2);
                const uint32_t w4[4] = {q4[bb].x, q4[bb].y, q4[bb].z, q4[bb].w};
#pragma unroll
                for (int wd = 0; wd < 4; wd++) deq_word_split(w4[wd], shi2, slo2, &vh[bb][wd * 4], &vl[bb][wd * 4]);
            }
            if (slot_wait) {
                if (!warp_wait(&mdone[(j - S_TM) % S_X], (uint32_t)((j - S_TM) / S_X) & 1u, &abort_flag)) {
                    ok = false;
                    break;
                }
                tmem_fence_after();
            }
#pragma unroll
            for (int bb = 0; bb < BLK_PER; bb++) {
                tmem_st_x16(tbase + (uint32_t)((blk0 + bb) * 16), vh[bb]);
                tmem_st_x16(tbase + (uint32_t)(64 + (blk0 + bb) * 16), vl[bb]);
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tmem_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&aready[a]);
        }
        // ---------------- epilogue (first warpgroup; SK: its own warpgroup)
        if (!SK && wg == 0) {
            epi_ok = __all_sync(0xffffffffu, ok) && warp_wait(dfull, 0, &abort_flag);
            grid_dependency_wait();  // y and the residual may be touched by the previous kernel
            // Every load of a 16-token chunk (residuals) is issued before the
            // first dependent add: one memory round trip per chunk.
            if (epi_ok && epi == EPI_SILU) {
                // rows [0, 64) of the tile are gate rows, [64, 128) the matching
                // up rows (the fused weight's blocked row order): each chunk of
                // the accumulator goes through shared memory (the rings are
                // idle), then the warpgroup writes y[t][c] = silu(gate) * up
                // for c = blockIdx.x * 64 + row and its fp16 copy in the next
                // GEMM's K order
                tmem_fence_after();
                float* xb = reinterpret_cast<float*>(smem);  // [BM][EPI_CH + 1]
                const int e = threadIdx.x - 128;             // 0..127 over the epilogue warpgroup
                const int orow = e & (GU_BLOCK - 1), half = e >> 6;
                const int col = blockIdx.x * GU_BLOCK + orow;
                const size_t ncols = (size_t)N / 2;
#pragma unroll 1
                for (int c0 = 0; c0 < TN; c0 += EPI_CH) {
                    uint32_t v[EPI_CH];
                    load_accumulators<C>(tmem, q, c0, nk, v);
#pragma unroll
                    for (int jj = 0; jj < EPI_CH; jj++) xb[r * (EPI_CH + 1) + jj] = __uint_as_float(v[jj]);
                    asm volatile("bar.sync 1, 128;" ::: "memory");  // the epilogue warpgroup
                    const int tl = min(EPI_CH, T - (t0 + c0));
#pragma unroll 1
                    for (int k = 0; k < EPI_CH / 2; k++) {
                        const int jj = half * (EPI_CH / 2) + k;
                        if (jj < tl) {
                            const float o = __fmul_rn(silu_f(xb[orow * (EPI_CH + 1) + jj]),
                                                      xb[(orow + GU_BLOCK) * (EPI_CH + 1) + jj]);
                            const size_t t = (size_t)(t0 + c0 + jj);
                            y[t * ldy + col] = o;
                            if (y16) store_x16(y16 + t * 2 * ncols, (int)ncols, col, o);
                        }
                    }
                    asm volatile("bar.sync 1, 128;" ::: "memory");  // before the next chunk reuses xb
                }
            }
            // split_stride > 0: split `split` stores its partial product to
            // its own slab y + split * split_stride (the caller adds the slabs)
            else if (epi_ok && (splits == 1 || split_stride)) {
                tmem_fence_after();
                float* ys = y + (size_t)split * split_stride;
                const bool add = epi == EPI_ADD && res && !split_stride;
#pragma unroll 1
                for (int c0 = 0; c0 < TN; c0 += EPI_CH) {
                    uint32_t v[EPI_CH];
                    load_accumulators<C>(tmem, q, c0, nk, v);
                    const int tl = min(EPI_CH, T - (t0 + c0));  // tokens of this chunk
                    if (row_ok && tl > 0)
                        store_chunk(ys + (size_t)(t0 + c0) * ldy + n, ldy, v, tl,
                                    add ? res + (size_t)(t0 + c0) * ldres + n : nullptr, ldres);
                }
            }
        }
    } else if (SK) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(C::REG_EPI));
        // ---------------- SK epilogue warpgroup.  Per piece: drain the
        // accumulators (the warp's TMEM lane quarter = its 32 weight rows) and
        // release them to the issuers; a piece that does not start its tile
        // goes to this CTA's workspace slot ([TN][BM] floats) under the flag
        // of (CTA, quarter); the owner piece adds the slots of the CTAs that
        // hold the rest of the tile, in K order, then runs the epilogue.
        // Every warp takes the same pieces and branches (the SiLU barriers).
        grid_dependency_wait();  // y, the residual and the workspace may be in use by the previous kernel
        const int q = warp & 3, r = q * 32 + lane;
        const int G = (int)gridDim.x, cta = (int)blockIdx.x;
        const int tb = sk_b / nk_all, te = (sk_e - 1) / nk_all;
        float* acc = reinterpret_cast<float*>(smem + C::xb_off());  // [TN][BM]: token t of row r at t * BM + r
        bool ok = true;
        for (int tp = tb; tp <= te; tp++) {
            const int p = tp - tb;
            const int us = max(sk_b, tp * nk_all), ue = min(sk_e, (tp + 1) * nk_all);
            const int len = ue - us, ps = us - sk_b;
            const bool has[2] = {len >= 2 || (ps & 1) == 0, len >= 2 || (ps & 1) == 1};
            const bool owner = us == tp * nk_all;
            // the owner: CTAs cta + 1 .. last hold the rest of the tile; they
            // published it early in their runs, so it is summed into acc
            // while this piece's MMAs still run (then acc += this piece)
            const int last = owner ? ((tp + 1) * nk_all * G + sk_u - 1) / sk_u - 1 : cta;
            for (int cc = cta + 1; cc <= last && ok; cc++) {
                ok = sk_flag_wait(sk_flag + cc * 4 + q, &abort_flag);
                if (ok) {
                    const float* slot = sk_part + (size_t)cc * TN * BM;
#pragma unroll
                    for (int c = 0; c < TN / EPI_CH; c++) {
                        float w[EPI_CH];
#pragma unroll
                        for (int jj = 0; jj < EPI_CH; jj++) w[jj] = slot[(c * EPI_CH + jj) * BM + r];
#pragma unroll
                        for (int jj = 0; jj < EPI_CH; jj++) {
                            float* o = acc + (c * EPI_CH + jj) * BM + r;
                            *o = cc == cta + 1 ? w[jj] : *o + w[jj];
                        }
                    }
                    __syncwarp();
                    if (lane == 0) sk_flag_set(sk_flag + cc * 4 + q, 0);
                }
            }
            // (tens of microseconds per piece: the warps sleep between polls
            // rather than take issue slots from the dequant warps)
            ok = ok && __all_sync(0xffffffffu, mbar_wait(dfull, (uint32_t)p & 1u, &abort_flag, 128));
            if (ok) {
                // acc (+)= (D_0 hi + lo) + (D_1 hi + lo) of the issuers that had stages
                tmem_fence_after();
                const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
#pragma unroll
                for (int i = 0; i < 2; i++) {
                    if (!has[i]) continue;
                    const bool first = last == cta && (i == 0 || !has[0]);
#pragma unroll
                    for (int c = 0; c < TN / EPI_CH; c++) {
                        uint32_t a[EPI_CH], b[EPI_CH];
                        const uint32_t base = lane_base + (uint32_t)(i * C::D_COLS + c * EPI_CH);
                        tmem_ld_x16(base, a);
                        tmem_ld_x16(base + (uint32_t)TN, b);
                        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                        for (int jj = 0; jj < EPI_CH; jj++) {
                            const float d = __uint_as_float(a[jj]) + __uint_as_float(b[jj]);
                            float* o = acc + (c * EPI_CH + jj) * BM + r;
                            *o = first ? d : *o + d;
                        }
                    }
                }
                tmem_fence_before();
            }
            __syncwarp();
            if (ok && lane == 0) mbar_arrive(dempty);
            if (!owner) {  // a later part of a tile that an earlier CTA owns
                if (ok) {
                    float* slot = sk_part + (size_t)cta * TN * BM;
#pragma unroll 8
                    for (int t = 0; t < TN; t++) slot[t * BM + r] = acc[t * BM + r];
                    __threadfence();
                    __syncwarp();
                    if (lane == 0) sk_flag_set(sk_flag + cta * 4 + q, 1);
                }
                continue;
            }
            const int n = tp * BM + r;
            if (epi == EPI_SILU) {
                // rows [0, 64) of the tile are gate rows, [64, 128) the
                // matching up rows: thread e writes column tp * 64 + (e & 63)
                // for the tokens [16 (e >> 6), + 16)
                named_sync(1, 128);  // every row of acc is in
                const int e = threadIdx.x - C::EPI_WARP0 * 32;
                const int orow = e & (GU_BLOCK - 1), half = e >> 6;
                const int col = tp * GU_BLOCK + orow;
                const size_t ncols = (size_t)N / 2;
                if (ok) {
#pragma unroll 1
                    for (int k = 0; k < TN / 2; k++) {
                        const int t = half * (TN / 2) + k;
                        if (t < T) {
                            const float o = __fmul_rn(silu_f(acc[t * BM + orow]), acc[t * BM + orow + GU_BLOCK]);
                            y[(size_t)t * ldy + col] = o;
                            if (y16) store_x16(y16 + (size_t)t * 2 * ncols, (int)ncols, col, o);
                        }
                    }
                }
                named_sync(1, 128);  // before the next piece overwrites acc
            } else if (ok && n < N) {
                const bool add = epi == EPI_ADD && res && !split_stride;
#pragma unroll 1
                for (int c = 0; c < TN / EPI_CH; c++) {
                    const int tl = min(EPI_CH, T - c * EPI_CH);
                    if (tl > 0) {
                        uint32_t v[EPI_CH];
#pragma unroll
                        for (int jj = 0; jj < EPI_CH; jj++) v[jj] = __float_as_uint(acc[(c * EPI_CH + jj) * BM + r]);
                        store_chunk(y + (size_t)(c * EPI_CH) * ldy + n, ldy, v, tl,
                                    add ? res + (size_t)(c * EPI_CH) * ldres + n : nullptr, ldres);
                    }
                }
            }
        }
    }
    tmem_fence_before();
    __syncthreads();
    // Split K: the splits of a tile form one thread-block cluster.  Rows of
    // the tile are divided among the cluster's CTAs (rank R owns rows
    // [rows R / splits, rows (R + 1) / splits)); after a cluster barrier (every
    // CTA is past its main loop, so its rings are free) each CTA stores its
    // partial sums of every row into the owner's shared memory over the
    // cluster (posted stores, no round trips), and after a second barrier each
    // owner adds the splits' partials of its rows in split order, so the
    // result is deterministic and no partial sum leaves the chip.  Every CTA
    // reaches both barriers, also after an abort (the error flag then reports
    // the garbage).
    const int rows = min(BM, N - n0), toks = min(TN, T - t0);
    const int slab = (BM + splits - 1) / splits;  // >= rows owned by any rank
    const uint32_t recv = smem_u32(smem);         // [split][slab][RED_PITCH] floats
    const bool cluster_reduce = splits > 1 && split_stride == 0;
    if (cluster_reduce) {
        cluster_sync();
        if (warp >= 4 && warp < 8 && epi_ok) {
            tmem_fence_after();
            const int q = warp & 3, r = q * 32 + lane;
            const bool has_row = r < rows;
            int owner = 0;
            while (has_row && owner + 1 < splits && rows * (owner + 1) / splits <= r) owner++;
            const uint32_t row_addr =
                recv + (uint32_t)(((split * slab + (has_row ? r - rows * owner / splits : 0)) * C::RED_PITCH) * 4);
#pragma unroll 1
            for (int c0 = 0; c0 < TN; c0 += EPI_CH) {
                uint32_t v[EPI_CH];
                load_accumulators<C>(tmem, q, c0, nk, v);  // warp-collective
                if (has_row) {
#pragma unroll
                    for (int jj = 0; jj < EPI_CH; jj++)
                        st_dsmem_f32(row_addr + (uint32_t)((c0 + jj) * 4), owner, __uint_as_float(v[jj]));
                }
            }
        }
        tmem_fence_before();
        __syncthreads();
    }
    if (warp == 2) {
        __syncwarp();  // lane 0 ran the X producer
        tmem_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::COLS) : "memory");
    }
    if (cluster_reduce) {
        cluster_sync();  // every partial has landed
        grid_dependency_wait();
        const int rank = (int)cluster_ctarank();
        const int r0 = rows * rank / splits, r1 = rows * (rank + 1) / splits, nr = r1 - r0;
        const float* rv = reinterpret_cast<const float*>(smem);
        for (int o = threadIdx.x; o < nr * toks; o += C::THREADS) {
            const int rr = o % nr, t = o / nr;
            float acc = 0.0f;
            for (int sp = 0; sp < splits; sp++) acc += rv[(sp * slab + rr) * C::RED_PITCH + t];
            if (epi == EPI_ADD && res) acc = acc + res[(size_t)(t0 + t) * ldres + n0 + r0 + rr];
            y[(size_t)(t0 + t) * ldy + n0 + r0 + rr] = acc;
        }
    }
    if (threadIdx.x == 0 && abort_flag) atomicExch(err, 1);
}

// fp32 rows -> the GEMM's split fp16 rows (store_x16): per token 2K halves,
// hi then lo, each in the K order of the weight tiles (see deq_word_split):
// within every 8 elements, [e0 e4 e1 e5 e2 e6 e3 e7].
__global__ void k_rows_to_f16_perm(const float* __restrict__ x, size_t ldx, __half* __restrict__ out, int K, int T) {
    pdl_trigger();
    int t = blockIdx.y;
    const float* xr = x + (size_t)t * ldx;
    __half2* oh = reinterpret_cast<__half2*>(out + (size_t)t * 2 * K);
    __half2* ol = oh + K / 2;
    for (int gi = blockIdx.x * blockDim.x + threadIdx.x; gi < K / 8; gi += gridDim.x * blockDim.x) {
        const float* e = xr + 8 * gi;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const float a = e[k], b = e[k + 4];
            const __half2 h = __floats2half2_rn(a, b);
            oh[4 * gi + k] = h;
            ol[4 * gi + k] = __floats2half2_rn(__fsub_rn(a, __low2float(h)), __fsub_rn(b, __high2float(h)));
        }
    }
}

}  // namespace

static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

int encode_2d(CUtensorMap* map, CUtensorMapDataType dt, void* base, uint64_t inner, uint64_t outer,
              uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
    auto fn = get_encode();
    HC_CHECK(fn, HC_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, dt, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    HC_CHECK(r == CUDA_SUCCESS, HC_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return HC_OK;
}

// Nibble plane as [n][k/2] bytes in 128-row x 64-byte boxes (64-byte swizzle);
// scale plane as [n][k/32] fp16 in 128-row x 8-scale boxes (16 bytes: the
// scales of a pair of 128-wide K stages, so every box starts 16-byte aligned).
int encode_weight_maps(const hc_q4_matrix& w, CUtensorMap* wmap, CUtensorMap* smap) {
    const size_t K = w.k, KB = K / 32;
    HC_TRY(encode_2d(wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.qs, K / 2, w.n, K / 2, BK / 2, BM,
                     CU_TENSOR_MAP_SWIZZLE_64B));
    HC_TRY(encode_2d(smap, CU_TENSOR_MAP_DATA_TYPE_UINT16, w.sc, KB, w.n, KB * 2, 8, BM, CU_TENSOR_MAP_SWIZZLE_NONE));
    return HC_OK;
}


struct GemmWorkspace {
    std::mutex mu;
    uint64_t generation = 0;  // bumped whenever a buffer a launch refers to moves
    __half* xh = nullptr;
    size_t xh_cap = 0;
    int* err = nullptr;
    int device = -1;
    // (nibble plane, scale plane, n, k) -> nibble and scale tensor maps
    std::map<std::tuple<const void*, const void*, size_t, size_t>, std::pair<CUtensorMap, CUtensorMap>> wmaps;
    // [token tile 32/64/128][splits] -> CTAs resident at once (0: not yet queried)
    int slots[3][MAX_SPLITS + 1] = {};
    // stream-K: one [32][BM] partial slot and 4 flags per CTA (sk_cap CTAs)
    float* sk_part = nullptr;
    int* sk_flag = nullptr;
    int sk_cap = 0;
};

GemmWorkspace* gemm_workspace_new() { return new GemmWorkspace(); }

void gemm_workspace_free(GemmWorkspace* ws) {
    if (!ws) return;
    if (ws->xh) cudaFree(ws->xh);
    if (ws->err) cudaFree(ws->err);
    if (ws->sk_part) cudaFree(ws->sk_part);
    if (ws->sk_flag) cudaFree(ws->sk_flag);
    delete ws;
}

bool gemm_tc_eligible(const hc_q4_matrix& w, size_t tokens) {
    // k % 256: the scale plane's row pitch (k / 32 fp16) is then a multiple of
    // 16 bytes, as a tensor map needs
    return tokens >= 2 && w.k % (2 * BK) == 0 && w.n >= BM && w.nblocks >= w.n * (w.k / 32) && w.k <= (1u << 20) &&
           ((uintptr_t)w.sc & 15) == 0;
}

namespace {
// Dynamic shared memory of a launch.  A CTA (512 tensor-memory columns) asks
// for at least 116 KB, so it is alone on its SM and its tensor-memory
// allocation never waits for another CTA of this kernel.
template <int TN, bool SK = false>
int launch_smem() {
    using C = Cfg<TN, SK>;
    return C::smem() < 118784 ? 118784 : C::smem();
}

// CTAs of the kernel resident at once when the splits of a tile form a
// cluster of `sp` CTAs.  A cluster must fit within one GPC, so with large
// clusters fewer CTAs than (blocks per SM x SMs) run together, and a grid of
// clusters beyond that number runs a second wave.
template <int TN>
int resident_ctas(int sp) {
    using C = Cfg<TN>;
    auto kfn = k_q4_gemm_tc<TN>;
    const int smem = launch_smem<TN>();
    int dev = 0, nsm = 0, nb = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kfn, C::THREADS, (size_t)smem) != cudaSuccess || nb < 1) {
        (void)cudaGetLastError();
        return 148 * C::MIN_BLOCKS;
    }
    if (sp == 1) return nb * nsm;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, 1, (unsigned)sp);
    cfg.blockDim = dim3(C::THREADS);
    cfg.dynamicSmemBytes = (size_t)smem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 1;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = (unsigned)sp;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int nc = 0;
    if (cudaOccupancyMaxActiveClusters(&nc, kfn, &cfg) != cudaSuccess || nc < 1) {
        (void)cudaGetLastError();
        return nb * nsm;
    }
    return nc * sp;
}

// SK: a stream-K grid of sk_grid CTAs (at most one per SM, so all of them
// are resident together and a tile's owner can wait for the others' flags)
// with its workspace; splits must then be 1.
template <int TN, bool SK = false>
int launch_tc(const hc_q4_matrix& w, const CUtensorMap& xmap, const CUtensorMap& wmap, const CUtensorMap& smap,
              size_t T, float* y,
              size_t ldy, int epi, const float* res, size_t ldres, int splits, int* err, cudaStream_t s,
              size_t split_stride = 0, __half* y16 = nullptr, float* sk_part = nullptr, int* sk_flag = nullptr,
              int sk_grid = 0) {
    using C = Cfg<TN, SK>;
    auto kfn = k_q4_gemm_tc<TN, SK>;
    const int smem = launch_smem<TN, SK>();
    HC_CUDA(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    HC_CHECK(splits >= 1 && splits <= MAX_SPLITS, HC_ERR_INVALID, "tcgen05 GEMM: %d K splits", splits);
    HC_CHECK(!SK || (splits == 1 && T <= (size_t)TN && sk_grid >= 1 && sk_part && sk_flag), HC_ERR_INVALID,
             "tcgen05 GEMM: stream-K launch arguments");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = SK ? dim3((unsigned)sk_grid)
                     : dim3((unsigned)((w.n + BM - 1) / BM), (unsigned)((T + TN - 1) / TN), (unsigned)splits);
    cfg.blockDim = dim3(C::THREADS);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    int na = 0;
    // programmatic dependent launch: the weight prefetch overlaps the tail of
    // the kernel that produces X (the kernel waits on the dependency itself)
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    na++;
    if (splits > 1 && split_stride == 0) {  // the splits of one tile form a cluster (reduction in shared memory)
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = 1;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = (unsigned)splits;
        na++;
    }
    cfg.attrs = attr;
    cfg.numAttrs = (unsigned)na;
    HC_CUDA(cudaLaunchKernelEx(&cfg, kfn, xmap, wmap, smap, y, ldy, res, ldres, epi, (int)w.n,
                               (int)w.k, (int)T, splits, split_stride, y16, err, sk_part, sk_flag));
    hc_count_launch();
    return HC_OK;
}

// K splits per tile (1..MAX_SPLITS) minimizing a time model in units of one
// pipeline stage: a CTA costs a fixed ~10 stages (launch, pipeline fill,
// epilogue) plus its stages; a split tile adds the cluster barriers and the
// reduction (~7 stages for two splits, ~10 up to four, ~15 up to eight);
// slots[sp] = CTAs resident at once with clusters of sp (one per SM without
// clusters), so CTAs beyond it run in further waves.
// With max_part > 0 the splits are not reduced in a cluster but written as
// slabs the caller adds (up to max_part of them): no cluster residency limit,
// and each extra slab costs the consumer about half a stage of reading.
int choose_splits(size_t tiles, size_t nk, const int* slots, int nsm, int max_part = 0, double* cost_out = nullptr) {
    const double fixed = 10.0;
    const int max_sp = max_part > 0 ? std::min(max_part, MAX_SPLITS) : MAX_SPLITS;
    int best = 1;
    double best_cost = 1e300;
    for (size_t sp = 1; sp <= (size_t)max_sp && (sp == 1 || nk / sp >= 2); sp++) {
        const int sl_raw = max_part > 0 ? nsm : slots[sp];
        const size_t sl = (size_t)(sl_raw > 0 ? sl_raw : 1);
        const size_t ctas = tiles * sp;
        const size_t waves = (ctas + sl - 1) / sl;
        const double reduce = max_part > 0 ? 0.5 * (double)(sp - 1)
                              : sp == 1    ? 0.0
                              : sp == 2    ? 7.0
                              : sp <= 4    ? 10.0
                                           : 15.0;
        const double cost = (double)waves * (fixed + (double)((nk + sp - 1) / sp)) + reduce;
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = (int)sp;
        }
    }
    if (cost_out) *cost_out = best_cost;
    return best;
}

// Stream-K on the same scale: every CTA of the grid (one per SM) pays the
// fixed cost once and takes ceil(U / G) stages; a piece boundary costs the
// issuers a wait for the accumulator drain (~1.5 stages), and a tile's owner
// adds the partials of the CTAs that hold the rest of it one after another
// (~0.75 stages each).  Only runs of at least one tile (per >= nk) qualify:
// then a piece that does not start its tile is the first piece of its CTA
// and shorter than a tile, so it is published well before its owner's last
// piece ends; with shorter runs it can be a CTA's whole run, and the owner
// waits for it at the end (the 112-tile gate/up of a 2-way tensor-parallel
// c4 rank ran 27.5 µs as stream-K against 24.7 µs as one wave of tiles).
// Taken when it beats the best tile-per-CTA launch by at least two stages.
double stream_k_cost(size_t tiles, size_t nk, int nsm) {
    const size_t U = tiles * nk, G = std::min<size_t>((size_t)nsm, U);
    const size_t per = (U + G - 1) / G;
    if (U / G < nk) return 1e300;
    const size_t others = (nk - 1 + per - 1) / per;  // CTAs after the owner on one tile, at most
    return 10.0 + (double)per + 1.5 + 0.75 * (double)others;
}

template <int TN>
const int* tile_slots(GemmWorkspace* ws, int ti) {
    int* sl = ws->slots[ti];
    if (!sl[1])
        for (int sp = 1; sp <= MAX_SPLITS; sp++) sl[sp] = resident_ctas<TN>(sp);
    return sl;
}
}  // namespace

namespace {
int gemm_tc_impl(GemmWorkspace* ws, const hc_q4_matrix& w, const float* x, size_t ldx, size_t tokens, float* y,
                 size_t ldy, int epi, const float* res, size_t ldres, cudaStream_t s, const __half* xh_ready,
                 int max_part, int* splits_out, __half* y16 = nullptr) {
    std::lock_guard<std::mutex> lock(ws->mu);
    const size_t K = w.k, T = tokens;
    int dev = 0;
    HC_CUDA(cudaGetDevice(&dev));
    if (ws->device != dev) {  // buffers belong to one device
        ws->xh = nullptr;
        ws->xh_cap = 0;
        ws->err = nullptr;
        ws->sk_part = nullptr;
        ws->sk_flag = nullptr;
        ws->sk_cap = 0;
        ws->wmaps.clear();
        for (auto& row : ws->slots)
            for (int& v : row) v = 0;
        ws->device = dev;
    }
    if (!ws->err) {
        HC_CUDA(cudaMalloc((void**)&ws->err, sizeof(int)));
        HC_CUDA(cudaMemset(ws->err, 0, sizeof(int)));
    }
    int nsm = 148;
    HC_CUDA(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
    if (ws->sk_cap < nsm) {  // with the error flag, on the first (eager) call
        if (ws->sk_part) cudaFree(ws->sk_part);
        if (ws->sk_flag) cudaFree(ws->sk_flag);
        ws->sk_part = nullptr;
        ws->sk_flag = nullptr;
        ws->sk_cap = 0;
        HC_CUDA(cudaMalloc((void**)&ws->sk_part, (size_t)nsm * 32 * BM * sizeof(float)));
        HC_CUDA(cudaMalloc((void**)&ws->sk_flag, (size_t)nsm * 4 * sizeof(int)));
        HC_CUDA(cudaMemset(ws->sk_flag, 0, (size_t)nsm * 4 * sizeof(int)));
        ws->sk_cap = nsm;
        ws->generation++;
    }
    if (!xh_ready && 2 * T * K > ws->xh_cap) {  // hi and lo rows
        if (ws->xh) cudaFree(ws->xh);
        ws->xh = nullptr;
        ws->generation++;
        HC_CUDA(cudaMalloc((void**)&ws->xh, 2 * T * K * sizeof(__half)));
        ws->xh_cap = 2 * T * K;
    }
    const __half* xh = xh_ready;
    if (!xh) {
        unsigned gx = (unsigned)std::min<size_t>((K / 8 + 255) / 256, 16);
        k_rows_to_f16_perm<<<dim3(gx, (unsigned)T), 256, 0, s>>>(x, ldx, ws->xh, (int)K, (int)T);
        HC_LAUNCH_CHECK();
        xh = ws->xh;
    }
    // Token tile: the smallest of 32/64/128 covering T (one tile for decode).
    const int tn = T <= 32 ? 32 : T <= 64 ? 64 : 128;
    CUtensorMap xmap;  // rows of 2K halves: hi, then lo
    HC_TRY(encode_2d(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, const_cast<__half*>(xh), 2 * K, T, K * 4, 64, (uint32_t)tn,
                     CU_TENSOR_MAP_SWIZZLE_128B));
    auto key = std::make_tuple((const void*)w.qs, (const void*)w.sc, w.n, w.k);
    auto itw = ws->wmaps.find(key);
    CUtensorMap wmap, smap;
    if (itw != ws->wmaps.end()) {
        wmap = itw->second.first;
        smap = itw->second.second;
    } else {
        HC_TRY(encode_weight_maps(w, &wmap, &smap));
        if (w.owns) ws->wmaps[key] = std::make_pair(wmap, smap);
    }
    size_t tiles = ((w.n + BM - 1) / BM) * ((T + tn - 1) / tn);
    const size_t nk = K / BK;
    const size_t stride = max_part > 0 ? T * ldy : 0;  // slab stride in partial mode
    const bool one = epi == EPI_SILU;                  // the SiLU epilogue needs whole sums
    int splits = 1;
    switch (tn) {
        case 32: {
            double cost = 0.0;
            if (!one)
                splits = choose_splits(tiles, nk, tile_slots<32>(ws, 0), nsm, max_part, &cost);
            else
                cost = (double)((tiles + nsm - 1) / nsm) * (10.0 + (double)nk);
            if (tiles * nk * (size_t)nsm < ((size_t)1 << 31) && stream_k_cost(tiles, nk, nsm) + 2.0 < cost) {  // one slab (partial mode) or the whole product
                splits = 1;
                const int g = (int)std::min<size_t>((size_t)nsm, tiles * nk);
                HC_TRY((launch_tc<32, true>(w, xmap, wmap, smap, T, y, ldy, epi, res, ldres, 1, ws->err, s, stride,
                                            y16, ws->sk_part, ws->sk_flag, g)));
            } else {
                HC_TRY(launch_tc<32>(w, xmap, wmap, smap, T, y, ldy, epi, res, ldres, splits, ws->err, s, stride,
                                     y16));
            }
            break;
        }
        case 64:
            if (!one) splits = choose_splits(tiles, nk, tile_slots<64>(ws, 1), nsm, max_part);
            HC_TRY(launch_tc<64>(w, xmap, wmap, smap, T, y, ldy, epi, res, ldres, splits, ws->err, s, stride, y16));
            break;
        default:
            if (!one) splits = choose_splits(tiles, nk, tile_slots<128>(ws, 2), nsm, max_part);
            HC_TRY(launch_tc<128>(w, xmap, wmap, smap, T, y, ldy, epi, res, ldres, splits, ws->err, s, stride, y16));
            break;
    }
    if (splits_out) *splits_out = splits;
    return HC_OK;
}
}  // namespace

int gemm_tc(GemmWorkspace* ws, const hc_q4_matrix& w, const float* x, size_t ldx, size_t tokens, float* y,
            size_t ldy, int epi, const float* res, size_t ldres, cudaStream_t s, const __half* xh_ready) {
    return gemm_tc_impl(ws, w, x, ldx, tokens, y, ldy, epi, res, ldres, s, xh_ready, 0, nullptr);
}

int gemm_tc_silu(GemmWorkspace* ws, const hc_q4_matrix& w, const float* x, size_t ldx, size_t tokens, float* act,
                 size_t ldact, __half* act16, cudaStream_t s, const __half* xh_ready) {
    HC_CHECK(w.n % (2 * GU_BLOCK) == 0, HC_ERR_INVALID, "gemm_tc_silu: %zu rows are not whole gate/up blocks", w.n);
    return gemm_tc_impl(ws, w, x, ldx, tokens, act, ldact, EPI_SILU, nullptr, 0, s, xh_ready, 0, nullptr, act16);
}

int gemm_tc_partials(GemmWorkspace* ws, const hc_q4_matrix& w, const float* x, size_t ldx, size_t tokens,
                     float* part, int max_splits, int* splits, cudaStream_t s, const __half* xh_ready) {
    HC_CHECK(max_splits >= 1 && splits, HC_ERR_INVALID, "gemm_tc_partials: max_splits %d", max_splits);
    return gemm_tc_impl(ws, w, x, ldx, tokens, part, w.n, EPI_STORE, nullptr, 0, s, xh_ready, max_splits, splits);
}

uint64_t gemm_generation(GemmWorkspace* ws) { return ws ? ws->generation : 0; }

int* gemm_error_flag(GemmWorkspace* ws) {
    std::lock_guard<std::mutex> lock(ws->mu);
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    if (ws->device != dev) {
        ws->xh = nullptr;
        ws->xh_cap = 0;
        ws->err = nullptr;
        ws->sk_part = nullptr;
        ws->sk_flag = nullptr;
        ws->sk_cap = 0;
        ws->wmaps.clear();
        for (auto& row : ws->slots)
            for (int& v : row) v = 0;
        ws->device = dev;
    }
    if (!ws->err) {
        if (cudaMalloc((void**)&ws->err, sizeof(int)) != cudaSuccess) return nullptr;
        if (cudaMemset(ws->err, 0, sizeof(int)) != cudaSuccess) return nullptr;
    }
    return ws->err;
}

int gemm_check(GemmWorkspace* ws) {
    if (!ws || !ws->err) return HC_OK;
    int h = 0;
    HC_CUDA(cudaMemcpy(&h, ws->err, sizeof(int), cudaMemcpyDeviceToHost));
    if (h) {
        HC_CUDA(cudaMemset(ws->err, 0, sizeof(int)));
        // an aborted stream-K launch may leave contributor flags raised;
        // a later owner would then add a stale slot without waiting
        if (ws->sk_flag) HC_CUDA(cudaMemset(ws->sk_flag, 0, (size_t)ws->sk_cap * 4 * sizeof(int)));
        hc_set_error("a bounded pipeline wait timed out in a tcgen05 GEMM or a TMA attention kernel (the kernel "
                     "aborted and skipped its stores)");
        return HC_ERR_TIMEOUT;
    }
    return HC_OK;
}

}  // namespace hc

// ============================================================ allocation-free entry point
//
// Some callers cannot allocate device memory once they are running: a serving
// process that hands all device memory to its own pool at start-up and must
// not grow it, or a caller that may not call cudaMalloc (which can
// synchronize the device) while other work is in flight.  For them the
// tensor-core matmul below keeps its scratch (the split fp16 copy of the
// activations and the pipeline abort flag) in a fixed array that lives in the
// library's device image, so a call allocates nothing.
namespace {

// Stated maximum: 8 MiB per device, held by every GPU that loads the library
// until the process exits.  The split fp16 rows (2 * tokens * k halves, i.e.
// tokens * k * 4 bytes) must fit after the flag.
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
constexpr size_t kNoAllocFlagBytes = 256;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
uint8_t* g_noalloc_ptr[kMaxDevices] = {nullptr};
std::mutex g_noalloc_mu;

// Device address of the array for the current device.  In host code the
// symbol is only a host-side stand-in, never a device address, so the address
// is looked up with cudaGetSymbolAddress once per device (with that device
// current), its abort flag is cleared, and the address is cached.
int noalloc_scratch(uint8_t** out) {
    int dev = 0;
    HC_CUDA(cudaGetDevice(&dev));
    HC_CHECK(dev >= 0 && dev < kMaxDevices, HC_ERR_UNSUPPORTED, "device index %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return hc_cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)", __FILE__, __LINE__);
        HC_CUDA(cudaMemset(p, 0, sizeof(int)));  // the abort flag starts clear
        g_noalloc_ptr[dev] = static_cast<uint8_t*>(p);
    }
    *out = g_noalloc_ptr[dev];
    return HC_OK;
}

// Reads the abort flag after the launch (a 4-byte copy into a host stack
// variable, then a wait for the stream): a bounded pipeline wait that ran out
// makes the kernel skip its stores, so the call must not report success.
int noalloc_status(int* err, cudaStream_t s) {
    int h = 0;
    HC_CUDA(cudaMemcpyAsync(&h, err, sizeof(int), cudaMemcpyDeviceToHost, s));
    HC_CUDA(cudaStreamSynchronize(s));
    if (h) {
        HC_CUDA(cudaMemsetAsync(err, 0, sizeof(int), s));
        HC_CUDA(cudaStreamSynchronize(s));
        hc_set_error("hc_q4_matmul_noalloc: a bounded pipeline wait timed out (the kernel aborted and skipped its "
                     "stores; y is not written)");
        return HC_ERR_TIMEOUT;
    }
    return HC_OK;
}

}  // namespace

// Y[mtok x n] = X[mtok x k] . W^T like hc_q4_matmul_dev, without allocating
// device or host memory: shapes the tensor cores take (mtok >= 2, k % 256 ==
// 0, n >= 128) run the tcgen05 kernel with its scratch in the fixed array and
// no split-K, then wait for the stream to read the kernel's abort flag; other
// shapes run the CUDA-core matvec, which needs no scratch.
HC_EXPORT int hc_q4_matmul_noalloc(const hc_q4_matrix* w, const float* x, size_t mtok, float* y, void* stream) {
    HC_CHECK(w && x && y, HC_ERR_INVALID, "hc_q4_matmul_noalloc: NULL argument");
    cudaStream_t s = (cudaStream_t)stream;
    if (!hc::gemm_tc_eligible(*w, mtok)) {
        DevWeight dw;
        dw.dtype = HC_DTYPE_Q4_0;
        dw.n = w->n;
        dw.k = w->k;
        dw.q4 = *w;
        dw.present = true;
        return hc::launch_matmul(dw, x, w->k, mtok, y, w->n, hc::EPI_STORE, nullptr, 0, s);
    }
    const size_t K = w->k, T = mtok;
    const size_t max_t = (kNoAllocScratchBytes - kNoAllocFlagBytes) / (2 * K * sizeof(__half));
    HC_CHECK(T <= max_t, HC_ERR_INVALID,
             "hc_q4_matmul_noalloc: %zu tokens x %zu columns exceed the fixed %zu-byte scratch (at most %zu tokens "
             "at this width)",
             T, K, kNoAllocScratchBytes, max_t);
    uint8_t* base = nullptr;
    HC_TRY(noalloc_scratch(&base));
    int* err = reinterpret_cast<int*>(base);
    __half* xh = reinterpret_cast<__half*>(base + kNoAllocFlagBytes);
    {
        unsigned gx = (unsigned)std::min<size_t>((K / 8 + 255) / 256, 16);
        hc::k_rows_to_f16_perm<<<dim3(gx, (unsigned)T), 256, 0, s>>>(x, K, xh, (int)K, (int)T);
        HC_LAUNCH_CHECK();
    }
    const int tn = T <= 32 ? 32 : T <= 64 ? 64 : 128;
    CUtensorMap xmap, wmap, smap;
    HC_TRY(hc::encode_2d(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xh, 2 * K, T, K * 4, 64, (uint32_t)tn,
                         CU_TENSOR_MAP_SWIZZLE_128B));
    HC_TRY(hc::encode_weight_maps(*w, &wmap, &smap));
    switch (tn) {
        case 32: HC_TRY(hc::launch_tc<32>(*w, xmap, wmap, smap, T, y, w->n, hc::EPI_STORE, nullptr, 0, 1, err, s)); break;
        case 64: HC_TRY(hc::launch_tc<64>(*w, xmap, wmap, smap, T, y, w->n, hc::EPI_STORE, nullptr, 0, 1, err, s)); break;
        default: HC_TRY(hc::launch_tc<128>(*w, xmap, wmap, smap, T, y, w->n, hc::EPI_STORE, nullptr, 0, 1, err, s)); break;
    }
    return noalloc_status(err, s);
}
