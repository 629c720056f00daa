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
//   TMA (warp 0)      X tile (fp16, K-major, 128B swizzle) + the Q4_0 nibble
//                     tile of 128 rows x 128 K  -> shared memory stage s
//   dequant (warps 4-11, two warpgroups, one weight row per thread)
//                     nibbles -> (nib - 8) * scale in fp16 -> tcgen05.st into
//                     tensor memory (the A operand never touches shared
//                     memory, so shared-memory bandwidth is left to the TMA
//                     traffic and the B operand)
//   MMA (warp 1)      tcgen05.mma.kind::f16, A from TMEM, B from the smem
//                     descriptor, f32 accumulator in TMEM; tcgen05.commit
//                     frees the stage
//   epilogue (warps 4-7)  tcgen05.ld of the accumulator -> Y (+ residual)
//
// No cluster multicast is used anywhere (the same code runs under tensor
// parallelism on several GPUs).  Every mbarrier wait is bounded by a clock
// deadline; on expiry the kernel records an error flag, skips its stores, and
// still frees its tensor memory before returning.
#include "hc_gemm.h"
#include "hc_common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <map>
#include <tuple>

namespace hc {

namespace {

constexpr int BM = 128;      // weight rows per tile (MMA M)
constexpr int BK = 128;      // K per pipeline stage
constexpr int TMEM_COLS = 512;
constexpr long long WAIT_CYCLES = 4000000000LL;  // ~2 s at 1.9 GHz

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on the phase with the given parity.  Returns false when the
// deadline passes or another role already reported a failure.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    long long start = clock64();
    for (uint32_t i = 0;; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255) == 255) {
            if (*abort_flag) return false;
            if (clock64() - start > WAIT_CYCLES) {
                *abort_flag = 1;
                return false;
            }
        }
    }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
        "[%2];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tmem_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld_x32(uint32_t taddr, uint32_t* v) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
          "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr)
        : "memory");
}

// Shared-memory matrix descriptor of a K-major tile in the 128-byte swizzle
// canonical layout: rows of 128 bytes, 8-row (1024-byte) atoms.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);         // start address
    d |= (uint64_t)1 << 16;                          // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;                // stride byte offset: 8 rows x 128 B
    d |= (uint64_t)1 << 46;                          // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;                          // layout: 128-byte swizzle
    return d;
}

// Instruction descriptor: f16 x f16 -> f32, A and B K-major, M = 128, N = tn.
__host__ __device__ constexpr uint32_t make_idesc(int tn) {
    return (1u << 4)                       // D format f32
           | (0u << 7) | (0u << 10)        // A, B format f16
           | (0u << 15) | (0u << 16)       // A, B K-major
           | ((uint32_t)(tn >> 3) << 17)   // N / 8
           | ((uint32_t)(BM >> 4) << 24);  // M / 16
}

__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// K order inside a 32-element Q4_0 block.  Word i (4 bytes = elements
// 8i..8i+7, low nibble first) yields four fp16 pairs with one shift and one
// and/or each: pair k = (element 8i+k, element 8i+k+4).  The A operand (the
// weights) is therefore laid out along K in the order
//   position 8i+2k <- element 8i+k,   position 8i+2k+1 <- element 8i+k+4,
// and the B operand (the activations) is written in the same order by
// k_rows_to_f16_perm, so every dot product sees matching pairs.
// (nib + 1024) is exact in fp16 (0x6400 | nib); subtracting 1032 is exact;
// multiplying by the fp16 scale rounds once: fp16((nib - 8) * scale).
__device__ __forceinline__ uint32_t deq_pair(uint32_t w, int k, __half2 s2) {
    uint32_t v = ((w >> (4 * k)) & 0x000F000Fu) | 0x64006400u;
    __half2 h = *reinterpret_cast<__half2*>(&v);
    h = __hsub2(h, __float2half2_rn(1032.0f));
    h = __hmul2(h, s2);
    return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void tmem_st_x16(uint32_t taddr, const uint32_t* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}

// Warp-uniform bounded wait: lane 0 polls, the verdict is broadcast, then
// every lane observes the completed phase once itself (acquire ordering for
// its own reads of the data the barrier guards).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    bool ok = true;
    if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort_flag);
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    if (ok) (void)mbar_try_wait(bar, parity);
    return ok;
}

template <int TN>
struct Cfg {
    static constexpr int STAGES = TN <= 64 ? 7 : (TN == 128 ? 5 : 3);
    static constexpr int A_COL = TN <= 64 ? 64 : TN;  // A stages start here; D occupies [0, TN)
    static constexpr int X_STAGE = 2 * TN * 128;      // two 64-element K halves, 128 B per token row
    static constexpr int W_STAGE = BM * (BK / 2);     // 128 rows x 64 nibble bytes
    __host__ __device__ static constexpr int x_off(int s) { return s * X_STAGE; }
    __host__ __device__ static constexpr int w_off(int s) { return STAGES * X_STAGE + s * W_STAGE; }
    __host__ __device__ static constexpr int bar_off() { return STAGES * (X_STAGE + W_STAGE); }
    __host__ __device__ static constexpr int smem() { return bar_off() + (3 * STAGES + 1) * 8 + 16 + 1024; }
    static_assert(A_COL + 64 * STAGES <= TMEM_COLS, "tensor memory budget");
};

constexpr int NDEQ_WARPS = 16;                  // 4 warpgroups, one Q4_0 block of the stage each
constexpr int GEMM_THREADS = 128 + 32 * NDEQ_WARPS;

template <int TN>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    k_q4_gemm_tc(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                 const __half* __restrict__ scales, float* __restrict__ y, size_t ldy, const float* res, size_t ldres,
                 int epi, int N, int K, int T, int splits, float* __restrict__ partial, int* __restrict__ err) {
    using C = Cfg<TN>;
    constexpr int STAGES = C::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::bar_off());
    uint64_t* aready = full + STAGES;
    uint64_t* empty = aready + STAGES;
    uint64_t* dfull = empty + STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dfull + 1);
    __shared__ int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BM, t0 = blockIdx.y * TN, split = blockIdx.z;
    const int KB = K / 32;
    const int nk_all = K / BK;
    const int it0 = (int)((long long)nk_all * split / splits), it1 = (int)((long long)nk_all * (split + 1) / splits);
    const int nk = it1 - it0;

    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int st = 0; st < STAGES; st++) {
            mbar_init(&full[st], 1);
            mbar_init(&aready[st], NDEQ_WARPS);
            mbar_init(&empty[st], 1);
        }
        mbar_init(dfull, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 2) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer
        if (lane == 0) {
            for (int j = 0; j < nk; j++) {
                int st = j % STAGES;
                uint32_t ph = (uint32_t)(j / STAGES) & 1u;
                if (!mbar_wait(&empty[st], ph ^ 1u, &abort_flag)) break;
                mbar_expect_tx(&full[st], (uint32_t)(C::X_STAGE + C::W_STAGE));
                uint8_t* xs = smem + C::x_off(st);
                int kk = (it0 + j) * BK;
                tma_load_2d(xs, &xmap, &full[st], kk, t0);
                tma_load_2d(xs + TN * 128, &xmap, &full[st], kk + 64, t0);
                tma_load_2d(smem + C::w_off(st), &wmap, &full[st], kk / 2, n0);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = make_idesc(TN);
            bool ok = true;
            for (int j = 0; j < nk; j++) {
                int st = j % STAGES;
                uint32_t ph = (uint32_t)(j / STAGES) & 1u;
                if (!mbar_wait(&aready[st], ph, &abort_flag)) {
                    ok = false;
                    break;
                }
                tmem_fence_after();
                const uint32_t xs = smem_u32(smem + C::x_off(st));
#pragma unroll
                for (int kk = 0; kk < BK / 16; kk++) {
                    uint32_t a_tmem = tmem + (uint32_t)(C::A_COL + st * 64 + kk * 8);
                    uint32_t b_addr = xs + (uint32_t)((kk >> 2) * TN * 128 + (kk & 3) * 32);
                    mma_f16_ts(tmem, a_tmem, sw128_desc(b_addr), idesc, (j > 0 || kk > 0) ? 1u : 0u);
                }
                mma_commit(&empty[st]);
            }
            if (ok) mma_commit(dfull);
        }
    } else if (warp >= 4) {
        // ---------------- dequant: thread <-> weight row (TMEM lane), warpgroup <-> Q4_0 block of the stage
        const int g = (warp - 4) >> 2;   // block 0..3 of the 128-element stage
        const int q = warp & 3;          // TMEM lane quarter of this warp
        const int r = q * 32 + lane;
        const int n = n0 + r;
        const bool row_ok = n < N;
        const __half* srow = scales + (size_t)(row_ok ? n : 0) * KB;
        unsigned short sc_next = row_ok ? __ldg(reinterpret_cast<const unsigned short*>(srow) + it0 * 4 + g) : 0;
        bool ok = true;
        for (int j = 0; j < nk; j++) {
            int st = j % STAGES;
            uint32_t ph = (uint32_t)(j / STAGES) & 1u;
            unsigned short sc = sc_next;
            if (j + 1 < nk && row_ok)
                sc_next = __ldg(reinterpret_cast<const unsigned short*>(srow) + (it0 + j + 1) * 4 + g);
            if (!warp_wait(&empty[st], ph ^ 1u, &abort_flag) || !warp_wait(&full[st], ph, &abort_flag)) {
                ok = false;
                break;
            }
            uint4 q4 = *reinterpret_cast<const uint4*>(smem + C::w_off(st) + r * (BK / 2) + g * 16);
            __half2 s2 = __half2half2(__ushort_as_half(sc));
            uint32_t v[16];
            const uint32_t w4[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
            for (int wd = 0; wd < 4; wd++)
#pragma unroll
                for (int k = 0; k < 4; k++) v[wd * 4 + k] = deq_pair(w4[wd], k, s2);
            tmem_st_x16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(C::A_COL + st * 64 + g * 16), v);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tmem_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&aready[st]);
        }
        // ---------------- epilogue (first warpgroup)
        if (g == 0) {
            bool okd = ok && warp_wait(dfull, 0, &abort_flag);
            if (okd) {
                tmem_fence_after();
#pragma unroll 1
                for (int c0 = 0; c0 < TN; c0 += 32) {
                    uint32_t v[32];
                    tmem_ld_x32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                    if (row_ok) {
#pragma unroll
                        for (int jj = 0; jj < 32; jj++) {
                            int t = t0 + c0 + jj;
                            if (t < T) {
                                float o = __uint_as_float(v[jj]);
                                if (splits > 1) {
                                    partial[((size_t)split * T + t) * N + n] = o;
                                } else {
                                    if (epi == EPI_ADD && res) o = o + res[(size_t)t * ldres + n];
                                    y[(size_t)t * ldy + n] = o;
                                }
                            }
                        }
                    }
                }
            }
        }
    }
    tmem_fence_before();
    __syncthreads();
    if (warp == 2) {
        tmem_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
    if (threadIdx.x == 0 && abort_flag) atomicExch(err, 1);
}

// y[t][n] = (res[t][n] +) sum_s partial[s][t][n], in split order.
__global__ void k_splitk_reduce(const float* __restrict__ partial, int splits, int T, int N, float* y, size_t ldy,
                                int epi, const float* res, size_t ldres) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)T * N) return;
    int t = (int)(i / N), n = (int)(i % N);
    float o = partial[i];
    for (int sp = 1; sp < splits; sp++) o += partial[(size_t)sp * T * N + i];
    if (epi == EPI_ADD && res) o = o + res[(size_t)t * ldres + n];
    y[(size_t)t * ldy + n] = o;
}

// fp32 rows -> fp16 rows in the K order of the weight tiles (see deq_pair):
// within every 8 elements, [e0 e4 e1 e5 e2 e6 e3 e7].
__global__ void k_rows_to_f16_perm(const float* __restrict__ x, size_t ldx, __half* __restrict__ out, int K, int T) {
    int t = blockIdx.y;
    const float* xr = x + (size_t)t * ldx;
    __half2* o = reinterpret_cast<__half2*>(out + (size_t)t * K);
    for (int gi = blockIdx.x * blockDim.x + threadIdx.x; gi < K / 8; gi += gridDim.x * blockDim.x) {
        const float* e = xr + 8 * gi;
#pragma unroll
        for (int k = 0; k < 4; k++) o[4 * gi + k] = __floats2half2_rn(e[k], e[k + 4]);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
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

}  // namespace

struct GemmWorkspace {
    std::mutex mu;
    uint64_t generation = 0;  // bumped whenever a buffer a launch refers to moves
    __half* xh = nullptr;
    size_t xh_cap = 0;
    float* part = nullptr;    // split-K partial sums
    size_t part_cap = 0;
    int* err = nullptr;
    int device = -1;
    std::map<std::tuple<const void*, size_t, size_t>, CUtensorMap> wmaps;  // (nibble plane, n, k)
};

GemmWorkspace* gemm_workspace_new() { return new GemmWorkspace(); }

void gemm_workspace_free(GemmWorkspace* ws) {
    if (!ws) return;
    if (ws->xh) cudaFree(ws->xh);
    if (ws->part) cudaFree(ws->part);
    if (ws->err) cudaFree(ws->err);
    delete ws;
}

bool gemm_tc_eligible(const hc_q4_matrix& w, size_t tokens) {
    return tokens >= 2 && w.k % BK == 0 && w.n >= BM && w.nblocks >= w.n * (w.k / 32) && w.k <= (1u << 20);
}

namespace {
template <int TN>
int launch_tc(const hc_q4_matrix& w, const CUtensorMap& xmap, const CUtensorMap& wmap, size_t T, float* y,
              size_t ldy, int epi, const float* res, size_t ldres, int splits, float* partial, int* err,
              cudaStream_t s) {
    using C = Cfg<TN>;
    static_assert(C::smem() <= 232448, "shared memory budget");
    auto kfn = k_q4_gemm_tc<TN>;
    // At least 116 KB of shared memory keeps one CTA per SM, so two CTAs never
    // contend for the 512 tensor-memory columns each allocates.
    const int smem = C::smem() < 118784 ? 118784 : C::smem();
    HC_CUDA(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    dim3 grid((unsigned)((w.n + BM - 1) / BM), (unsigned)((T + TN - 1) / TN), (unsigned)splits);
    kfn<<<grid, GEMM_THREADS, smem, s>>>(xmap, wmap, w.sc, y, ldy, res, ldres, epi, (int)w.n, (int)w.k, (int)T, splits,
                                         partial, err);
    HC_LAUNCH_CHECK();
    if (splits > 1) {
        size_t tot = T * w.n;
        k_splitk_reduce<<<(unsigned)((tot + 255) / 256), 256, 0, s>>>(partial, splits, (int)T, (int)w.n, y, ldy, epi,
                                                                        res, ldres);
        HC_LAUNCH_CHECK();
    }
    return HC_OK;
}

// Split K so that row tiles x token tiles x splits fills the 148 SMs
// (one CTA per SM) without splits shorter than 4 pipeline stages.
int choose_splits(size_t tiles, size_t nk) {
    const size_t sms = 148;
    if (tiles >= sms) return 1;
    size_t best = 1;
    double best_eff = (double)tiles / (double)sms;
    for (size_t sp = 2; sp <= 16 && nk / sp >= 4; sp++) {
        size_t ctas = tiles * sp;
        size_t waves = (ctas + sms - 1) / sms;
        double eff = (double)ctas / (double)(waves * sms);
        if (eff > best_eff + 1e-9) {
            best_eff = eff;
            best = sp;
        }
    }
    return (int)best;
}
}  // namespace

int gemm_tc(GemmWorkspace* ws, const hc_q4_matrix& w, const float* x, size_t ldx, size_t tokens, float* y,
            size_t ldy, int epi, const float* res, size_t ldres, cudaStream_t s) {
    std::lock_guard<std::mutex> lock(ws->mu);
    const size_t K = w.k, T = tokens;
    int dev = 0;
    HC_CUDA(cudaGetDevice(&dev));
    if (ws->device != dev) {  // buffers belong to one device
        ws->xh = nullptr;
        ws->xh_cap = 0;
        ws->err = nullptr;
        ws->wmaps.clear();
        ws->device = dev;
    }
    if (!ws->err) {
        HC_CUDA(cudaMalloc((void**)&ws->err, sizeof(int)));
        HC_CUDA(cudaMemset(ws->err, 0, sizeof(int)));
    }
    if (T * K > ws->xh_cap) {
        if (ws->xh) cudaFree(ws->xh);
        ws->xh = nullptr;
        ws->generation++;
        HC_CUDA(cudaMalloc((void**)&ws->xh, T * K * sizeof(__half)));
        ws->xh_cap = T * K;
    }
    {
        unsigned gx = (unsigned)std::min<size_t>((K / 8 + 255) / 256, 16);
        k_rows_to_f16_perm<<<dim3(gx, (unsigned)T), 256, 0, s>>>(x, ldx, ws->xh, (int)K, (int)T);
        HC_LAUNCH_CHECK();
    }
    // Token tile: the smallest of 32/64/128/256 covering T (one tile for decode).
    int tn = T <= 32 ? 32 : T <= 64 ? 64 : T <= 128 ? 128 : 256;
    CUtensorMap xmap;
    HC_TRY(encode_2d(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, ws->xh, K, T, K * 2, 64, (uint32_t)tn,
                     CU_TENSOR_MAP_SWIZZLE_128B));
    auto key = std::make_tuple((const void*)w.qs, w.n, w.k);
    auto itw = ws->wmaps.find(key);
    CUtensorMap wmap;
    if (itw != ws->wmaps.end()) {
        wmap = itw->second;
    } else {
        HC_TRY(encode_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.qs, K / 2, w.n, K / 2, BK / 2, BM,
                         CU_TENSOR_MAP_SWIZZLE_NONE));
        if (w.owns) ws->wmaps[key] = wmap;
    }
    size_t tiles = ((w.n + BM - 1) / BM) * ((T + tn - 1) / tn);
    int splits = choose_splits(tiles, K / BK);
    if (splits > 1 && (size_t)splits * T * w.n > ws->part_cap) {
        if (ws->part) cudaFree(ws->part);
        ws->part = nullptr;
        ws->part_cap = 0;
        ws->generation++;
        HC_CUDA(cudaMalloc((void**)&ws->part, (size_t)splits * T * w.n * sizeof(float)));
        ws->part_cap = (size_t)splits * T * w.n;
    }
    switch (tn) {
        case 32: return launch_tc<32>(w, xmap, wmap, T, y, ldy, epi, res, ldres, splits, ws->part, ws->err, s);
        case 64: return launch_tc<64>(w, xmap, wmap, T, y, ldy, epi, res, ldres, splits, ws->part, ws->err, s);
        case 128: return launch_tc<128>(w, xmap, wmap, T, y, ldy, epi, res, ldres, splits, ws->part, ws->err, s);
        default: return launch_tc<256>(w, xmap, wmap, T, y, ldy, epi, res, ldres, splits, ws->part, ws->err, s);
    }
}

uint64_t gemm_generation(GemmWorkspace* ws) { return ws ? ws->generation : 0; }

int gemm_check(GemmWorkspace* ws) {
    if (!ws || !ws->err) return HC_OK;
    int h = 0;
    HC_CUDA(cudaMemcpy(&h, ws->err, sizeof(int), cudaMemcpyDeviceToHost));
    if (h) {
        HC_CUDA(cudaMemset(ws->err, 0, sizeof(int)));
        hc_set_error("tcgen05 GEMM: a pipeline wait timed out (the kernel aborted and skipped its stores)");
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
// tensor-core matmul below keeps its scratch (the fp16 copy of the
// activations and the pipeline abort flag) in a fixed array that lives in the
// library's device image, so a call allocates nothing.
namespace {

// Stated maximum: 8 MiB per device, held by every GPU that loads the library
// until the process exits.  tokens * k * 2 bytes must fit after the flag.
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
constexpr size_t kNoAllocFlagBytes = 256;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
uint8_t* g_noalloc_ptr[kMaxDevices] = {nullptr};
std::mutex g_noalloc_mu;

// Device address of the array for the current device.  In host code the
// symbol is only a host-side stand-in, never a device address, so the address
// is looked up with cudaGetSymbolAddress once per device (with that device
// current) and cached.
int noalloc_scratch(uint8_t** out) {
    int dev = 0;
    HC_CUDA(cudaGetDevice(&dev));
    HC_CHECK(dev >= 0 && dev < kMaxDevices, HC_ERR_UNSUPPORTED, "device index %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return hc_cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)", __FILE__, __LINE__);
        g_noalloc_ptr[dev] = static_cast<uint8_t*>(p);
    }
    *out = g_noalloc_ptr[dev];
    return HC_OK;
}

}  // namespace

// Y[mtok x n] = X[mtok x k] . W^T like hc_q4_matmul_dev, without allocating
// device or host memory: shapes the tensor cores take (mtok >= 2, k % 128 ==
// 0, n >= 128) run the tcgen05 kernel with its scratch in the fixed array and
// no split-K; other shapes run the CUDA-core matvec, which needs no scratch.
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
    HC_CHECK(T <= (kNoAllocScratchBytes - kNoAllocFlagBytes) / (K * sizeof(__half)), HC_ERR_INVALID,
             "hc_q4_matmul_noalloc: %zu tokens x %zu columns exceed the fixed %zu-byte scratch (at most %zu tokens "
             "at this width)",
             T, K, kNoAllocScratchBytes, (kNoAllocScratchBytes - kNoAllocFlagBytes) / (K * sizeof(__half)));
    uint8_t* base = nullptr;
    HC_TRY(noalloc_scratch(&base));
    int* err = reinterpret_cast<int*>(base);
    __half* xh = reinterpret_cast<__half*>(base + kNoAllocFlagBytes);
    // The array keeps the previous call's contents: the abort flag must start at zero.
    HC_CUDA(cudaMemsetAsync(err, 0, sizeof(int), s));
    {
        unsigned gx = (unsigned)std::min<size_t>((K / 8 + 255) / 256, 16);
        hc::k_rows_to_f16_perm<<<dim3(gx, (unsigned)T), 256, 0, s>>>(x, K, xh, (int)K, (int)T);
        HC_LAUNCH_CHECK();
    }
    int tn = T <= 32 ? 32 : T <= 64 ? 64 : T <= 128 ? 128 : 256;
    CUtensorMap xmap, wmap;
    HC_TRY(hc::encode_2d(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xh, K, T, K * 2, 64, (uint32_t)tn,
                         CU_TENSOR_MAP_SWIZZLE_128B));
    HC_TRY(hc::encode_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, w->qs, K / 2, w->n, K / 2, hc::BK / 2, hc::BM,
                         CU_TENSOR_MAP_SWIZZLE_NONE));
    switch (tn) {
        case 32: return hc::launch_tc<32>(*w, xmap, wmap, T, y, w->n, hc::EPI_STORE, nullptr, 0, 1, nullptr, err, s);
        case 64: return hc::launch_tc<64>(*w, xmap, wmap, T, y, w->n, hc::EPI_STORE, nullptr, 0, 1, nullptr, err, s);
        case 128: return hc::launch_tc<128>(*w, xmap, wmap, T, y, w->n, hc::EPI_STORE, nullptr, 0, 1, nullptr, err, s);
        default: return hc::launch_tc<256>(*w, xmap, wmap, T, y, w->n, hc::EPI_STORE, nullptr, 0, 1, nullptr, err, s);
    }
}

