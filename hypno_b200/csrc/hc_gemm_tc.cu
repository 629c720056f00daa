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
constexpr int NTHREADS = 384;
constexpr int TMEM_COLS = 512;
constexpr int D_COL = 256;   // accumulator column base; A stages use [0, 64 * STAGES)
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

__device__ __forceinline__ void tmem_st_x32(uint32_t taddr, const uint32_t* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
        "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
        "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}

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

// Two nibbles (low = element 2j, high = element 2j+1 of byte j) -> fp16x2 of
// (nib - 8) * scale, the low half holding the lower K index.  1024 + nib is
// exact in fp16 (0x6400 | nib); subtracting 1032 is exact; the product by the
// fp16 scale rounds once, like converting the exact f32 product to fp16.
__device__ __forceinline__ uint32_t deq_pair(uint32_t lo_nibs, uint32_t hi_nibs, int j, __half2 s2) {
    uint32_t sel = (uint32_t)j | ((uint32_t)(j + 4) << 8);  // byte0 <- lo byte j, byte2 <- hi byte j
    uint32_t v = __byte_perm(lo_nibs, hi_nibs, sel) & 0x000F000Fu;
    v |= 0x64006400u;
    __half2 h = *reinterpret_cast<__half2*>(&v);
    h = __hsub2(h, __float2half2_rn(1032.0f));
    h = __hmul2(h, s2);
    return *reinterpret_cast<uint32_t*>(&h);
}

struct SmemLayout {
    int stages, tn;
    __host__ __device__ constexpr int x_stage_bytes() const { return 2 * tn * 128; }
    __host__ __device__ constexpr int w_stage_bytes() const { return BM * (BK / 2); }
    __host__ __device__ constexpr int x_off(int s) const { return s * x_stage_bytes(); }
    __host__ __device__ constexpr int w_off(int s) const { return stages * x_stage_bytes() + s * w_stage_bytes(); }
    __host__ __device__ constexpr int bar_off() const { return stages * (x_stage_bytes() + w_stage_bytes()); }
    __host__ __device__ constexpr int total() const { return bar_off() + (3 * stages + 1) * 8 + 16 + 1024; }
};

template <int TN, int STAGES>
__global__ void __launch_bounds__(NTHREADS, 1)
    k_q4_gemm_tc(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                 const __half* __restrict__ scales, float* __restrict__ y, size_t ldy, const float* res, size_t ldres,
                 int epi, int N, int K, int T, int* __restrict__ err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    constexpr SmemLayout L{STAGES, TN};
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off());
    uint64_t* aready = full + STAGES;
    uint64_t* empty = aready + STAGES;
    uint64_t* dfull = empty + STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dfull + 1);
    __shared__ int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BM, t0 = blockIdx.y * TN;
    const int KB = K / 32;
    const int nk = K / BK;

    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&aready[s], 8);
            mbar_init(&empty[s], 1);
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
            for (int it = 0; it < nk; it++) {
                int s = it % STAGES;
                uint32_t ph = (uint32_t)(it / STAGES) & 1u;
                if (!mbar_wait(&empty[s], ph ^ 1u, &abort_flag)) break;
                mbar_expect_tx(&full[s], (uint32_t)(L.x_stage_bytes() + L.w_stage_bytes()));
                uint8_t* xs = smem + L.x_off(s);
                tma_load_2d(xs, &xmap, &full[s], it * BK, t0);
                tma_load_2d(xs + TN * 128, &xmap, &full[s], it * BK + 64, t0);
                tma_load_2d(smem + L.w_off(s), &wmap, &full[s], it * (BK / 2), n0);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = make_idesc(TN);
            const uint32_t d_tmem = tmem + D_COL;
            bool ok = true;
            for (int it = 0; it < nk && ok; it++) {
                int s = it % STAGES;
                uint32_t ph = (uint32_t)(it / STAGES) & 1u;
                if (!mbar_wait(&aready[s], ph, &abort_flag)) {
                    ok = false;
                    break;
                }
                tmem_fence_after();
                const uint32_t xs = smem_u32(smem + L.x_off(s));
#pragma unroll
                for (int kk = 0; kk < BK / 16; kk++) {
                    uint32_t a_tmem = tmem + (uint32_t)(s * 64 + kk * 8);
                    uint32_t b_addr = xs + (uint32_t)((kk >> 2) * TN * 128 + (kk & 3) * 32);
                    mma_f16_ts(d_tmem, a_tmem, sw128_desc(b_addr), idesc, (it > 0 || kk > 0) ? 1u : 0u);
                }
                mma_commit(&empty[s]);
            }
            if (ok) mma_commit(dfull);
        }
    } else if (warp >= 4) {
        // ---------------- dequant: thread <-> weight row (TMEM lane)
        const int g = (warp - 4) >> 2;   // warpgroup: K half of the stage
        const int q = warp & 3;          // TMEM lane quarter accessible to this warp
        const int r = q * 32 + lane;     // row within the tile
        const int n = n0 + r;
        const bool row_ok = n < N;
        const __half* srow = scales + (size_t)(row_ok ? n : 0) * KB;
        uint32_t sc_next = row_ok ? __ldg(reinterpret_cast<const unsigned int*>(srow + 2 * g)) : 0u;
        bool ok = true;
        for (int it = 0; it < nk; it++) {
            int s = it % STAGES;
            uint32_t ph = (uint32_t)(it / STAGES) & 1u;
            uint32_t sc = sc_next;
            if (it + 1 < nk && row_ok)
                sc_next = __ldg(reinterpret_cast<const unsigned int*>(srow + (it + 1) * (BK / 32) + 2 * g));
            bool w1 = mbar_wait(&empty[s], ph ^ 1u, &abort_flag);
            bool w2 = w1 && mbar_wait(&full[s], ph, &abort_flag);
            if (!__all_sync(0xffffffffu, w2)) {
                ok = false;
                break;
            }
            const uint4* nib = reinterpret_cast<const uint4*>(smem + L.w_off(s) + r * (BK / 2) + g * 32);
            uint32_t v[32];
#pragma unroll
            for (int b = 0; b < 2; b++) {  // two Q4_0 blocks of 32 elements
                uint4 q4 = nib[b];
                __half2 s2 = __half2half2(__ushort_as_half((uint16_t)(b == 0 ? (sc & 0xFFFF) : (sc >> 16))));
                uint32_t w4[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
                for (int wd = 0; wd < 4; wd++) {
                    uint32_t lo = w4[wd] & 0x0F0F0F0Fu, hi = (w4[wd] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
                    for (int j = 0; j < 4; j++) v[b * 16 + wd * 4 + j] = deq_pair(lo, hi, j, s2);
                }
            }
            uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(s * 64 + g * 32);
            tmem_st_x32(taddr, v);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tmem_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&aready[s]);
        }
        // ---------------- epilogue (first dequant warpgroup)
        if (g == 0) {
            bool okd = ok && mbar_wait(dfull, 0, &abort_flag);
            okd = __all_sync(0xffffffffu, okd);
            if (okd) {
                tmem_fence_after();
#pragma unroll 1
                for (int c0 = 0; c0 < TN; c0 += 32) {
                    uint32_t v[32];
                    tmem_ld_x32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(D_COL + c0), v);
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                    if (row_ok) {
#pragma unroll
                        for (int j = 0; j < 32; j++) {
                            int t = t0 + c0 + j;
                            if (t < T) {
                                float o = __uint_as_float(v[j]);
                                if (epi == EPI_ADD && res) o = o + res[(size_t)t * ldres + n];
                                y[(size_t)t * ldy + n] = o;
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

// fp32 rows -> fp16 rows (the B operand of the MMA).
__global__ void k_rows_to_f16(const float* __restrict__ x, size_t ldx, __half* __restrict__ out, int K, int T) {
    int t = blockIdx.y;
    const float* xr = x + (size_t)t * ldx;
    __half2* o = reinterpret_cast<__half2*>(out + (size_t)t * K);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < K / 2; i += gridDim.x * blockDim.x)
        o[i] = __floats2half2_rn(xr[2 * i], xr[2 * i + 1]);
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

template <int TN, int STAGES>
int launch_tc(GemmWorkspace* ws, const hc_q4_matrix& w, const CUtensorMap& xmap, const CUtensorMap& wmap, size_t T,
              float* y, size_t ldy, int epi, const float* res, size_t ldres, int* err, cudaStream_t s);

}  // namespace

struct GemmWorkspace {
    std::mutex mu;
    uint64_t generation = 0;  // bumped whenever a buffer a launch refers to moves
    __half* xh = nullptr;
    size_t xh_cap = 0;
    int* err = nullptr;
    int device = -1;
    std::map<std::tuple<const void*, size_t, size_t>, CUtensorMap> wmaps;  // (nibble plane, n, k)
};

GemmWorkspace* gemm_workspace_new() { return new GemmWorkspace(); }

void gemm_workspace_free(GemmWorkspace* ws) {
    if (!ws) return;
    if (ws->xh) cudaFree(ws->xh);
    if (ws->err) cudaFree(ws->err);
    delete ws;
}

bool gemm_tc_eligible(const hc_q4_matrix& w, size_t tokens) {
    return tokens >= 2 && w.k % BK == 0 && w.n >= BM && w.nblocks >= w.n * (w.k / 32) && w.k <= (1u << 20);
}

namespace {
template <int TN, int STAGES>
int launch_tc(GemmWorkspace* ws, const hc_q4_matrix& w, const CUtensorMap& xmap, const CUtensorMap& wmap, size_t T,
              float* y, size_t ldy, int epi, const float* res, size_t ldres, int* err, cudaStream_t s) {
    constexpr SmemLayout L{STAGES, TN};
    static_assert(L.total() <= 232448, "shared memory budget");
    auto kfn = k_q4_gemm_tc<TN, STAGES>;
    // At least 116 KB of shared memory keeps one CTA per SM, so two CTAs never
    // contend for the 512 tensor-memory columns each allocates.
    const int smem = L.total() < 118784 ? 118784 : L.total();
    HC_CUDA(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    dim3 grid((unsigned)((w.n + BM - 1) / BM), (unsigned)((T + TN - 1) / TN));
    kfn<<<grid, NTHREADS, smem, s>>>(xmap, wmap, w.sc, y, ldy, res, ldres, epi, (int)w.n, (int)w.k, (int)T, err);
    HC_LAUNCH_CHECK();
    return HC_OK;
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
        unsigned gx = (unsigned)std::min<size_t>((K / 2 + 255) / 256, 16);
        k_rows_to_f16<<<dim3(gx, (unsigned)T), 256, 0, s>>>(x, ldx, ws->xh, (int)K, (int)T);
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
    switch (tn) {
        case 32: return launch_tc<32, 4>(ws, w, xmap, wmap, T, y, ldy, epi, res, ldres, ws->err, s);
        case 64: return launch_tc<64, 4>(ws, w, xmap, wmap, T, y, ldy, epi, res, ldres, ws->err, s);
        case 128: return launch_tc<128, 4>(ws, w, xmap, wmap, T, y, ldy, epi, res, ldres, ws->err, s);
        default: return launch_tc<256, 3>(ws, w, xmap, wmap, T, y, ldy, epi, res, ldres, ws->err, s);
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
