// Device helpers shared by the kernels of libhypno_cuda.so.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace hc {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum for blockDim.x a multiple of 32 and <= 1024.  `red` holds
// 32 floats of shared memory.  Every thread receives the total.
// ---- mbarrier helpers (shared memory, CTA scope) for the TMA pipelines

constexpr long long WAIT_CYCLES = 4000000000LL;  // bound of every pipeline wait, ~2 s at 1.9 GHz

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

// Non-blocking probe of the phase with the given parity (try_wait may
// suspend the thread for a while when the phase is still open; test_wait
// returns at once).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on the phase with the given parity.  Returns false when the
// deadline passes or another role already reported a failure.  Waits that are
// off the critical path pass sleep_ns > 0 and back off between probes, which
// leaves the issue slots of their SMSP to the warps doing the work.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          unsigned sleep_ns = 0) {
    long long start = clock64();
    for (uint32_t i = 0;; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if (sleep_ns) __nanosleep(sleep_ns);
        if ((i & 255) == 255) {
            if (*abort_flag) return false;
            if (clock64() - start > WAIT_CYCLES) {
                *abort_flag = 1;
                return false;
            }
        }
    }
}

// Programmatic dependent launch: lets the next kernel in the stream, when it
// is launched as a programmatic dependent (the tensor-core GEMM), start its
// prologue and weight prefetch now; it waits for this grid's completion
// before it touches anything this grid writes.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// The other side: a kernel launched as a programmatic dependent (launch_pdl)
// may start while the previous kernel still runs; it calls this before its
// first global memory access, which returns once that kernel has completed
// and its writes are visible (a no-op for an ordinary launch).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ float block_sum(float v, float* red) {
    int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    int nw = blockDim.x >> 5;
    float t = (lane < nw) ? red[lane] : 0.0f;
    t = warp_sum(t);
    return t;
}

__device__ __forceinline__ float block_max(float v, float* red) {
    int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    int nw = blockDim.x >> 5;
    float t = (lane < nw) ? red[lane] : -INFINITY;
    t = warp_max(t);
    return t;
}

// The 4th-order Taylor polynomial of exp(v/8) that the reference's AVX2
// softmax uses for lanes below floor(n/8)*8 (kernels.rs:673-697): clamp to
// [-87, 87], x2 = v*v, x3 = x2*v, x4 = x3*v, then the fma chain
// 1 + c1 v -> + c2 x2 -> + c3 x3 -> + c4 x4.  Explicit _rn intrinsics keep
// the exact operation sequence (no contraction or reassociation).
__device__ __forceinline__ float poly_exp8(float v) {
    v = fminf(fmaxf(v, -87.0f), 87.0f);
    const float c1 = 1.0f / 8.0f, c2 = 1.0f / 128.0f, c3 = 1.0f / 3072.0f, c4 = 1.0f / 98304.0f;
    float x2 = __fmul_rn(v, v);
    float x3 = __fmul_rn(x2, v);
    float x4 = __fmul_rn(x3, v);
    float t1 = __fmaf_rn(c1, v, 1.0f);
    float t2 = __fmaf_rn(c2, x2, t1);
    float t3 = __fmaf_rn(c3, x3, t2);
    return __fmaf_rn(c4, x4, t3);
}

// Weight of entry i of an n-long softmax row before normalisation
// (kernels.rs:642-652): polynomial on the 8-lane body, libm exp on the tail.
// x / (1 + exp(-x)) as the reference computes it (transformer.rs:446-449)
__device__ __forceinline__ float silu_f(float v) { return __fdiv_rn(v, __fadd_rn(1.0f, expf(-v))); }

__device__ __forceinline__ float softmax_weight(float s, float mx, int i, int n8) {
    float d = __fsub_rn(s, mx);
    return (i < n8) ? poly_exp8(d) : expf(d);
}

// 64-bit SplitMix finaliser (integer only).
__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Element `idx` of the seeded normal stream: 12 16-bit uniforms from three
// hashes, summed exactly as integers, centred, converted (exactly, |z| < 2^20)
// and scaled by one IEEE multiply.  Identical on host and device.
__host__ __device__ __forceinline__ float synth_normal(uint64_t key, uint64_t idx, float scale) {
    uint32_t s = 0;
#pragma unroll
    for (int j = 0; j < 3; j++) {
        uint64_t h = splitmix64(key + 3ull * idx + (uint64_t)j);
        s += (uint32_t)(h & 0xFFFF) + (uint32_t)((h >> 16) & 0xFFFF) + (uint32_t)((h >> 32) & 0xFFFF) +
             (uint32_t)(h >> 48);
    }
    int32_t z = (int32_t)s - 393210;
#ifdef __CUDA_ARCH__
    return __fmul_rn((float)z, scale);
#else
    return (float)z * scale;
#endif
}

__host__ __device__ __forceinline__ uint64_t synth_key(uint64_t seed, uint64_t stream) {
    return splitmix64(seed * 0x100000001B3ull ^ splitmix64(stream + 0x51ED270B2ull));
}

}  // namespace hc
