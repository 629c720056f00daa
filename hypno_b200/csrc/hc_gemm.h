// Tensor-core (tcgen05) Q4_0 GEMM interface (see hc_gemm_tc.cu).
#pragma once
#include "hc_internal.h"

namespace hc {

struct GemmWorkspace;
GemmWorkspace* gemm_workspace_new();
void gemm_workspace_free(GemmWorkspace* ws);

// True when Y = X . W^T for `tokens` rows should run on the tcgen05 path.
bool gemm_tc_eligible(const hc_q4_matrix& w, size_t tokens);

// Y[t][n] (+)= sum_k X[t][k] * deq(W)[n][k] for t < tokens, fp16 operands and
// f32 accumulation in tensor memory; same epilogue contract as launch_matmul.
// xh_ready: the same activations already in fp16, rows of k elements in the
// GEMM's K order (within every 8 elements: e0 e4 e1 e5 e2 e6 e3 e7); when
// null, x is converted first.
int gemm_tc(GemmWorkspace* ws, const hc_q4_matrix& w, const float* x, size_t ldx, size_t tokens, float* y,
            size_t ldy, int epi, const float* res, size_t ldres, cudaStream_t s, const __half* xh_ready = nullptr);

// act[t][i] = silu(gate_i . x_t) * (up_i . x_t) for a fused gate/up weight
// whose rows alternate in blocks of GU_BLOCK (gate rows, then the matching up
// rows), computed in the GEMM epilogue; act16 (may be null) gets the fp16
// copy in the GEMM K order.  act has w.n / 2 columns (row stride ldact).
int gemm_tc_silu(GemmWorkspace* ws, const hc_q4_matrix& w, const float* x, size_t ldx, size_t tokens, float* act,
                 size_t ldact, __half* act16, cudaStream_t s, const __half* xh_ready = nullptr);

// The same product with K split over up to max_splits CTAs per tile whose
// partial products are NOT added here: split i writes its [tokens][n] slab
// at part + i * tokens * n; *splits reports how many slabs were written (the
// caller adds them in slab order, e.g. launch_residual_splits_norm).
int gemm_tc_partials(GemmWorkspace* ws, const hc_q4_matrix& w, const float* x, size_t ldx, size_t tokens,
                     float* part, int max_splits, int* splits, cudaStream_t s, const __half* xh_ready = nullptr);

// Index of element e of a row in the GEMM's fp16 K order.
__host__ __device__ inline int perm_k(int e) { return (e & ~7) | ((e & 3) << 1) | ((e >> 2) & 1); }

#ifdef __CUDACC__
// The tensor-core GEMM reads its activations as one row of 2k fp16 values per
// token: hi = fp16(v) in the first k, lo = fp16(v - hi) in the second k (both
// in perm_k order).  v - hi is exact in f32, so hi + lo carries v to ~22
// significant bits: the products of the exact two-term weights with hi and
// lo keep the GEMM within ~1e-6 of an f32 dot product, where one fp16 operand
// would leave errors of ~3e-4 per product.
__device__ __forceinline__ void store_x16(__half* row, int k, int e, float v) {
    const __half h = __float2half_rn(v);
    const int p = perm_k(e);
    row[p] = h;
    row[k + p] = __float2half_rn(__fsub_rn(v, __half2float(h)));
}
#endif

// Reads and clears the device flag set by a timed-out pipeline wait
// (synchronizes the device); HC_ERR_TIMEOUT when a kernel aborted.
int gemm_check(GemmWorkspace* ws);

// The workspace's device error flag (allocated on first use; null when that
// fails): other pipelined kernels report expired waits through it too, so
// gemm_check covers them.
int* gemm_error_flag(GemmWorkspace* ws);

// Changes whenever a workspace buffer captured by earlier launches moved
// (captured CUDA graphs must then be rebuilt).
uint64_t gemm_generation(GemmWorkspace* ws);

}  // namespace hc
