// Placeholder until the tcgen05 path lands: every Q4_0 matmul runs on the
// CUDA-core kernels of hc_kernels.cu.
#include "hc_gemm.h"

namespace hc {
struct GemmWorkspace {
    int unused = 0;
};
GemmWorkspace* gemm_workspace_new() { return new GemmWorkspace(); }
void gemm_workspace_free(GemmWorkspace* ws) { delete ws; }
bool gemm_tc_eligible(const hc_q4_matrix&, size_t) { return false; }
int gemm_tc(GemmWorkspace*, const hc_q4_matrix&, const float*, size_t, size_t, float*, size_t, int, const float*,
            size_t, cudaStream_t) {
    hc_set_error("tcgen05 GEMM not built");
    return HC_ERR_UNSUPPORTED;
}
}  // namespace hc
