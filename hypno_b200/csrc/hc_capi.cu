// Library-level and op-level C ABI of libhypno_cuda.so: error reporting, the
// drop-in replacements of ops.rs / quant.rs entry points on host slices, the
// device-resident Q4_0 matrix, and the seeded synthetic generator.
#include "hc_internal.h"
#include "hc_common.cuh"
#include "hc_gemm.h"

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>
#include <string>

// ============================================================ errors

static thread_local std::string g_err;

void hc_set_error(const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
}

int hc_cuda_fail(cudaError_t e, const char* what, const char* file, int line) {
    hc_set_error("CUDA error %d (%s) in %s at %s:%d", (int)e, cudaGetErrorString(e), what, file, line);
    // Clear a sticky launch error so the next call starts clean when possible.
    cudaGetLastError();
    return HC_ERR_CUDA;
}

HC_EXPORT const char* hc_last_error(void) { return g_err.c_str(); }

static std::atomic<unsigned long long> g_launches{0};
void hc_count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
void hc_count_launches(size_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
HC_EXPORT uint64_t hc_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

HC_EXPORT int hc_version(void) { return 100; }

HC_EXPORT int hc_set_device(int device) {
    HC_CUDA(cudaSetDevice(device));
    return HC_OK;
}

// ============================================================ device scratch
// Per-thread growable device buffers used by the host-slice entry points so
// repeated calls do not allocate.
namespace {
struct HostCallScratch {
    int device = -1;
    void* buf[4] = {nullptr, nullptr, nullptr, nullptr};
    size_t cap[4] = {0, 0, 0, 0};
    ~HostCallScratch() {
        for (void* p : buf)
            if (p) cudaFree(p);
    }
};
thread_local HostCallScratch t_scratch;

int scratch(int i, size_t bytes, void** out) {
    cudaGetLastError();  // host-slice entry points start from a clean error state
    int dev = 0;
    HC_CUDA(cudaGetDevice(&dev));
    if (t_scratch.device != dev) {
        for (int j = 0; j < 4; j++) {
            t_scratch.buf[j] = nullptr;  // buffers of another device are left to process exit
            t_scratch.cap[j] = 0;
        }
        t_scratch.device = dev;
    }
    if (bytes > t_scratch.cap[i]) {
        if (t_scratch.buf[i]) cudaFree(t_scratch.buf[i]);
        t_scratch.buf[i] = nullptr;
        t_scratch.cap[i] = 0;
        size_t b = bytes < 256 ? 256 : bytes;
        cudaError_t e = cudaMalloc(&t_scratch.buf[i], b);
        if (e != cudaSuccess) {
            cudaGetLastError();
            hc_set_error("device scratch allocation of %zu bytes failed: %s", b, cudaGetErrorString(e));
            return e == cudaErrorMemoryAllocation ? HC_ERR_OOM : HC_ERR_CUDA;
        }
        t_scratch.cap[i] = b;
    }
    *out = t_scratch.buf[i];
    return HC_OK;
}

// Uploads an .hypno weight payload as a DevWeight backed by scratch slot 0/3.
int stage_weight(const uint8_t* w, size_t w_len, uint32_t dtype, size_t n, size_t m, DevWeight& dw) {
    dw = DevWeight{};
    dw.dtype = dtype;
    dw.n = n;
    dw.k = m;
    dw.present = true;
    if (dtype == HC_DTYPE_Q4_0) {
        size_t nb = w_len / 18;
        void *aos, *planes;
        HC_TRY(scratch(0, nb * 18 + 16, &aos));
        HC_TRY(scratch(3, nb * 18 + 64, &planes));
        HC_CUDA(cudaMemcpy(aos, w, nb * 18, cudaMemcpyHostToDevice));
        dw.q4.n = n;
        dw.q4.k = m;
        dw.q4.nblocks = nb;
        dw.q4.qs = (uint4*)planes;
        dw.q4.sc = (__half*)((uint8_t*)planes + ((nb * 16 + 63) / 64) * 64);
        dw.q4.owns = false;
        HC_TRY(hc::launch_q4_split((const uint8_t*)aos, nb, dw.q4.qs, dw.q4.sc, 0));
        return HC_OK;
    }
    size_t es = dtype == HC_DTYPE_FP32 ? 4 : (dtype == HC_DTYPE_FP16 ? 2 : 0);
    HC_CHECK(es != 0, HC_ERR_UNSUPPORTED, "dtype %u (Q8_0) is not supported by the GPU backend", dtype);
    HC_CHECK(w_len >= n * m * es, HC_ERR_INVALID, "weight buffer of %zu bytes is shorter than %zu x %zu", w_len, n, m);
    void* d;
    HC_TRY(scratch(0, n * m * es, &d));
    HC_CUDA(cudaMemcpy(d, w, n * m * es, cudaMemcpyHostToDevice));
    dw.dense = d;
    return HC_OK;
}
}  // namespace

// ============================================================ op level (host slices)

HC_EXPORT int hc_batch_matmul(float* y, const uint8_t* w, size_t w_len, uint32_t dtype, const float* x, size_t n,
                              size_t dim, size_t batch) {
    HC_CHECK(y && w && x, HC_ERR_INVALID, "hc_batch_matmul: NULL argument");
    if (n == 0 || batch == 0) return HC_OK;
    DevWeight dw;
    HC_TRY(stage_weight(w, w_len, dtype, n, dim, dw));
    void *dx, *dy;
    HC_TRY(scratch(1, batch * dim * 4 + 16, &dx));
    HC_TRY(scratch(2, batch * n * 4 + 16, &dy));
    HC_CUDA(cudaMemcpy(dx, x, batch * dim * 4, cudaMemcpyHostToDevice));
    int r;
    if (dtype == HC_DTYPE_Q4_0 && hc::gemm_tc_eligible(dw.q4, batch)) {
        static hc::GemmWorkspace* ws = hc::gemm_workspace_new();
        r = hc::gemm_tc(ws, dw.q4, (const float*)dx, dim, batch, (float*)dy, n, hc::EPI_STORE, nullptr, 0, 0);
        if (r == HC_OK) r = hc::gemm_check(ws);
    } else {
        r = hc::launch_matmul(dw, (const float*)dx, dim, batch, (float*)dy, n, hc::EPI_STORE, nullptr, 0, 0);
    }
    HC_TRY(r);
    HC_CUDA(cudaMemcpy(y, dy, batch * n * 4, cudaMemcpyDeviceToHost));
    return HC_OK;
}

HC_EXPORT int hc_matmul_vec_auto(float* y, const uint8_t* w, size_t w_len, uint32_t dtype, const float* x,
                                 const float* bias, size_t n, size_t m) {
    HC_CHECK(y && w && x, HC_ERR_INVALID, "hc_matmul_vec_auto: NULL argument");
    if (n == 0) return HC_OK;
    DevWeight dw;
    HC_TRY(stage_weight(w, w_len, dtype, n, m, dw));
    void *dx, *dy, *db = nullptr;
    HC_TRY(scratch(1, m * 4 + (bias ? n * 4 : 0) + 64, &dx));
    HC_TRY(scratch(2, n * 4 + 16, &dy));
    HC_CUDA(cudaMemcpy(dx, x, m * 4, cudaMemcpyHostToDevice));
    if (bias) {
        db = (uint8_t*)dx + ((m * 4 + 63) / 64) * 64;
        HC_CUDA(cudaMemcpy(db, bias, n * 4, cudaMemcpyHostToDevice));
    }
    HC_TRY(hc::launch_matmul(dw, (const float*)dx, m, 1, (float*)dy, n, bias ? hc::EPI_ADD : hc::EPI_STORE,
                             (const float*)db, 0, 0));
    HC_CUDA(cudaMemcpy(y, dy, n * 4, cudaMemcpyDeviceToHost));
    return HC_OK;
}

HC_EXPORT int hc_rms_norm_in_place(float* x, const float* w, size_t n, float eps) {
    HC_CHECK(x && w, HC_ERR_INVALID, "hc_rms_norm_in_place: NULL argument");
    if (n == 0) return HC_OK;
    void *dx, *dw;
    HC_TRY(scratch(1, n * 4, &dx));
    HC_TRY(scratch(2, n * 4, &dw));
    HC_CUDA(cudaMemcpy(dx, x, n * 4, cudaMemcpyHostToDevice));
    HC_CUDA(cudaMemcpy(dw, w, n * 4, cudaMemcpyHostToDevice));
    HC_TRY(hc::launch_rmsnorm((const float*)dx, n, (const float*)dw, (float*)dx, n, 1, n, eps, 0));
    HC_CUDA(cudaMemcpy(x, dx, n * 4, cudaMemcpyDeviceToHost));
    return HC_OK;
}

HC_EXPORT int hc_softmax_in_place(float* x, size_t n) {
    HC_CHECK(x || n == 0, HC_ERR_INVALID, "hc_softmax_in_place: NULL argument");
    if (n == 0) return HC_OK;
    void* dx;
    HC_TRY(scratch(1, n * 4, &dx));
    HC_CUDA(cudaMemcpy(dx, x, n * 4, cudaMemcpyHostToDevice));
    HC_TRY(hc::launch_softmax_rows((float*)dx, 1, n, 0));
    HC_CUDA(cudaMemcpy(x, dx, n * 4, cudaMemcpyDeviceToHost));
    return HC_OK;
}

HC_EXPORT int hc_silu_in_place(float* x, size_t n) {
    HC_CHECK(x || n == 0, HC_ERR_INVALID, "hc_silu_in_place: NULL argument");
    if (n == 0) return HC_OK;
    void* dx;
    HC_TRY(scratch(1, n * 4, &dx));
    HC_CUDA(cudaMemcpy(dx, x, n * 4, cudaMemcpyHostToDevice));
    HC_TRY(hc::launch_silu((float*)dx, n, 0));
    HC_CUDA(cudaMemcpy(x, dx, n * 4, cudaMemcpyDeviceToHost));
    return HC_OK;
}

HC_EXPORT int hc_rope(float* q, float* k, size_t head_dim, size_t pos, float theta) {
    HC_CHECK(q && k, HC_ERR_INVALID, "hc_rope: NULL argument");
    HC_CHECK(head_dim % 2 == 0, HC_ERR_INVALID, "hc_rope: head_dim must be even");
    if (head_dim == 0) return HC_OK;
    // Only the row for `pos` of the angle table is needed (same host libm
    // arithmetic as hc_rope_table).
    std::vector<float2> row(head_dim / 2);
    for (size_t j = 0; j < head_dim / 2; j++) {
        float freq = 1.0f / powf(theta, (float)(2 * j) / (float)head_dim);
        float a = (float)pos * freq;
        row[j] = make_float2(cosf(a), sinf(a));
    }
    void *dqk, *dcs;
    HC_TRY(scratch(1, head_dim * 8, &dqk));
    HC_TRY(scratch(2, head_dim * 4, &dcs));
    HC_CUDA(cudaMemcpy(dqk, q, head_dim * 4, cudaMemcpyHostToDevice));
    HC_CUDA(cudaMemcpy((float*)dqk + head_dim, k, head_dim * 4, cudaMemcpyHostToDevice));
    HC_CUDA(cudaMemcpy(dcs, row.data(), head_dim / 2 * sizeof(float2), cudaMemcpyHostToDevice));
    // q and k are two "heads" of one row at table row 0.
    HC_TRY(hc::launch_rope_rows((float*)dqk, 2 * head_dim, 1, 2, head_dim, (const float2*)dcs, 1, nullptr, 0, 0));
    HC_CUDA(cudaMemcpy(q, dqk, head_dim * 4, cudaMemcpyDeviceToHost));
    HC_CUDA(cudaMemcpy(k, (float*)dqk + head_dim, head_dim * 4, cudaMemcpyDeviceToHost));
    return HC_OK;
}

HC_EXPORT int hc_q4_0_quantize(const float* x, size_t n, uint8_t* out) {
    HC_CHECK((x && out) || n < 32, HC_ERR_INVALID, "hc_q4_0_quantize: NULL argument");
    size_t nb = n / 32;
    if (nb == 0) return HC_OK;
    void *dx, *dq;
    HC_TRY(scratch(1, nb * 128, &dx));
    HC_TRY(scratch(2, nb * 18, &dq));
    HC_CUDA(cudaMemcpy(dx, x, nb * 128, cudaMemcpyHostToDevice));
    HC_TRY(hc::launch_q4_quantize((const float*)dx, nb, (uint8_t*)dq, 0));
    HC_CUDA(cudaMemcpy(out, dq, nb * 18, cudaMemcpyDeviceToHost));
    return HC_OK;
}

HC_EXPORT int hc_q4_0_dequantize(const uint8_t* q, size_t nbytes, float* out) {
    size_t nb = nbytes / 18;
    HC_CHECK((q && out) || nb == 0, HC_ERR_INVALID, "hc_q4_0_dequantize: NULL argument");
    if (nb == 0) return HC_OK;
    void *dq, *dx;
    HC_TRY(scratch(1, nb * 18, &dq));
    HC_TRY(scratch(2, nb * 128, &dx));
    HC_CUDA(cudaMemcpy(dq, q, nb * 18, cudaMemcpyHostToDevice));
    HC_TRY(hc::launch_q4_dequantize((const uint8_t*)dq, nb, (float*)dx, 0));
    HC_CUDA(cudaMemcpy(out, dx, nb * 128, cudaMemcpyDeviceToHost));
    return HC_OK;
}

// ============================================================ op level (device)

HC_EXPORT int hc_q4_0_quantize_dev(const float* x, size_t n, uint8_t* out, void* stream) {
    HC_CHECK(((uintptr_t)x & 3) == 0, HC_ERR_INVALID, "hc_q4_0_quantize_dev: x must be 4-byte aligned");
    HC_CHECK(((uintptr_t)out & 1) == 0, HC_ERR_INVALID, "hc_q4_0_quantize_dev: out must be 2-byte aligned");
    return hc::launch_q4_quantize(x, n / 32, out, (cudaStream_t)stream);
}

HC_EXPORT int hc_q4_0_dequantize_dev(const uint8_t* q, size_t nbytes, float* out, void* stream) {
    return hc::launch_q4_dequantize(q, nbytes / 18, out, (cudaStream_t)stream);
}

static int q4_matrix_new(size_t w_len, size_t n, size_t k, hc_q4_matrix** out) {
    HC_CHECK(out, HC_ERR_INVALID, "q4 matrix: out is NULL");
    HC_CHECK(n > 0 && k > 0, HC_ERR_INVALID, "q4 matrix: empty shape");
    size_t need = (n * k + 31) / 32;
    size_t nb = w_len / 18;
    HC_CHECK(nb >= need, HC_ERR_INVALID, "q4 matrix: payload of %zu bytes holds %zu blocks, shape needs %zu", w_len, nb,
             need);
    hc_q4_matrix* m = new hc_q4_matrix();
    m->n = n;
    m->k = k;
    m->nblocks = need;
    cudaError_t e = cudaMalloc((void**)&m->qs, need * 16);
    if (e == cudaSuccess) e = cudaMalloc((void**)&m->sc, need * 2 + 16);
    if (e != cudaSuccess) {
        cudaGetLastError();
        if (m->qs) cudaFree(m->qs);
        delete m;
        hc_set_error("q4 matrix: allocation failed (%s)", cudaGetErrorString(e));
        return HC_ERR_OOM;
    }
    *out = m;
    return HC_OK;
}

HC_EXPORT int hc_q4_matrix_upload(const uint8_t* w, size_t w_len, size_t n, size_t k, hc_q4_matrix** out) {
    HC_CHECK(w, HC_ERR_INVALID, "hc_q4_matrix_upload: NULL weights");
    HC_TRY(q4_matrix_new(w_len, n, k, out));
    hc_q4_matrix* m = *out;
    void* aos;
    int r = scratch(0, m->nblocks * 18, &aos);
    if (r == HC_OK) {
        cudaError_t e = cudaMemcpy(aos, w, m->nblocks * 18, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) r = hc_cuda_fail(e, "cudaMemcpy", __FILE__, __LINE__);
    }
    if (r == HC_OK) r = hc::launch_q4_split((const uint8_t*)aos, m->nblocks, m->qs, m->sc, 0);
    if (r == HC_OK) {
        cudaError_t e = cudaDeviceSynchronize();
        if (e != cudaSuccess) r = hc_cuda_fail(e, "cudaDeviceSynchronize", __FILE__, __LINE__);
    }
    if (r != HC_OK) {
        cudaFree(m->qs);
        cudaFree(m->sc);
        delete m;
        *out = nullptr;
    }
    return r;
}

HC_EXPORT int hc_q4_matrix_from_dev(const uint8_t* w_dev, size_t w_len, size_t n, size_t k, void* stream,
                                    hc_q4_matrix** out) {
    HC_CHECK(w_dev, HC_ERR_INVALID, "hc_q4_matrix_from_dev: NULL weights");
    HC_TRY(q4_matrix_new(w_len, n, k, out));
    hc_q4_matrix* m = *out;
    int r = hc::launch_q4_split(w_dev, m->nblocks, m->qs, m->sc, (cudaStream_t)stream);
    if (r != HC_OK) {
        cudaFree(m->qs);
        cudaFree(m->sc);
        delete m;
        *out = nullptr;
    }
    return r;
}

HC_EXPORT int hc_q4_matrix_free(hc_q4_matrix* m) {
    if (!m) return HC_OK;
    cudaFree(m->qs);
    cudaFree(m->sc);
    delete m;
    return HC_OK;
}

HC_EXPORT int hc_q4_matmul_dev(const hc_q4_matrix* w, const float* x, size_t mtok, float* y, void* stream) {
    HC_CHECK(w && x && y, HC_ERR_INVALID, "hc_q4_matmul_dev: NULL argument");
    cudaStream_t s = (cudaStream_t)stream;
    if (hc::gemm_tc_eligible(*w, mtok)) {
        static hc::GemmWorkspace* ws = hc::gemm_workspace_new();
        static std::atomic<unsigned> calls{0};
        HC_TRY(hc::gemm_tc(ws, *w, x, w->k, mtok, y, w->n, hc::EPI_STORE, nullptr, 0, s));
        // The abort flag is read (with a device sync) only every 64th call so
        // timing loops stay asynchronous, and never while the stream is being
        // captured into a graph (a capturing stream cannot be synchronized).
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        HC_CUDA(cudaStreamIsCapturing(s, &cs));
        if (cs == cudaStreamCaptureStatusNone && (++calls & 63u) == 0) return hc::gemm_check(ws);
        return HC_OK;
    }
    DevWeight dw;
    dw.dtype = HC_DTYPE_Q4_0;
    dw.n = w->n;
    dw.k = w->k;
    dw.q4 = *w;
    dw.present = true;
    return hc::launch_matmul(dw, x, w->k, mtok, y, w->n, hc::EPI_STORE, nullptr, 0, s);
}

// ============================================================ synthetic inputs

HC_EXPORT int hc_synth_normal_host(uint64_t seed, uint64_t stream, uint64_t offset, uint64_t n, float std,
                                   float* out) {
    HC_CHECK(out || n == 0, HC_ERR_INVALID, "hc_synth_normal_host: NULL out");
    uint64_t key = hc::synth_key(seed, stream);
    float scale = std / 65536.0f;
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; i++) out[i] = hc::synth_normal(key, offset + (uint64_t)i, scale);
    return HC_OK;
}

HC_EXPORT int hc_synth_normal_dev(uint64_t seed, uint64_t stream, uint64_t offset, uint64_t n, float std, float* out,
                                  void* cuda_stream) {
    HC_CHECK(out || n == 0, HC_ERR_INVALID, "hc_synth_normal_dev: NULL out");
    return hc::launch_synth_normal(seed, stream, offset, n, std, out, (cudaStream_t)cuda_stream);
}
