// One-shot peer all-reduce for decode-sized tensor-parallel messages, fused
// with the residual add and the following RMSNorm.
//
// After a row-parallel projection (o_proj, down_proj) every rank holds a
// partial [rows][H] product.  NCCL's all-reduce costs tens of microseconds
// per call at these sizes (512 KiB for 32 x 4096 f32) and is followed by a
// separate add and a separate RMSNorm.  Here each rank writes its partial
// into a buffer that every peer has mapped (CUDA IPC over NVLink; plain peer
// loads and stores, no multicast), and one CTA per row:
//   1. tells every peer its partial of this row is complete (a release store
//      of the row's epoch into the peer's "ready" flags, system scope),
//   2. waits until every peer said the same (acquire loads, bounded),
//   3. sums the ranks' partials IN RANK ORDER (the same float sum on every
//      rank, so the replicated residual stream stays identical), adds the
//      residual, writes it back, and computes the RMSNorm of the new row
//      (kernels.rs:592-625 arithmetic) plus its fp16 copy in GEMM K order,
// When the projection wrote split-K slabs (local memory), each CTA first adds
// its row's slabs in slab order into this rank's peer-visible partial row and
// fences before the handshake.
// Each rank has two partial buffers, one for o_proj and one for down_proj,
// which alternate.  A peer that says its partial for one of them is complete
// has finished reading this rank's other buffer (its previous all-reduce
// kernel completed before its projection ran), so a rank never overwrites a
// partial a peer still reads, without a second handshake.
// The epochs live in device memory, one counter per row slot, so the kernel
// can be replayed from a CUDA graph.  Every wait is bounded; on expiry the
// CTA sets the error flag the host checks after the step and skips the rest.
#include "hc_internal.h"
#include "hc_common.cuh"
#include "hc_comm.h"
#include "hc_gemm.h"

#include <algorithm>
#include <cstring>
#include <vector>

namespace hc {

namespace {

constexpr int AR_MAX_RANKS = 8;
constexpr long long AR_WAIT_CYCLES = 2000000000LL;  // ~1 s at 1.9 GHz

constexpr int AR_MAX_SLABS = 8;  // split-K slabs of the local product (the model's kPartSplits)

struct ArParams {
    const float* partial[AR_MAX_RANKS];  // rank-ordered partial buffers ([rows][H] each)
    float* partial_mine;                 // this rank's, written here when slabs are given
    const float* slabs;                  // this rank's split-K slabs (slab i at slabs + i * slab), or null
    int splits;
    size_t slab;
    uint32_t* ready_peer[AR_MAX_RANKS];  // rank p's ready flags ([row][AR_MAX_RANKS])
    uint32_t* ready_mine;
    uint32_t* epochs;  // [row] this rank's completed epochs
    int rank, size, H;
    float* hidden;
    size_t ldh;
    const float* w;  // RMSNorm weight (null: residual update only)
    float eps;
    float* xn;
    size_t ldxn;
    __half* xn16;
    int* err;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Signals epoch e to every peer's flag slot [row][rank] and waits until every
// peer's signal for e sits in this rank's slots [row][p].  Thread 0 only.
__device__ bool handshake(uint32_t* const* peer_flags, const uint32_t* mine, int row, int rank, int size, uint32_t e) {
    __threadfence_system();
    for (int p = 0; p < size; p++)
        if (p != rank) st_release_sys(peer_flags[p] + (size_t)row * AR_MAX_RANKS + rank, e);
    const long long t0 = clock64();
    for (int p = 0; p < size; p++) {
        if (p == rank) continue;
        while ((int)(ld_acquire_sys(mine + (size_t)row * AR_MAX_RANKS + p) - e) < 0)
            if (clock64() - t0 > AR_WAIT_CYCLES) return false;
    }
    return true;
}

template <int VPT>
__global__ void __launch_bounds__(1024) k_ar_residual_norm(ArParams P) {
    // the next projection (a programmatic dependent) may start streaming its
    // weights while this kernel waits for the peers; it reads nothing this
    // kernel writes before its own grid-dependency wait
    pdl_trigger();
    __shared__ float red[32];
    __shared__ int ok_s;
    const int row = blockIdx.x;
    const int n4 = P.H / 4;
    const uint32_t e = P.epochs[row] + 1;  // read by thread 0 alone below, after every thread read it here
    // This rank's partial row: the sum of its split-K slabs (slab order),
    // published in its peer-visible buffer before the handshake.
    float4 mine[VPT];
    if (P.slabs) {
        float4* prow = reinterpret_cast<float4*>(P.partial_mine + (size_t)row * P.H);
        const float4* srow = reinterpret_cast<const float4*>(P.slabs + (size_t)row * P.H);
#pragma unroll
        for (int j = 0; j < VPT; j++) {
            const int i = threadIdx.x + j * blockDim.x;
            if (i < n4) {
                float4 q[AR_MAX_SLABS];
#pragma unroll
                for (int sp = 0; sp < AR_MAX_SLABS; sp++)
                    if (sp < P.splits) q[sp] = srow[(size_t)sp * (P.slab / 4) + i];
                float4 acc = q[0];
#pragma unroll
                for (int sp = 1; sp < AR_MAX_SLABS; sp++) {
                    if (sp < P.splits) {
                        acc.x = acc.x + q[sp].x; acc.y = acc.y + q[sp].y; acc.z = acc.z + q[sp].z; acc.w = acc.w + q[sp].w;
                    }
                }
                prow[i] = acc;
                mine[j] = acc;
            }
        }
    }
    // every thread's stores happen before thread 0's system-scope fence and
    // release stores in handshake() (ordered by this barrier)
    __syncthreads();
    if (threadIdx.x == 0) ok_s = handshake(P.ready_peer, P.ready_mine, row, P.rank, P.size, e) ? 1 : 0;
    __syncthreads();
    const bool ok = ok_s != 0;
    float4 v[VPT];
    float ss = 0.0f;
    if (ok) {
        float4* hrow = reinterpret_cast<float4*>(P.hidden + (size_t)row * P.ldh);
#pragma unroll
        for (int j = 0; j < VPT; j++) {
            const int i = threadIdx.x + j * blockDim.x;
            if (i < n4) {
                // every peer's partial (loads over NVLink) and the residual
                // are requested before the first add: one round trip instead
                // of one per rank; the sum keeps rank order
                float4 q[AR_MAX_RANKS];
#pragma unroll
                for (int p = 0; p < AR_MAX_RANKS; p++)
                    if (p < P.size && !(P.slabs && p == P.rank))
                        q[p] = __ldcg(reinterpret_cast<const float4*>(P.partial[p] + (size_t)row * P.H) + i);
                if (P.slabs) {
#pragma unroll
                    for (int p = 0; p < AR_MAX_RANKS; p++)
                        if (p == P.rank) q[p] = mine[j];
                }
                float4 r = hrow[i];
                float4 acc = q[0];
#pragma unroll
                for (int p = 1; p < AR_MAX_RANKS; p++) {
                    if (p < P.size) {
                        acc.x += q[p].x; acc.y += q[p].y; acc.z += q[p].z; acc.w += q[p].w;
                    }
                }
                r.x = r.x + acc.x; r.y = r.y + acc.y; r.z = r.z + acc.z; r.w = r.w + acc.w;
                hrow[i] = r;
                v[j] = r;
                ss = fmaf(r.x, r.x, ss);
                ss = fmaf(r.y, r.y, ss);
                ss = fmaf(r.z, r.z, ss);
                ss = fmaf(r.w, r.w, ss);
            } else {
                v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
    }
    if (P.w) {  // uniform over the grid
        const float4* wr = reinterpret_cast<const float4*>(P.w);
        float4 wv[VPT];  // the norm weights travel while the block reduces
#pragma unroll
        for (int j = 0; j < VPT; j++) {
            const int i = threadIdx.x + j * blockDim.x;
            wv[j] = i < n4 ? wr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        ss = block_sum(ss, red);
        const float ms = __fdiv_rn(ss, (float)P.H);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, P.eps)));
        if (ok) {
            float4* orow = reinterpret_cast<float4*>(P.xn + (size_t)row * P.ldxn);
            __half* r16 = P.xn16 ? P.xn16 + (size_t)row * 2 * P.H : nullptr;
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
                    if (r16) {
                        store_x16(r16, P.H, 4 * i, o.x);
                        store_x16(r16, P.H, 4 * i + 1, o.y);
                        store_x16(r16, P.H, 4 * i + 2, o.z);
                        store_x16(r16, P.H, 4 * i + 3, o.w);
                    }
                }
            }
        }
    }
    if (threadIdx.x == 0) {
        if (ok) P.epochs[row] = e;
        else if (P.err) atomicExch(P.err, 1);
    }
}

}  // namespace

// Layout of the block every rank allocates and maps from its peers.
struct PeerAr {
    size_t rows_cap = 0, H = 0;
    uint8_t* base = nullptr;                  // this rank's block
    uint8_t* peer[AR_MAX_RANKS] = {};         // every rank's block (peer[rank] == base)
    size_t partial_off[2] = {0, 0}, ready_off = 0, epoch_off = 0, bytes = 0;
};

static void layout(PeerAr& a) {
    const size_t part = (a.rows_cap * a.H * sizeof(float) + 255) & ~(size_t)255;
    a.partial_off[0] = 0;
    a.partial_off[1] = part;
    a.ready_off = 2 * part;
    a.epoch_off = a.ready_off + a.rows_cap * AR_MAX_RANKS * sizeof(uint32_t);
    a.bytes = a.epoch_off + a.rows_cap * sizeof(uint32_t);
}

void peer_ar_free(PeerAr* a, int rank, int size) {
    if (!a) return;
    for (int p = 0; p < size && p < AR_MAX_RANKS; p++)
        if (p != rank && a->peer[p]) cudaIpcCloseMemHandle(a->peer[p]);
    if (a->base) cudaFree(a->base);
    delete a;
    (void)cudaGetLastError();
}

// Allocates this rank's block, shares its IPC handle with the peers through
// the communicator and maps theirs.  Returns HC_OK with *out == nullptr when
// peer mappings are not available (the caller then keeps NCCL).
int peer_ar_init(Comm* c, int rank, int size, size_t rows_cap, size_t H, PeerAr** out) {
    *out = nullptr;
    if (size < 2 || size > AR_MAX_RANKS || H % 4 != 0 || H > 4 * 1024 * 2) return HC_OK;  // rows held in registers
    PeerAr* a = new PeerAr();
    a->rows_cap = rows_cap;
    a->H = H;
    layout(*a);
    if (cudaMalloc((void**)&a->base, a->bytes) != cudaSuccess) {
        delete a;
        (void)cudaGetLastError();
        return HC_OK;
    }
    HC_CUDA(cudaMemset(a->base, 0, a->bytes));
    HC_CUDA(cudaDeviceSynchronize());
    cudaIpcMemHandle_t mine;
    std::vector<uint8_t> all((size_t)size * sizeof(cudaIpcMemHandle_t));
    int ok = cudaIpcGetMemHandle(&mine, a->base) == cudaSuccess ? 1 : 0;
    if (!ok) std::memset(&mine, 0, sizeof(mine));
    // every rank takes part in the exchange (also when its own handle failed)
    HC_TRY(comm_allgather_host(c, &mine, all.data(), sizeof(mine)));
    std::vector<int32_t> oks(size);
    HC_TRY(comm_allgather_host(c, &ok, oks.data(), sizeof(int32_t)));
    bool all_ok = true;
    for (int p = 0; p < size; p++) all_ok = all_ok && oks[p];
    int mapped = 1;
    for (int p = 0; p < size && all_ok; p++) {
        if (p == rank) {
            a->peer[p] = a->base;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, all.data() + (size_t)p * sizeof(h), sizeof(h));
        void* ptr = nullptr;
        if (cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            (void)cudaGetLastError();
            mapped = 0;
            break;
        }
        a->peer[p] = (uint8_t*)ptr;
    }
    // all ranks must agree to use the peer path
    std::vector<int32_t> maps(size);
    int32_t mine_ok = (all_ok && mapped) ? 1 : 0;
    HC_TRY(comm_allgather_host(c, &mine_ok, maps.data(), sizeof(int32_t)));
    bool use = true;
    for (int p = 0; p < size; p++) use = use && maps[p];
    if (!use) {
        peer_ar_free(a, rank, size);
        return HC_OK;
    }
    *out = a;
    return HC_OK;
}

float* peer_ar_partial(PeerAr* a, int slot) {
    return a ? reinterpret_cast<float*>(a->base + a->partial_off[slot & 1]) : nullptr;
}

bool peer_ar_fits(const PeerAr* a, size_t rows, size_t H) { return a && rows >= 1 && rows <= a->rows_cap && H == a->H; }

int peer_ar_residual_norm(PeerAr* a, int slot, int rank, int size, size_t rows, const float* slabs, int splits,
                          float* hidden, size_t ldh, const float* w, float eps, float* xn, size_t ldxn, __half* xn16,
                          int* err, cudaStream_t s) {
    HC_CHECK(peer_ar_fits(a, rows, a ? a->H : 0), HC_ERR_INVALID, "peer all-reduce: %zu rows do not fit", rows);
    HC_CHECK(!slabs || (splits >= 1 && splits <= AR_MAX_SLABS && ((uintptr_t)slabs & 15) == 0), HC_ERR_INVALID,
             "peer all-reduce: %d split-K slabs", splits);
    HC_CHECK((ldh % 4) == 0 && (ldxn % 4) == 0 && ((uintptr_t)hidden & 15) == 0 && ((uintptr_t)xn & 15) == 0 &&
                 (!w || ((uintptr_t)w & 15) == 0),
             HC_ERR_INVALID, "peer all-reduce: rows must be 16-byte aligned");
    ArParams P{};
    for (int p = 0; p < size; p++) {
        P.partial[p] = reinterpret_cast<const float*>(a->peer[p] + a->partial_off[slot & 1]);
        P.ready_peer[p] = reinterpret_cast<uint32_t*>(a->peer[p] + a->ready_off);
    }
    P.ready_mine = reinterpret_cast<uint32_t*>(a->base + a->ready_off);
    P.partial_mine = reinterpret_cast<float*>(a->base + a->partial_off[slot & 1]);
    P.slabs = slabs;
    P.splits = slabs ? splits : 0;
    P.slab = rows * a->H;
    P.epochs = reinterpret_cast<uint32_t*>(a->base + a->epoch_off);
    P.rank = rank;
    P.size = size;
    P.H = (int)a->H;
    P.hidden = hidden;
    P.ldh = ldh;
    P.w = w;
    P.eps = eps;
    P.xn = xn;
    P.ldxn = ldxn;
    P.xn16 = xn16;
    P.err = err;
    const size_t n4 = a->H / 4;
    const unsigned threads = (unsigned)std::min<size_t>(1024, ((n4 + 31) / 32) * 32);
    const size_t vpt = (n4 + threads - 1) / threads;
    if (vpt <= 1) k_ar_residual_norm<1><<<(unsigned)rows, threads, 0, s>>>(P);
    else k_ar_residual_norm<2><<<(unsigned)rows, threads, 0, s>>>(P);
    HC_LAUNCH_CHECK();
    return HC_OK;
}

}  // namespace hc
