// Token sampling on the device: sample_token and XorShift64 of run.rs:203-278,
// one CTA per row of logits, so that a serving loop reads back B token ids
// instead of B x vocab logits.
//
// Per row (temperature T, top_p, top_k, the row's XorShift64 state):
//   p_i = T > 0 ? exp(l_i * (1 / T)) : l_i                     (run.rs:207-210)
//   top_k in (0, V): keep p_i >= the top_k-th largest p        (run.rs:212-217)
//   top_p < 1: with sum = sum of p, keep p_i >= the value at which the
//     descending cumulative sum of p / sum first exceeds top_p; when it never
//     does, keep nothing                                        (run.rs:219-231)
//   sum of the kept p <= 0: the last maximal logit (max_by)     (run.rs:233-238)
//   else r = next_f32(); the first i whose cumulative kept p / sum exceeds r,
//     or the last maximal kept p when rounding leaves none      (run.rs:240-250)
// The thresholds are exact values of the row, found by a 3-pass radix search
// over order-preserving keys (11 + 11 + 10 bits) with per-bucket counts and
// f64 sums; every sum is accumulated in f64, where the reference adds f32
// terms one by one (up to ~V * 2^-24 relative apart), so a draw that falls
// within that rounding of a bucket edge may pick the neighbouring token.
// exp is CUDA's expf (within 2 ulp of libm); NaN values are never kept.
#include "hc_internal.h"
#include "hc_common.cuh"

#include <cfloat>

namespace hc {

namespace {

constexpr int SMP_THREADS = 1024;
constexpr int HB = 2048;  // buckets per radix pass

// Larger float -> larger key (NaN with a clear sign bit above +inf).
__device__ __forceinline__ uint32_t fkey(float f) {
    const uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float keyf(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

struct SampleRow {
    const float* l;
    int V;
    bool texp;
    float inv;
    __device__ __forceinline__ float prob(int i) const { return texp ? expf(__fmul_rn(l[i], inv)) : l[i]; }
};

__device__ __forceinline__ double block_sum_f64(double v, double* red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    double t = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0;
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    return t;
}

// Warp 0 walks the buckets from the top: the first bucket at which the
// running total (counts when by_sum is false, f64 sums otherwise) reaches
// `need` (counts: >= need; sums: > need).  Returns the bucket and the total
// of the buckets above it, or -1 when the total never gets there.
__device__ void find_from_top(const uint32_t* cnt, const double* sum, int nb, bool by_sum, double need, int* sel_out,
                              double* above_out) {
    if (threadIdx.x >= 32) return;
    const int lane = threadIdx.x;
    const int per = nb / 32;  // buckets per lane, lane 0 taking the top ones
    double mine = 0.0;
    for (int k = 0; k < per; k++) {
        const int b = nb - 1 - (lane * per + k);
        mine += by_sum ? sum[b] : (double)cnt[b];
    }
    double incl = mine;  // inclusive scan over lanes (top buckets first)
    for (int o = 1; o < 32; o <<= 1) {
        const double t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    const double excl = incl - mine;
    const double total = __shfl_sync(0xffffffffu, incl, 31);
    const bool hit = by_sum ? (incl > need) : (incl >= need);
    const unsigned ball = __ballot_sync(0xffffffffu, hit);
    if (!ball) {
        if (lane == 0) {
            *sel_out = -1;
            *above_out = total;
        }
        return;
    }
    const int first = __ffs(ball) - 1;
    if (lane == first) {
        double run = excl;
        int sel = nb - 1 - lane * per;
        for (int k = 0; k < per; k++) {
            const int b = nb - 1 - (lane * per + k);
            const double add = by_sum ? sum[b] : (double)cnt[b];
            if (by_sum ? (run + add > need) : (run + add >= need)) {
                sel = b;
                break;
            }
            run += add;
        }
        *sel_out = sel;
        *above_out = run;
    }
}

// The key of the row's value at which the descending running count reaches
// `need` (by_sum false) or the descending running sum of the kept values
// exceeds `need` (by_sum true); kept = value >= floor_v.  Returns false when
// the sum never exceeds need.
__device__ bool radix_select(const SampleRow& R, float floor_v, bool by_sum, double need, uint32_t* key_out,
                             uint32_t* hcnt, double* hsum, int* s_sel, double* s_above) {
    uint32_t prefix = 0, mask = 0;
    const int shifts[3] = {21, 10, 0};
    const int widths[3] = {11, 11, 10};
    for (int pass = 0; pass < 3; pass++) {
        const int nb = 1 << widths[pass];
        for (int b = threadIdx.x; b < nb; b += blockDim.x) {
            hcnt[b] = 0;
            hsum[b] = 0.0;
        }
        __syncthreads();
        for (int i = threadIdx.x; i < R.V; i += blockDim.x) {
            const float p = R.prob(i);
            if (!(p >= floor_v)) continue;
            const uint32_t k = fkey(p);
            if ((k & mask) != prefix) continue;
            const int b = (int)((k >> shifts[pass]) & (uint32_t)(nb - 1));
            if (by_sum) atomicAdd(&hsum[b], (double)p);
            else atomicAdd(&hcnt[b], 1u);
        }
        __syncthreads();
        find_from_top(hcnt, hsum, nb, by_sum, need, s_sel, s_above);
        __syncthreads();
        const int sel = *s_sel;
        if (sel < 0) return false;
        need -= *s_above;
        prefix |= (uint32_t)sel << shifts[pass];
        mask |= (uint32_t)(nb - 1) << shifts[pass];
        __syncthreads();
    }
    *key_out = prefix;
    return true;
}

// Last index of the row maximum (max_by: the later of equal values wins).
__device__ int last_max(const SampleRow& R, bool use_prob, float floor_v, float* red_v, int* red_i) {
    float best = -INFINITY;
    int bi = -1;
    for (int i = threadIdx.x; i < R.V; i += blockDim.x) {
        float v = use_prob ? R.prob(i) : R.l[i];
        if (use_prob && !(v >= floor_v)) v = 0.0f;
        if (bi < 0 || v >= best) {
            best = v;
            bi = i;
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oi >= 0 && (bi < 0 || ov > best || (ov == best && oi > bi))) {
            best = ov;
            bi = oi;
        }
    }
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) {
        red_v[w] = best;
        red_i[w] = bi;
    }
    __syncthreads();
    if (w == 0) {
        const int nw = blockDim.x >> 5;
        best = lane < nw ? red_v[lane] : -INFINITY;
        bi = lane < nw ? red_i[lane] : -1;
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi >= 0 && (bi < 0 || ov > best || (ov == best && oi > bi))) {
                best = ov;
                bi = oi;
            }
        }
        if (lane == 0) red_i[0] = bi;
    }
    __syncthreads();
    const int r = red_i[0];
    __syncthreads();
    return r < 0 ? 0 : r;
}

__global__ void __launch_bounds__(SMP_THREADS) k_sample(const float* __restrict__ logits, size_t ld, int V,
                                                        const float* __restrict__ temp, const float* __restrict__ top_p,
                                                        const int* __restrict__ top_k, uint64_t* __restrict__ rng,
                                                        uint32_t* __restrict__ out) {
    __shared__ uint32_t hcnt[HB];
    __shared__ double hsum[HB];
    __shared__ double red[32];
    __shared__ float red_v[32];
    __shared__ int red_i[32];
    __shared__ int s_sel;
    __shared__ double s_above;
    __shared__ double s_chunk[SMP_THREADS];
    __shared__ float s_r;
    const int row = blockIdx.x;
    const float T = temp[row], tp = top_p[row];
    const int tk = top_k[row];
    SampleRow R;
    R.l = logits + (size_t)row * ld;
    R.V = V;
    R.texp = T > 0.0f;
    R.inv = R.texp ? __fdiv_rn(1.0f, T) : 1.0f;

    // top-k: keep p >= the top_k-th largest value
    float floor_v = -INFINITY;
    if (tk > 0 && tk < V) {
        uint32_t key;
        if (radix_select(R, -INFINITY, false, (double)tk, &key, hcnt, hsum, &s_sel, &s_above)) floor_v = keyf(key);
    }
    // top-p on the kept values
    bool none = false;
    if (tp < 1.0f) {
        double s = 0.0;
        for (int i = threadIdx.x; i < V; i += blockDim.x) {
            const float p = R.prob(i);
            if (p >= floor_v) s += (double)p;
        }
        const float sum = (float)block_sum_f64(s, red);
        if (sum > 0.0f) {
            uint32_t key;
            // the running sum of p / sum exceeds top_p where the running sum of p exceeds top_p * sum
            if (radix_select(R, floor_v, true, (double)tp * (double)sum, &key, hcnt, hsum, &s_sel, &s_above))
                floor_v = fmaxf(floor_v, keyf(key));
            else
                none = true;  // threshold f32::MAX: every p is cleared
        }
    }
    // the sum of what is kept
    double s = 0.0;
    if (!none)
        for (int i = threadIdx.x; i < V; i += blockDim.x) {
            const float p = R.prob(i);
            if (p >= floor_v) s += (double)p;
        }
    const float sum = none ? 0.0f : (float)block_sum_f64(s, red);
    if (!(sum > 0.0f)) {
        const int i = last_max(R, false, -INFINITY, red_v, red_i);
        if (threadIdx.x == 0) out[row] = (uint32_t)i;
        return;
    }
    if (threadIdx.x == 0) {
        uint64_t x = rng[row];
        x ^= x << 13;
        x ^= x >> 7;
        x ^= x << 17;
        rng[row] = x;
        s_r = (float)(x >> 40) / 16777216.0f;
    }
    __syncthreads();
    // first i (ascending) whose running kept p exceeds r * sum: contiguous
    // chunks per thread, an exclusive scan of the chunk sums, then the thread
    // whose chunk holds the crossing walks it
    const double target = (double)s_r * (double)sum;
    const int per = (V + (int)blockDim.x - 1) / (int)blockDim.x;
    const int i0 = (int)threadIdx.x * per, i1 = min(V, i0 + per);
    double cs = 0.0;
    for (int i = i0; i < i1; i++) {
        const float p = R.prob(i);
        if (p >= floor_v) cs += (double)p;
    }
    s_chunk[threadIdx.x] = cs;
    __syncthreads();
    if (threadIdx.x < 32) {  // warp 0: exclusive scan over the chunks (32 per lane)
        const int lane = threadIdx.x, nper = (int)blockDim.x / 32;
        double mine = 0.0;
        for (int k = 0; k < nper; k++) mine += s_chunk[lane * nper + k];
        double incl = mine;
        for (int o = 1; o < 32; o <<= 1) {
            const double t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        double run = incl - mine;
        for (int k = 0; k < nper; k++) {
            const double c = s_chunk[lane * nper + k];
            s_chunk[lane * nper + k] = run;
            run += c;
        }
    }
    __shared__ unsigned int s_pick;
    if (threadIdx.x == 0) s_pick = 0xFFFFFFFFu;
    __syncthreads();
    double run = s_chunk[threadIdx.x];
    if (run <= target) {  // only the chunk holding the crossing finds one
        for (int i = i0; i < i1; i++) {
            const float p = R.prob(i);
            if (p >= floor_v) run += (double)p;
            if (run > target) {
                atomicMin(&s_pick, (unsigned int)i);
                break;
            }
        }
    }
    __syncthreads();
    const int pick = s_pick == 0xFFFFFFFFu ? -1 : (int)s_pick;
    if (pick >= 0) {
        if (threadIdx.x == 0) out[row] = (uint32_t)pick;
        return;
    }
    const int i = last_max(R, true, floor_v, red_v, red_i);
    if (threadIdx.x == 0) out[row] = (uint32_t)i;
}

}  // namespace

int launch_sample(const float* logits, size_t ld, int B, int V, const float* temp, const float* top_p,
                  const int* top_k, uint64_t* rng, uint32_t* out, cudaStream_t s) {
    if (B <= 0) return HC_OK;
    k_sample<<<(unsigned)B, SMP_THREADS, 0, s>>>(logits, ld, V, temp, top_p, top_k, rng, out);
    HC_LAUNCH_CHECK();
    return HC_OK;
}

}  // namespace hc

// run.rs:203-278 for B rows of device logits (row stride ld floats): per-row
// temperature, top_p, top_k (device arrays of B) and XorShift64 states
// (device array of B, advanced by one draw for every row that draws).
HC_EXPORT int hc_sample_dev(const float* logits_dev, size_t ld, int B, int V, const float* temperature_dev,
                            const float* top_p_dev, const int* top_k_dev, uint64_t* rng_state_dev, uint32_t* out_dev,
                            void* stream) {
    HC_CHECK(B >= 0 && V > 0 && ld >= (size_t)V, HC_ERR_INVALID, "hc_sample_dev: bad shape (B %d, V %d, ld %zu)", B,
             V, ld);
    HC_CHECK(B == 0 || (logits_dev && temperature_dev && top_p_dev && top_k_dev && rng_state_dev && out_dev),
             HC_ERR_INVALID, "hc_sample_dev: NULL argument");
    return hc::launch_sample(logits_dev, ld, B, V, temperature_dev, top_p_dev, top_k_dev, rng_state_dev, out_dev,
                             (cudaStream_t)stream);
}
