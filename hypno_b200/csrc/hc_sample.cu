// Token sampling on the device: sample_token and XorShift64 of run.rs:203-278,
// one CTA per row of logits, so that a serving loop reads back B token ids
// instead of B x vocab logits.
//
// Per row (temperature T, top_p, top_k, the row's XorShift64 state):
//   p_i = T > 0 ? exp(l_i * (1 / T)) : l_i                     (run.rs:207-210)
//   top_k in (0, V): p_i = 0 where p_i < the top_k-th largest p (run.rs:212-217)
//   top_p < 1: sum = sum of p; walking p in descending order, the first value
//     at which the running sum of p / sum exceeds top_p is the threshold
//     (f32::MAX when it never does); p_i = 0 below it          (run.rs:219-231)
//   sum of p <= 0: the last maximal logit (max_by)              (run.rs:233-238)
//   else r = next_f32(); the first i at which the running sum of p_i / sum
//     exceeds r, or the last maximal p when rounding leaves none (run.rs:240-250)
// Every sum is the reference's: f32 additions one term at a time in the
// reference's order.  One thread performs each such chain while the other
// warps produce the next chunk of terms (exp, masking, the IEEE division) in
// shared memory, so a chain costs about one f32 add latency per term.  The
// top-k threshold is an exact value of the row, found by a 3-pass radix search
// over order-preserving keys (11 + 11 + 10 bits); the top-p walk visits the
// positive values in descending order in sorted chunks of up to SORT_CAP keys
// (each chunk bounded below by a radix-selected key, its ties added last).
// exp is CUDA's expf (within 2 ulp of the C library's), so a draw can differ
// from the reference's only when it falls within a few ulp of a boundary.
// NaN values are never kept (the reference would panic comparing them).
#include "hc_internal.h"
#include "hc_common.cuh"

#include <cfloat>

namespace hc {

namespace {

constexpr int SMP_THREADS = 1024;
constexpr int HB = 2048;        // buckets per radix pass
constexpr int CH = 2048;        // terms per chain chunk
constexpr int SORT_CAP = 2048;  // keys per sorted top-p chunk (<= HB: the sort reuses the bucket array)

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
    // p_i after masking everything below floor_v to 0 (NaN is dropped too)
    __device__ __forceinline__ float kept(int i, float floor_v) const {
        const float p = prob(i);
        return p >= floor_v ? p : 0.0f;
    }
};

struct __align__(16) Shared {
    uint32_t hcnt[HB];   // radix buckets; the top-p sort buffer
    float cbuf[2][CH];   // chain chunks (double-buffered)
    float red_v[32];
    int red_i[32];
    uint32_t red_u[32];
    int sel;
    uint32_t above;
    int stop;
    int n_gather;
    float r;
    float sumv;
};

__device__ __forceinline__ uint32_t block_sum_u32(uint32_t v, Shared& S) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) S.red_u[w] = v;
    __syncthreads();
    uint32_t t = lane < (int)(blockDim.x >> 5) ? S.red_u[lane] : 0u;
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    return t;
}

// The reference's sequential f32 chain over i = 0..V-1 of the terms
// a_i = kept p_i (divided by `div` when div != 0):
//   pick == false: returns the sum a_0 + a_1 + ... (added left to right);
//   pick == true: returns the first i at which r < the running sum, or -1.
// Thread 0 adds chunk c while warps 1.. fill chunk c + 1.
__device__ float chain_index(const SampleRow& R, float floor_v, float div, bool pick, float r, Shared& S,
                             int* pick_out) {
    const int V = R.V, nch = (V + CH - 1) / CH;
    for (int j = threadIdx.x; j < CH && j < V; j += blockDim.x) {
        const float p = R.kept(j, floor_v);
        S.cbuf[0][j] = div != 0.0f ? __fdiv_rn(p, div) : p;
    }
    if (threadIdx.x == 0) S.stop = -1;
    __syncthreads();
    float acc = 0.0f;
    for (int c = 0; c < nch; c++) {
        const int base = c * CH, len = min(CH, V - base);
        if (threadIdx.x == 0) {
            const float* b = S.cbuf[c & 1];
            if (pick) {
                for (int j = 0; j < len; j++) {
                    acc = __fadd_rn(acc, b[j]);
                    if (r < acc) {
                        S.stop = base + j;
                        break;
                    }
                }
            } else {
                int j = 0;
                for (; j + 8 <= len; j += 8) {
                    const float4 u = *reinterpret_cast<const float4*>(b + j);
                    const float4 v = *reinterpret_cast<const float4*>(b + j + 4);
                    acc = __fadd_rn(acc, u.x);
                    acc = __fadd_rn(acc, u.y);
                    acc = __fadd_rn(acc, u.z);
                    acc = __fadd_rn(acc, u.w);
                    acc = __fadd_rn(acc, v.x);
                    acc = __fadd_rn(acc, v.y);
                    acc = __fadd_rn(acc, v.z);
                    acc = __fadd_rn(acc, v.w);
                }
                for (; j < len; j++) acc = __fadd_rn(acc, b[j]);
            }
        } else if (threadIdx.x >= 32 && c + 1 < nch) {
            const int nb = (c + 1) * CH, nl = min(CH, V - nb);
            float* d = S.cbuf[(c + 1) & 1];
            for (int j = (int)threadIdx.x - 32; j < nl; j += (int)blockDim.x - 32) {
                const float p = R.kept(nb + j, floor_v);
                d[j] = div != 0.0f ? __fdiv_rn(p, div) : p;
            }
        }
        __syncthreads();
        if (S.stop >= 0) break;
    }
    if (pick_out) *pick_out = S.stop;
    if (threadIdx.x == 0) S.sumv = acc;  // thread 0's chain
    __syncthreads();
    const float out = S.sumv;
    __syncthreads();
    return out;
}

// Warp 0 walks the buckets from the top: the first bucket at which the
// running count reaches `need`.  Returns the bucket and the count of the
// buckets above it, or -1 when the count never gets there.
__device__ void find_from_top(const uint32_t* cnt, int nb, uint32_t need, int* sel_out, uint32_t* above_out) {
    if (threadIdx.x >= 32) return;
    const int lane = threadIdx.x;
    const int per = nb / 32;  // buckets per lane, lane 0 taking the top ones
    uint32_t mine = 0;
    for (int k = 0; k < per; k++) mine += cnt[nb - 1 - (lane * per + k)];
    uint32_t incl = mine;  // inclusive scan over lanes (top buckets first)
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    const uint32_t excl = incl - mine;
    const unsigned ball = __ballot_sync(0xffffffffu, incl >= need);
    if (!ball) {
        if (lane == 0) *sel_out = -1;
        return;
    }
    const int first = __ffs(ball) - 1;
    if (lane == first) {
        uint32_t run = excl;
        int sel = nb - 1 - lane * per;
        for (int k = 0; k < per; k++) {
            const int b = nb - 1 - (lane * per + k);
            if (run + cnt[b] >= need) {
                sel = b;
                break;
            }
            run += cnt[b];
        }
        *sel_out = sel;
        *above_out = run;
    }
}

// Candidates: p >= floor_v whose key lies in [lo_key, hi_key].  Returns the
// key at which the descending running count of candidates reaches `need`
// (the need-th largest), or false when there are fewer candidates.
__device__ bool radix_select(const SampleRow& R, float floor_v, uint32_t lo_key, uint32_t hi_key, uint32_t need,
                             uint32_t* key_out, Shared& S) {
    uint32_t prefix = 0, mask = 0;
    const int shifts[3] = {21, 10, 0};
    const int widths[3] = {11, 11, 10};
    for (int pass = 0; pass < 3; pass++) {
        const int nb = 1 << widths[pass];
        for (int b = threadIdx.x; b < nb; b += blockDim.x) S.hcnt[b] = 0;
        __syncthreads();
        for (int i = threadIdx.x; i < R.V; i += blockDim.x) {
            const float p = R.prob(i);
            if (!(p >= floor_v)) continue;
            const uint32_t k = fkey(p);
            if (k < lo_key || k > hi_key || (k & mask) != prefix) continue;
            atomicAdd(&S.hcnt[(k >> shifts[pass]) & (uint32_t)(nb - 1)], 1u);
        }
        __syncthreads();
        find_from_top(S.hcnt, nb, need, &S.sel, &S.above);
        __syncthreads();
        const int sel = S.sel;
        if (sel < 0) return false;
        need -= S.above;
        prefix |= (uint32_t)sel << shifts[pass];
        mask |= (uint32_t)(nb - 1) << shifts[pass];
        __syncthreads();
    }
    *key_out = prefix;
    return true;
}

// Descending bitonic sort of S.hcnt[0..n) (n <= SORT_CAP), padded with 0 keys.
__device__ void sort_keys_desc(int n, Shared& S) {
    int m = 1;
    while (m < n) m <<= 1;
    for (int j = n + (int)threadIdx.x; j < m; j += blockDim.x) S.hcnt[j] = 0u;
    __syncthreads();
    for (int k = 2; k <= m; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < m; i += blockDim.x) {
                const int o = i ^ j;
                if (o > i) {
                    const uint32_t a = S.hcnt[i], b = S.hcnt[o];
                    const bool desc = (i & k) == 0;
                    if (desc ? (a < b) : (a > b)) {
                        S.hcnt[i] = b;
                        S.hcnt[o] = a;
                    }
                }
            }
            __syncthreads();
        }
    }
}

// run.rs:219-231: the top-p threshold over p >= floor_v (the top-k survivors),
// given their sequential sum `sum` > 0.  The running sum of p / sum only
// grows at positive terms, so the walk visits the positive values in
// descending order: chunks of the SORT_CAP largest keys still unvisited
// (radix-selected bound, gathered, sorted), then that bound's ties.  Returns
// false when the running sum never exceeds top_p.
__device__ bool top_p_threshold(const SampleRow& R, float floor_v, float sum, float top_p, Shared& S, float* thr_out) {
    const uint32_t lo = 0x80000001u;  // key of the smallest positive (denormal) value
    uint32_t hi = 0xFFFFFFFFu;
    float cum = 0.0f;  // thread 0's chain
    for (;;) {
        // keys of positive candidates in [lo, hi]
        uint32_t cut;
        bool all = !radix_select(R, floor_v, lo, hi, (uint32_t)SORT_CAP, &cut, S);
        // gather the keys above the cut (all of them when fewer than SORT_CAP remain)
        if (threadIdx.x == 0) S.n_gather = 0;
        __syncthreads();
        for (int i = threadIdx.x; i < R.V; i += blockDim.x) {
            const float p = R.prob(i);
            if (!(p >= floor_v)) continue;
            const uint32_t k = fkey(p);
            if (k < lo || k > hi || (!all && k <= cut)) continue;
            S.hcnt[atomicAdd(&S.n_gather, 1)] = k;
        }
        __syncthreads();
        const int n = S.n_gather;
        __syncthreads();
        uint32_t ties = 0;
        if (!all) {
            uint32_t t = 0;
            for (int i = threadIdx.x; i < R.V; i += blockDim.x) {
                const float p = R.prob(i);
                t += (p >= floor_v && fkey(p) == cut) ? 1u : 0u;
            }
            ties = block_sum_u32(t, S);
        }
        if (n > 0) {
            sort_keys_desc(n, S);
            for (int j = threadIdx.x; j < n; j += blockDim.x) S.cbuf[0][j] = __fdiv_rn(keyf(S.hcnt[j]), sum);
            __syncthreads();
            if (threadIdx.x == 0) {
                S.stop = -1;
                for (int j = 0; j < n; j++) {
                    cum = __fadd_rn(cum, S.cbuf[0][j]);
                    if (cum > top_p) {
                        S.stop = j;
                        S.r = keyf(S.hcnt[j]);
                        break;
                    }
                }
            }
            __syncthreads();
            const bool found = S.stop >= 0;
            const float thr = S.r;
            __syncthreads();
            if (found) {
                *thr_out = thr;
                return true;
            }
        }
        if (all) return false;
        if (threadIdx.x == 0) {
            const float v = keyf(cut), q = __fdiv_rn(v, sum);
            S.stop = -1;
            for (uint32_t t = 0; t < ties; t++) {
                cum = __fadd_rn(cum, q);
                if (cum > top_p) {
                    S.stop = 0;
                    S.r = v;
                    break;
                }
            }
        }
        __syncthreads();
        const bool found = S.stop >= 0;
        const float thr = S.r;
        __syncthreads();
        if (found) {
            *thr_out = thr;
            return true;
        }
        if (cut <= lo) return false;
        hi = cut - 1u;
    }
}

// Last index of the row maximum (max_by: the later of equal values wins);
// over the logits (use_prob false) or over the masked p.
__device__ int last_max(const SampleRow& R, bool use_prob, float floor_v, Shared& S) {
    float best = -INFINITY;
    int bi = -1;
    for (int i = threadIdx.x; i < R.V; i += blockDim.x) {
        const float v = use_prob ? R.kept(i, floor_v) : R.l[i];
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
        S.red_v[w] = best;
        S.red_i[w] = bi;
    }
    __syncthreads();
    if (w == 0) {
        const int nw = blockDim.x >> 5;
        best = lane < nw ? S.red_v[lane] : -INFINITY;
        bi = lane < nw ? S.red_i[lane] : -1;
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi >= 0 && (bi < 0 || ov > best || (ov == best && oi > bi))) {
                best = ov;
                bi = oi;
            }
        }
        if (lane == 0) S.red_i[0] = bi;
    }
    __syncthreads();
    const int r = S.red_i[0];
    __syncthreads();
    return r < 0 ? 0 : r;
}

__global__ void __launch_bounds__(SMP_THREADS) k_sample(const float* __restrict__ logits, size_t ld, int V,
                                                        const float* __restrict__ temp, const float* __restrict__ top_p,
                                                        const int* __restrict__ top_k, uint64_t* __restrict__ rng,
                                                        uint32_t* __restrict__ out) {
    __shared__ Shared S;
    const int row = blockIdx.x;
    const float T = temp[row], tp = top_p[row];
    const int tk = top_k[row];
    SampleRow R;
    R.l = logits + (size_t)row * ld;
    R.V = V;
    R.texp = T > 0.0f;
    R.inv = R.texp ? __fdiv_rn(1.0f, T) : 1.0f;

    // top-k: p below the top_k-th largest value become 0
    float floor_v = -INFINITY;
    if (tk > 0 && tk < V) {
        uint32_t key;
        if (radix_select(R, -INFINITY, 0u, 0xFFFFFFFFu, (uint32_t)tk, &key, S)) floor_v = keyf(key);
    }
    // top-p over what top-k kept
    bool none = false;
    if (tp < 1.0f) {
        const float sum = chain_index(R, floor_v, 0.0f, false, 0.0f, S, nullptr);
        if (sum > 0.0f) {
            float thr;
            if (top_p_threshold(R, floor_v, sum, tp, S, &thr)) floor_v = fmaxf(floor_v, thr);
            else none = true;  // threshold f32::MAX: every p becomes 0
        }
    }
    const float sum = none ? 0.0f : chain_index(R, floor_v, 0.0f, false, 0.0f, S, nullptr);
    if (!(sum > 0.0f)) {
        const int i = last_max(R, false, -INFINITY, S);
        if (threadIdx.x == 0) out[row] = (uint32_t)i;
        return;
    }
    if (threadIdx.x == 0) {
        uint64_t x = rng[row];
        x ^= x << 13;
        x ^= x >> 7;
        x ^= x << 17;
        rng[row] = x;
        S.r = (float)(x >> 40) / 16777216.0f;
    }
    __syncthreads();
    const float r = S.r;
    __syncthreads();
    int pick = -1;
    chain_index(R, floor_v, sum, true, r, S, &pick);
    if (pick >= 0) {
        if (threadIdx.x == 0) out[row] = (uint32_t)pick;
        return;
    }
    const int i = last_max(R, true, floor_v, S);
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

HC_EXPORT int hc_argmax_dev(const float* logits_dev, size_t ld, int B, int V, int shards, float* pairs_dev,
                            uint32_t* out_dev, void* stream) {
    HC_CHECK(B >= 0 && V > 0 && ld >= (size_t)V && shards >= 1 && V % shards == 0, HC_ERR_INVALID,
             "hc_argmax_dev: bad shape (B %d, V %d, ld %zu, shards %d)", B, V, ld, shards);
    HC_CHECK(B == 0 || (logits_dev && out_dev && (shards == 1 || pairs_dev)), HC_ERR_INVALID,
             "hc_argmax_dev: NULL argument");
    cudaStream_t s = (cudaStream_t)stream;
    if (shards == 1) return hc::launch_argmax(logits_dev, (size_t)B, (size_t)V, ld, out_dev, s);
    const size_t vs = (size_t)(V / shards);
    float2* pairs = reinterpret_cast<float2*>(pairs_dev);
    for (int r = 0; r < shards; r++)
        HC_TRY(hc::launch_argmax_pairs(logits_dev + r * vs, (size_t)B, vs, ld, (uint32_t)(r * vs),
                                       pairs + (size_t)r * B, s));
    return hc::launch_pick_pairs(pairs, (size_t)B, shards, out_dev, s);
}
