/*
 * hypno_oracle.c — CPU restatement of hypno's Q4_0 inference path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the sm_100a
 * backend in hypno_b200/: only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load it.  It is never
 * the thing measured or shipped on the GPU path.
 *
 * The reference (HypnotizerAI/hypno, Rust) cannot be compiled in this image
 * (no cargo/rustc), so this is a from-scratch C restatement that keeps the
 * reference's arithmetic order: the AVX2 kernels are reproduced with the same
 * intrinsics in the same order, scalar loops keep Rust's "no FMA contraction"
 * semantics (build with -ffp-contract=off), and libm calls (expf, powf, cosf,
 * sinf, sqrtf, roundf) are the same glibc functions Rust's f32 methods bind to
 * on Linux.  Every function cites the reference file:line it follows
 * (paths relative to crates/hypno/src/).
 *
 * Parity pinning: the reference ships no golden vectors.  The restatement is
 * pinned by the reference's own unit tests re-expressed in
 * tests/test_oracle_reference_cases.py (quant.rs:213-237, kernels.rs:708-742,
 * ops.rs:113-137, transformer.rs:671-719, loader.rs:298-319,
 * sft_convert.rs:430-457, turbo.rs:474-1005) and by known-answer tests for
 * the f16 rounding of the `half` 2.7.1 crate (IEEE round-to-nearest-even).
 * Beyond those self-consistency checks parity with the reference is
 * "unpinned" (no runnable reference exists in this image).
 */
#include <immintrin.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <stdio.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------ */
/* f16 <-> f32 (half 2.7.1 semantics: IEEE 754 binary16, RNE)           */
/* ------------------------------------------------------------------ */

/* f16::from_f32 — round to nearest, ties to even; overflow -> inf. */
ORC_API uint16_t orc_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xFFu;
    uint32_t man = x & 0x7FFFFFu;
    if (exp == 0xFFu) {
        if (man == 0) return (uint16_t)(sign | 0x7C00u);
        return (uint16_t)(sign | 0x7E00u | (man >> 13));
    }
    int e = (int)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        /* f16 subnormal: value = m * 2^-24 */
        if (exp == 0) return (uint16_t)sign; /* f32 subnormal/zero -> 0 */
        uint32_t full = man | 0x800000u;
        int shift = 14 - e;
        if (shift > 24) return (uint16_t)sign;
        uint32_t m = full >> shift;
        uint32_t rem = full & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (m & 1u))) m++;
        return (uint16_t)(sign | m);
    }
    uint32_t m = man >> 13;
    uint32_t rem = man & 0x1FFFu;
    uint32_t out = sign | ((uint32_t)e << 10);
    if (rem > 0x1000u || (rem == 0x1000u && (m & 1u))) m++;
    return (uint16_t)(out + m); /* mantissa carry rolls into the exponent */
}

/* f16::to_f32 — exact. */
ORC_API float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = ((uint32_t)h >> 10) & 0x1Fu;
    uint32_t man = (uint32_t)h & 0x3FFu;
    uint32_t out;
    if (exp == 0) {
        if (man == 0) {
            out = sign;
        } else {
            int e = -1;
            do { e++; man <<= 1; } while (!(man & 0x400u));
            out = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FFu) << 13);
        }
    } else if (exp == 0x1F) {
        out = sign | 0x7F800000u | (man << 13);
    } else {
        out = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &out, 4);
    return f;
}

static inline float rd_f16(const uint8_t* p) {
    return orc_f16_to_f32((uint16_t)(p[0] | ((uint16_t)p[1] << 8)));
}

/* ------------------------------------------------------------------ */
/* Q4_0 blocks — quant.rs:10-153                                       */
/* ------------------------------------------------------------------ */

/* Q4_0Block::quantize, quant.rs:49-71. */
static void q4_quantize_block(const float* src, uint8_t* out18) {
    float max_abs = 0.0f;
    for (int i = 0; i < 32; i++) {
        float a = fabsf(src[i]);
        max_abs = fmaxf(max_abs, a); /* fold(0.0, f32::max) */
    }
    float scale = (max_abs > 0.0f) ? max_abs / 7.0f : 1.0f;
    uint16_t h = orc_f32_to_f16(scale);
    out18[0] = (uint8_t)(h & 0xFF);
    out18[1] = (uint8_t)(h >> 8);
    for (int i = 0; i < 16; i++) {
        float v0 = src[i * 2], v1 = src[i * 2 + 1];
        /* (v / scale).round() as i32 — the UNROUNDED f32 scale, half away from zero */
        float r0 = roundf(v0 / scale), r1 = roundf(v1 / scale);
        int q0 = isnan(r0) ? 0 : (r0 >= 2147483647.0f ? 2147483647 : (r0 <= -2147483648.0f ? (-2147483647 - 1) : (int)r0));
        int q1 = isnan(r1) ? 0 : (r1 >= 2147483647.0f ? 2147483647 : (r1 <= -2147483648.0f ? (-2147483647 - 1) : (int)r1));
        if (q0 < -8) q0 = -8;
        if (q0 > 7) q0 = 7;
        if (q1 < -8) q1 = -8;
        if (q1 > 7) q1 = 7;
        uint8_t n0 = (uint8_t)((q0 + 8) & 0x0F), n1 = (uint8_t)((q1 + 8) & 0x0F);
        out18[2 + i] = (uint8_t)(n0 | (n1 << 4));
    }
}

/* quantize_f32_to_q4_0, quant.rs:108-117: floor(n/32) blocks. */
ORC_API void orc_q4_0_quantize(const float* x, size_t n, uint8_t* out) {
    size_t nb = n / 32;
    #pragma omp parallel for schedule(static)
    for (long long b = 0; b < (long long)nb; b++) q4_quantize_block(x + (size_t)b * 32, out + (size_t)b * 18);
}

/* Q4_0Block::dequantize, quant.rs:25-34. */
static inline void q4_dequant_block(const uint8_t* blk, float* dst) {
    float scale = rd_f16(blk);
    for (int i = 0; i < 16; i++) {
        uint8_t byte = blk[2 + i];
        dst[i * 2] = (float)((int)(byte & 0x0F) - 8) * scale;
        dst[i * 2 + 1] = (float)((int)((byte >> 4) & 0x0F) - 8) * scale;
    }
}

/* dequantize_q4_0, quant.rs:120-132: floor(len/18) blocks. */
ORC_API void orc_q4_0_dequantize(const uint8_t* q, size_t nbytes, float* out) {
    size_t nb = nbytes / 18;
    #pragma omp parallel for schedule(static)
    for (long long b = 0; b < (long long)nb; b++) q4_dequant_block(q + (size_t)b * 18, out + (size_t)b * 32);
}

/* q4_0_extract_row, quant.rs:139-153. */
ORC_API void orc_q4_0_extract_row(const uint8_t* q, size_t row, size_t width, float* out) {
    size_t bpr = width / 32, start = row * bpr;
    for (size_t i = 0; i < bpr; i++) q4_dequant_block(q + (start + i) * 18, out + i * 32);
}

/* ------------------------------------------------------------------ */
/* SIMD helpers — kernels.rs:166-178                                   */
/* ------------------------------------------------------------------ */

/* hsum256, kernels.rs:169-178: (lo+hi) then two hadds. */
static inline float hsum256(__m256 v) {
    __m128 hi = _mm256_extractf128_ps(v, 1);
    __m128 lo = _mm256_castps256_ps128(v);
    __m128 s = _mm_add_ps(lo, hi);
    s = _mm_hadd_ps(s, s);
    s = _mm_hadd_ps(s, s);
    return _mm_cvtss_f32(s);
}

static int g_has_avx512 = -1;
static int has_avx512(void) {
    if (g_has_avx512 < 0) {
        __builtin_cpu_init();
        g_has_avx512 = __builtin_cpu_supports("avx512f") ? 1 : 0;
    }
    return g_has_avx512;
}

/* ------------------------------------------------------------------ */
/* Q4_0 matvec — kernels.rs:256-359 (AVX2 path)                        */
/* ------------------------------------------------------------------ */

static void q4_row(float* yi, const uint8_t* wq, size_t wlen, const float* x, const float* bias,
                   size_t row, size_t m) {
    size_t row_start = row * m, row_end = row_start + m;
    size_t first_block = row_start / 32;
    size_t last_block = (row_end > 0 ? row_end - 1 : 0) / 32;
    __m256 acc0 = _mm256_setzero_ps(), acc1 = _mm256_setzero_ps();
    __m256 acc2 = _mm256_setzero_ps(), acc3 = _mm256_setzero_ps();
    float scalar_tail = 0.0f;
    float deq[32];
    for (size_t b = first_block; b <= last_block; b++) {
        size_t bo = b * 18;
        if (bo + 18 > wlen) break;
        q4_dequant_block(wq + bo, deq);
        size_t block_start = b * 32;
        size_t ov_start = block_start < row_start ? row_start - block_start : 0;
        size_t ov_end = block_start + 32 > row_end ? row_end - block_start : 32;
        size_t x_off = block_start > row_start ? block_start - row_start : 0;
        if (ov_start == 0 && ov_end == 32) {
            acc0 = _mm256_fmadd_ps(_mm256_loadu_ps(deq), _mm256_loadu_ps(x + x_off), acc0);
            acc1 = _mm256_fmadd_ps(_mm256_loadu_ps(deq + 8), _mm256_loadu_ps(x + x_off + 8), acc1);
            acc2 = _mm256_fmadd_ps(_mm256_loadu_ps(deq + 16), _mm256_loadu_ps(x + x_off + 16), acc2);
            acc3 = _mm256_fmadd_ps(_mm256_loadu_ps(deq + 24), _mm256_loadu_ps(x + x_off + 24), acc3);
        } else {
            for (size_t i = ov_start; i < ov_end; i++) scalar_tail += deq[i] * x[x_off + (i - ov_start)];
        }
    }
    __m256 s01 = _mm256_add_ps(acc0, acc1);
    __m256 s23 = _mm256_add_ps(acc2, acc3);
    __m256 sall = _mm256_add_ps(s01, s23);
    float total = hsum256(sall) + scalar_tail;
    if (bias) total += bias[row];
    *yi = total;
}

/* matmul_q4_0_scalar, kernels.rs:362-400 (used when the buffer is short). */
static void q4_row_scalar(float* yi, const uint8_t* wq, size_t wlen, const float* x, const float* bias,
                          size_t row, size_t m) {
    size_t row_start = row * m, row_end = row_start + m;
    size_t first_block = row_start / 32;
    size_t last_block = (row_end > 0 ? row_end - 1 : 0) / 32;
    float sum = 0.0f, deq[32];
    for (size_t b = first_block; b <= last_block; b++) {
        size_t bo = b * 18;
        if (bo + 18 > wlen) break;
        q4_dequant_block(wq + bo, deq);
        size_t block_start = b * 32;
        size_t ov_start = block_start < row_start ? row_start - block_start : 0;
        size_t ov_end = block_start + 32 > row_end ? row_end - block_start : 32;
        size_t x_off = block_start > row_start ? block_start - row_start : 0;
        for (size_t i = ov_start; i < ov_end; i++) sum += deq[i] * x[x_off + (i - ov_start)];
    }
    *yi = sum + (bias ? bias[row] : 0.0f);
}

/* matmul_q4_0 dispatch, kernels.rs:256-265 / 270-277. */
ORC_API void orc_matmul_q4_0(float* y, const uint8_t* wq, size_t wlen, const float* x, const float* bias,
                             size_t n, size_t m) {
    size_t total_blocks = (n * m + 31) / 32;
    int short_buf = wlen < total_blocks * 18;
    #pragma omp parallel for schedule(static)
    for (long long r = 0; r < (long long)n; r++) {
        if (short_buf) q4_row_scalar(y + r, wq, wlen, x, bias, (size_t)r, m);
        else q4_row(y + r, wq, wlen, x, bias, (size_t)r, m);
    }
}

/* ------------------------------------------------------------------ */
/* FP32 / FP16 matvec — kernels.rs:69-241, 537-586                     */
/* ------------------------------------------------------------------ */

__attribute__((target("avx512f")))
static float f32_row_avx512(const float* row, const float* x, size_t m) {
    size_t m16 = m - (m % 16);
    __m512 acc = _mm512_setzero_ps();
    for (size_t j = 0; j < m16; j += 16) acc = _mm512_fmadd_ps(_mm512_loadu_ps(row + j), _mm512_loadu_ps(x + j), acc);
    float sum = _mm512_reduce_add_ps(acc);
    for (size_t j = m16; j < m; j++) sum += row[j] * x[j];
    return sum;
}

/* matmul_f32: AVX-512 path kernels.rs:214-230, else AVX2 kernels.rs:93-164. */
ORC_API void orc_matmul_f32(float* y, const float* w, const float* x, const float* bias, size_t n, size_t m) {
    if (has_avx512()) {
        #pragma omp parallel for schedule(static)
        for (long long r = 0; r < (long long)n; r++)
            y[r] = f32_row_avx512(w + (size_t)r * m, x, m) + (bias ? bias[r] : 0.0f);
        return;
    }
    size_t m8 = m - (m % 8), n16 = n - (n % 16);
    #pragma omp parallel for schedule(static)
    for (long long base = 0; base < (long long)n16; base += 16) {
        for (int r = 0; r < 16; r++) {
            const float* row = w + ((size_t)base + r) * m;
            __m256 acc[8];
            for (int k = 0; k < 8; k++) acc[k] = _mm256_setzero_ps();
            for (size_t j = 0; j < m8; j += 64) {
                for (int k = 0; k < 8; k++) {
                    size_t col = j + (size_t)k * 8;
                    if (col + 8 > m) break;
                    acc[k] = _mm256_fmadd_ps(_mm256_loadu_ps(row + col), _mm256_loadu_ps(x + col), acc[k]);
                }
            }
            __m256 sum = acc[0];
            for (int k = 1; k < 8; k++) sum = _mm256_add_ps(sum, acc[k]);
            float s = hsum256(sum);
            for (size_t j = m8; j < m; j++) s += row[j] * x[j];
            if (bias) s += bias[base + r];
            y[base + r] = s;
        }
    }
    for (size_t r = n16; r < n; r++) {
        const float* row = w + r * m;
        float s = 0.0f;
        for (size_t j = 0; j < m8; j += 8) s += hsum256(_mm256_mul_ps(_mm256_loadu_ps(row + j), _mm256_loadu_ps(x + j)));
        for (size_t j = m8; j < m; j++) s += row[j] * x[j];
        y[r] = s + (bias ? bias[r] : 0.0f);
    }
}

/* matmul_f16_avx2_fma, kernels.rs:543-565. */
ORC_API void orc_matmul_f16(float* y, const uint16_t* w, const float* x, const float* bias, size_t n, size_t m) {
    size_t m8 = m - (m % 8);
    #pragma omp parallel for schedule(static)
    for (long long r = 0; r < (long long)n; r++) {
        const uint16_t* row = w + (size_t)r * m;
        __m256 acc = _mm256_setzero_ps();
        for (size_t j = 0; j < m8; j += 8) {
            float wf[8];
            for (int t = 0; t < 8; t++) wf[t] = orc_f16_to_f32(row[j + t]);
            acc = _mm256_fmadd_ps(_mm256_loadu_ps(wf), _mm256_loadu_ps(x + j), acc);
        }
        float s = hsum256(acc);
        for (size_t j = m8; j < m; j++) s += orc_f16_to_f32(row[j]) * x[j];
        y[r] = s + (bias ? bias[r] : 0.0f);
    }
}

/* ------------------------------------------------------------------ */
/* RMSNorm — kernels.rs:592-625 (AVX2 path)                            */
/* ------------------------------------------------------------------ */
ORC_API void orc_rms_norm(float* x, const float* w, size_t n, float eps) {
    size_t n8 = n - (n % 8);
    __m256 sq = _mm256_setzero_ps();
    for (size_t i = 0; i < n8; i += 8) {
        __m256 v = _mm256_loadu_ps(x + i);
        sq = _mm256_fmadd_ps(v, v, sq);
    }
    float mean_sq = hsum256(sq);
    for (size_t i = n8; i < n; i++) mean_sq += x[i] * x[i];
    mean_sq /= (float)n;
    __m256 inv = _mm256_set1_ps(1.0f / sqrtf(mean_sq + eps));
    for (size_t i = 0; i < n8; i += 8) {
        __m256 v = _mm256_loadu_ps(x + i);
        __m256 ww = _mm256_loadu_ps(w + i);
        _mm256_storeu_ps(x + i, _mm256_mul_ps(_mm256_mul_ps(v, inv), ww));
    }
    for (size_t i = n8; i < n; i++) x[i] = x[i] / sqrtf(mean_sq + eps) * w[i];
}

/* ------------------------------------------------------------------ */
/* Softmax — kernels.rs:631-697 (AVX2 path with the exp(v/8) Taylor   */
/* polynomial on the first floor(n/8)*8 entries, libm exp on the tail) */
/* ------------------------------------------------------------------ */
static inline __m256 vsubexp(__m256 v) {
    v = _mm256_min_ps(_mm256_max_ps(v, _mm256_set1_ps(-87.0f)), _mm256_set1_ps(87.0f));
    __m256 c1 = _mm256_set1_ps(1.0f / 8.0f), c2 = _mm256_set1_ps(1.0f / 128.0f);
    __m256 c3 = _mm256_set1_ps(1.0f / 3072.0f), c4 = _mm256_set1_ps(1.0f / 98304.0f);
    __m256 x2 = _mm256_mul_ps(v, v);
    __m256 x3 = _mm256_mul_ps(x2, v);
    __m256 x4 = _mm256_mul_ps(x3, v);
    __m256 t1 = _mm256_fmadd_ps(c1, v, _mm256_set1_ps(1.0f));
    __m256 t2 = _mm256_fmadd_ps(c2, x2, t1);
    __m256 t3 = _mm256_fmadd_ps(c3, x3, t2);
    return _mm256_fmadd_ps(c4, x4, t3);
}

ORC_API void orc_softmax(float* x, size_t n) {
    float mx = -INFINITY;
    for (size_t i = 0; i < n; i++) mx = fmaxf(mx, x[i]); /* fold(NEG_INFINITY, f32::max) */
    size_t n8 = n - (n % 8);
    __m256 mv = _mm256_set1_ps(mx);
    __m256 sum = _mm256_setzero_ps();
    for (size_t i = 0; i < n8; i += 8) {
        __m256 e = vsubexp(_mm256_sub_ps(_mm256_loadu_ps(x + i), mv));
        _mm256_storeu_ps(x + i, e);
        sum = _mm256_add_ps(sum, e);
    }
    float total = hsum256(sum);
    for (size_t i = n8; i < n; i++) {
        x[i] = expf(x[i] - mx);
        total += x[i];
    }
    __m256 inv = _mm256_set1_ps(1.0f / total);
    for (size_t i = 0; i < n8; i += 8) _mm256_storeu_ps(x + i, _mm256_mul_ps(_mm256_loadu_ps(x + i), inv));
    for (size_t i = n8; i < n; i++) x[i] /= total;
}

/* silu_in_place, ops.rs:81-83. */
ORC_API void orc_silu(float* x, size_t n) {
    for (size_t i = 0; i < n; i++) x[i] = x[i] / (1.0f + expf(-x[i]));
}

/* rope, ops.rs:86-99 (adjacent pairs). */
ORC_API void orc_rope(float* q, float* k, size_t head_dim, size_t pos, float theta) {
    float pf = (float)pos;
    for (size_t i = 0; i < head_dim; i += 2) {
        float freq = 1.0f / powf(theta, (float)i / (float)head_dim);
        float c = cosf(pf * freq), s = sinf(pf * freq);
        float q0 = q[i], q1 = q[i + 1];
        q[i] = q0 * c - q1 * s;
        q[i + 1] = q0 * s + q1 * c;
        float k0 = k[i], k1 = k[i + 1];
        k[i] = k0 * c - k1 * s;
        k[i + 1] = k0 * s + k1 * c;
    }
}

/* ------------------------------------------------------------------ */
/* .hypno reader — format.rs:1-131, loader.rs:39-160                   */
/* ------------------------------------------------------------------ */
enum { DT_FP32 = 0, DT_FP16 = 1, DT_Q8_0 = 2, DT_Q4_0 = 3 };

typedef struct {
    char* name;
    uint32_t ndim;
    uint64_t shape[8];
    uint32_t dtype;
    uint64_t offset, len;
} orc_tensor;

typedef struct {
    const uint8_t* data;
    size_t size;
    uint32_t n_meta, n_tensors;
    char** keys;
    char** vals;
    orc_tensor* tensors;
    /* HypnoConfig, transformer.rs:27-63 */
    size_t hidden, inter, nh, nkv, layers, vocab, max_pos, head_dim;
    float eps, theta;
} orc_model;

static int rd_u32(const uint8_t* d, size_t size, size_t* cur, uint32_t* out) {
    if (*cur + 4 > size) return -1;
    memcpy(out, d + *cur, 4);
    *cur += 4;
    return 0;
}
static int rd_u64(const uint8_t* d, size_t size, size_t* cur, uint64_t* out) {
    if (*cur + 8 > size) return -1;
    memcpy(out, d + *cur, 8);
    *cur += 8;
    return 0;
}
static char* rd_str(const uint8_t* d, size_t size, size_t* cur, uint32_t len) {
    if (*cur + len > size) return NULL;
    char* s = (char*)malloc((size_t)len + 1);
    memcpy(s, d + *cur, len);
    s[len] = 0;
    *cur += len;
    return s;
}

ORC_API const char* orc_meta(const orc_model* m, const char* key) {
    for (uint32_t i = 0; i < m->n_meta; i++)
        if (strcmp(m->keys[i], key) == 0) return m->vals[i];
    return NULL;
}

static const orc_tensor* find_tensor(const orc_model* m, const char* name) {
    for (uint32_t i = 0; i < m->n_tensors; i++)
        if (strcmp(m->tensors[i].name, name) == 0) return &m->tensors[i];
    return NULL;
}

ORC_API void orc_model_free(orc_model* m);

/* HypnoModel::open, loader.rs:39-133, over an in-memory image (the bytes an
 * mmap would expose).  Returns NULL with *err set on a malformed image. */
ORC_API orc_model* orc_model_open(const uint8_t* data, size_t size, int* err) {
    *err = 0;
    if (size < 16) { *err = 1; return NULL; }
    if (memcmp(data, "HYPN", 4) != 0) { *err = 2; return NULL; }
    uint32_t ver, nkv, nt;
    memcpy(&ver, data + 4, 4);
    memcpy(&nkv, data + 8, 4);
    memcpy(&nt, data + 12, 4);
    if (ver != 1) { *err = 3; return NULL; }
    orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
    m->data = data;
    m->size = size;
    m->keys = (char**)calloc(nkv + 1, sizeof(char*));
    m->vals = (char**)calloc(nkv + 1, sizeof(char*));
    m->tensors = (orc_tensor*)calloc(nt + 1, sizeof(orc_tensor));
    size_t cur = 16;
    for (uint32_t i = 0; i < nkv; i++) {
        uint32_t kl, vl;
        if (rd_u32(data, size, &cur, &kl)) goto fail;
        if (!(m->keys[i] = rd_str(data, size, &cur, kl))) goto fail;
        m->n_meta = i + 1;
        if (rd_u32(data, size, &cur, &vl)) goto fail;
        if (!(m->vals[i] = rd_str(data, size, &cur, vl))) goto fail;
    }
    for (uint32_t i = 0; i < nt; i++) {
        orc_tensor* t = &m->tensors[i];
        uint32_t nl;
        if (rd_u32(data, size, &cur, &nl)) goto fail;
        if (!(t->name = rd_str(data, size, &cur, nl))) goto fail;
        m->n_tensors = i + 1;
        if (rd_u32(data, size, &cur, &t->ndim)) goto fail;
        if (t->ndim > 8) goto fail;
        for (uint32_t d = 0; d < t->ndim; d++)
            if (rd_u64(data, size, &cur, &t->shape[d])) goto fail;
        if (rd_u32(data, size, &cur, &t->dtype)) goto fail;
        if (t->dtype > 3) { *err = 5; goto fail2; }
        if (rd_u64(data, size, &cur, &t->offset)) goto fail;
        if (rd_u64(data, size, &cur, &t->len)) goto fail;
        if (t->offset > size || t->offset + t->len > size) { *err = 6; goto fail2; }
    }
    {
        /* HypnoConfig::from_model, transformer.rs:42-63 */
        const char* s;
        if (!(s = orc_meta(m, "hidden_size"))) { *err = 7; goto fail2; }
        m->hidden = strtoull(s, NULL, 10);
        if (!(s = orc_meta(m, "num_attention_heads"))) { *err = 7; goto fail2; }
        m->nh = strtoull(s, NULL, 10);
        m->nkv = (s = orc_meta(m, "num_key_value_heads")) ? strtoull(s, NULL, 10) : m->nh;
        m->head_dim = m->hidden / m->nh;
        m->inter = (s = orc_meta(m, "intermediate_size")) ? strtoull(s, NULL, 10) : m->hidden * 8 / 3;
        m->layers = (s = orc_meta(m, "num_hidden_layers")) ? strtoull(s, NULL, 10) : 0;
        m->vocab = (s = orc_meta(m, "vocab_size")) ? strtoull(s, NULL, 10) : 32000;
        m->max_pos = (s = orc_meta(m, "max_position_embeddings")) ? strtoull(s, NULL, 10) : 2048;
        m->eps = (s = orc_meta(m, "rms_norm_eps")) ? strtof(s, NULL) : 1e-5f;
        m->theta = (s = orc_meta(m, "rope_theta")) ? strtof(s, NULL) : 10000.0f;
    }
    m->n_meta = nkv;
    m->n_tensors = nt;
    return m;
fail:
    *err = 4;
fail2:
    orc_model_free(m);
    return NULL;
}

ORC_API void orc_model_free(orc_model* m) {
    if (!m) return;
    for (uint32_t i = 0; i < m->n_meta; i++) { free(m->keys[i]); free(m->vals[i]); }
    for (uint32_t i = 0; i < m->n_tensors; i++) free(m->tensors[i].name);
    free(m->keys);
    free(m->vals);
    free(m->tensors);
    free(m);
}

ORC_API void orc_model_config(const orc_model* m, uint64_t* out10, float* out2) {
    out10[0] = m->hidden; out10[1] = m->inter; out10[2] = m->nh; out10[3] = m->nkv;
    out10[4] = m->layers; out10[5] = m->vocab; out10[6] = m->max_pos; out10[7] = m->head_dim;
    out10[8] = m->n_tensors; out10[9] = m->n_meta;
    out2[0] = m->eps; out2[1] = m->theta;
}

/* get_tensor_data, loader.rs:139-148. Returns 0 and fills ptr/len/dtype, -1 if absent. */
ORC_API int orc_tensor_data(const orc_model* m, const char* name, const uint8_t** ptr, uint64_t* len, uint32_t* dtype) {
    const orc_tensor* t = find_tensor(m, name);
    if (!t || t->offset + t->len > m->size) return -1;
    *ptr = m->data + t->offset;
    *len = t->len;
    *dtype = t->dtype;
    return 0;
}

/* ------------------------------------------------------------------ */
/* Forward pass — transformer.rs:89-528, turbo.rs:22-368               */
/* ------------------------------------------------------------------ */

/* FlatKVCache, transformer.rs:89-184: per layer [nkv][max_pos][hd]. */
typedef struct {
    size_t layers, nkv, max_pos, hd, pos;
    float* k;
    float* v;
} orc_kv;

ORC_API orc_kv* orc_kv_new(size_t layers, size_t nkv, size_t max_pos, size_t hd) {
    orc_kv* c = (orc_kv*)calloc(1, sizeof(orc_kv));
    c->layers = layers; c->nkv = nkv; c->max_pos = max_pos; c->hd = hd; c->pos = 0;
    size_t n = layers * nkv * max_pos * hd;
    c->k = (float*)calloc(n ? n : 1, sizeof(float));
    c->v = (float*)calloc(n ? n : 1, sizeof(float));
    return c;
}
ORC_API void orc_kv_free(orc_kv* c) { if (c) { free(c->k); free(c->v); free(c); } }
ORC_API size_t orc_kv_pos(const orc_kv* c) { return c->pos; }
ORC_API void orc_kv_set_pos(orc_kv* c, size_t p) { c->pos = p; }
ORC_API float* orc_kv_k(orc_kv* c) { return c->k; }
ORC_API float* orc_kv_v(orc_kv* c) { return c->v; }

static inline float* kv_at(const orc_kv* c, float* base, size_t layer, size_t h, size_t pos) {
    return base + ((layer * c->nkv + h) * c->max_pos + pos) * c->hd;
}

/* store_at, transformer.rs:161-173. */
static void kv_store_at(orc_kv* c, size_t layer, const float* k, const float* v, size_t pos) {
    for (size_t h = 0; h < c->nkv; h++) {
        memcpy(kv_at(c, c->k, layer, h, pos), k + h * c->hd, c->hd * sizeof(float));
        memcpy(kv_at(c, c->v, layer, h, pos), v + h * c->hd, c->hd * sizeof(float));
    }
}

/* matmul_vec_auto, ops.rs:25-38 (Q8_0 not supported by the oracle). */
static int matvec_auto(float* y, const uint8_t* w, uint64_t wlen, uint32_t dt, const float* x, size_t n, size_t m) {
    switch (dt) {
        case DT_FP32: orc_matmul_f32(y, (const float*)w, x, NULL, n, m); return 0;
        case DT_FP16: orc_matmul_f16(y, (const uint16_t*)w, x, NULL, n, m); return 0;
        case DT_Q4_0: orc_matmul_q4_0(y, w, wlen, x, NULL, n, m); return 0;
        default: return -1;
    }
}

/* Looks up "<prefix><suffix>"; missing tensors are skipped the way the
 * reference's `if let Some(..)` branches skip them. */
static int get_w(const orc_model* m, const char* prefix, const char* suffix, const uint8_t** p, uint64_t* len, uint32_t* dt) {
    char name[256];
    snprintf(name, sizeof name, "%s%s", prefix, suffix);
    return orc_tensor_data(m, name, p, len, dt);
}

/* load_1d_f32 / load_norm_f32, transformer.rs:250-264, turbo.rs:355-368. */
static void load_norm(const orc_model* m, const char* name, size_t len, float* out) {
    const uint8_t* p; uint64_t l; uint32_t dt;
    if (orc_tensor_data(m, name, &p, &l, &dt) == 0 && (dt == DT_FP32 || dt == DT_FP16)) {
        for (size_t i = 0; i < len; i++) {
            if (dt == DT_FP32) memcpy(&out[i], p + 4 * i, 4);
            else out[i] = rd_f16(p + 2 * i);
        }
    } else {
        for (size_t i = 0; i < len; i++) out[i] = 1.0f;
    }
}

/* Embedding row, transformer.rs:477-500 / turbo.rs:40-66. */
static void embed_row(const orc_model* m, uint32_t tid, float* out) {
    const uint8_t* p; uint64_t l; uint32_t dt;
    size_t hd = m->hidden;
    if (orc_tensor_data(m, "model.embed_tokens.weight", &p, &l, &dt) != 0) {
        memset(out, 0, hd * sizeof(float));
        return;
    }
    if (dt == DT_FP32) memcpy(out, p + (size_t)tid * hd * 4, hd * 4);
    else if (dt == DT_FP16) { for (size_t i = 0; i < hd; i++) out[i] = rd_f16(p + ((size_t)tid * hd + i) * 2); }
    else if (dt == DT_Q4_0) orc_q4_0_extract_row(p, tid, hd, out);
    else memset(out, 0, hd * sizeof(float));
}

static void lm_head(const orc_model* m, const float* h, float* logits) {
    const uint8_t* p; uint64_t l; uint32_t dt;
    if (orc_tensor_data(m, "lm_head.weight", &p, &l, &dt) == 0 ||
        orc_tensor_data(m, "model.embed_tokens.weight", &p, &l, &dt) == 0) {
        if (matvec_auto(logits, p, l, dt, h, m->vocab, m->hidden) == 0) return;
    }
    memset(logits, 0, m->vocab * sizeof(float));
}

/* transformer_layer_forward (use_kv_cache = true, row-major),
 * transformer.rs:281-462. */
static void layer_forward(const orc_model* m, orc_kv* kv, size_t li, float* hidden, float* scratch) {
    size_t hd = m->hidden, im = m->inter, nh = m->nh, nkv = m->nkv, hdim = m->head_dim;
    float* residual = scratch;
    float* q = residual + hd;
    float* k = q + nh * hdim;
    float* v = k + nkv * hdim;
    float* attn = v + nkv * hdim;
    float* gate = attn + hd;
    float* up = gate + im;
    float* down = up + im;
    float* scores = down + hd;
    float* normw = scores + kv->max_pos + 8;
    float* tmp = normw + hd;
    char prefix[64];
    snprintf(prefix, sizeof prefix, "model.layers.%zu.", li);
    const uint8_t* p; uint64_t l; uint32_t dt;
    char nm[256];

    memcpy(residual, hidden, hd * 4);
    snprintf(nm, sizeof nm, "%sinput_layernorm.weight", prefix);
    load_norm(m, nm, hd, normw);
    orc_rms_norm(hidden, normw, hd, m->eps);

    if (get_w(m, prefix, "self_attn.q_proj.weight", &p, &l, &dt) == 0) matvec_auto(q, p, l, dt, hidden, nh * hdim, hd);
    if (get_w(m, prefix, "self_attn.k_proj.weight", &p, &l, &dt) == 0) matvec_auto(k, p, l, dt, hidden, nkv * hdim, hd);
    if (get_w(m, prefix, "self_attn.v_proj.weight", &p, &l, &dt) == 0) matvec_auto(v, p, l, dt, hidden, nkv * hdim, hd);

    size_t pos = kv->pos;
    /* K RoPE, transformer.rs:317-328 */
    for (size_t h = 0; h < nkv; h++) {
        float* kk = k + h * hdim;
        for (size_t i = 0; i < hdim; i += 2) {
            float freq = 1.0f / powf(m->theta, (float)i / (float)hdim);
            float c = cosf((float)pos * freq), s = sinf((float)pos * freq);
            float k0 = kk[i], k1 = kk[i + 1];
            kk[i] = k0 * c - k1 * s;
            kk[i + 1] = k0 * s + k1 * c;
        }
    }
    /* Q RoPE via ops::rope on a copy of K, transformer.rs:330-343 */
    for (size_t h = 0; h < nh; h++) {
        float dummy[512];
        size_t kvh = h * nkv / nh;
        if (kvh > nkv - 1) kvh = nkv - 1;
        memcpy(dummy, k + kvh * hdim, hdim * 4);
        orc_rope(q + h * hdim, dummy, hdim, pos, m->theta);
    }
    kv_store_at(kv, li, k, v, pos); /* store, transformer.rs:124-139 */

    size_t seq_len = kv->pos;
    float scale = 1.0f / sqrtf((float)hdim);
    size_t per = nh / nkv;
    memset(attn, 0, hd * 4);
    for (size_t qh = 0; qh < nh; qh++) {
        size_t kvh = qh / per;
        float* qq = q + qh * hdim;
        float* o = attn + qh * hdim;
        if (seq_len > 1) {
            for (size_t ps = 0; ps < seq_len; ps++) {
                const float* kp = kv_at(kv, kv->k, li, kvh, ps);
                float dot = 0.0f;
                for (size_t d = 0; d < hdim; d++) dot += qq[d] * kp[d];
                scores[ps] = dot * scale;
            }
            orc_softmax(scores, seq_len);
            for (size_t ps = 0; ps < seq_len; ps++) {
                float aw = scores[ps];
                const float* vp = kv_at(kv, kv->v, li, kvh, ps);
                for (size_t d = 0; d < hdim; d++) o[d] += aw * vp[d];
            }
        } else {
            float aw = 1.0f;
            if (seq_len > 0) {
                float dot = 0.0f;
                for (size_t d = 0; d < hdim; d++) dot += qq[d] * k[kvh * hdim + d];
                scores[0] = dot * scale;
                orc_softmax(scores, 1);
                aw = scores[0];
            }
            for (size_t d = 0; d < hdim; d++) o[d] = aw * v[kvh * hdim + d];
        }
    }

    if (get_w(m, prefix, "self_attn.o_proj.weight", &p, &l, &dt) == 0) {
        memcpy(tmp, attn, hd * 4);
        matvec_auto(hidden, p, l, dt, tmp, hd, hd);
    } else {
        memcpy(hidden, attn, hd * 4);
    }
    for (size_t i = 0; i < hd; i++) hidden[i] += residual[i];

    memcpy(residual, hidden, hd * 4);
    snprintf(nm, sizeof nm, "%spost_attention_layernorm.weight", prefix);
    load_norm(m, nm, hd, normw);
    orc_rms_norm(hidden, normw, hd, m->eps);
    if (get_w(m, prefix, "mlp.gate_proj.weight", &p, &l, &dt) == 0) matvec_auto(gate, p, l, dt, hidden, im, hd);
    if (get_w(m, prefix, "mlp.up_proj.weight", &p, &l, &dt) == 0) matvec_auto(up, p, l, dt, hidden, im, hd);
    orc_silu(gate, im);
    for (size_t i = 0; i < im; i++) gate[i] *= up[i];
    if (get_w(m, prefix, "mlp.down_proj.weight", &p, &l, &dt) == 0) matvec_auto(down, p, l, dt, gate, hd, im);
    else memcpy(down, gate, hd * 4);
    for (size_t i = 0; i < hd; i++) hidden[i] = residual[i] + down[i];
}

static size_t scratch_floats(const orc_model* m, size_t max_pos) {
    return 8 * m->hidden + 2 * m->nh * m->head_dim + 4 * m->nkv * m->head_dim + 3 * m->inter + max_pos + 64;
}

/* model_forward(use_kv_cache = true, col_major = false), transformer.rs:465-528.
 * hidden_io (len hidden) receives the final hidden state when non-NULL. */
ORC_API int orc_model_forward(const orc_model* m, orc_kv* kv, uint32_t token, float* logits) {
    if (kv->pos >= kv->max_pos) return -1;
    if (m->head_dim > 512 || m->nkv == 0) return -2;
    float* hidden = (float*)malloc(m->hidden * 4);
    float* scratch = (float*)malloc(scratch_floats(m, kv->max_pos) * 4);
    float* normw = (float*)malloc(m->hidden * 4);
    embed_row(m, token, hidden);
    for (size_t li = 0; li < m->layers; li++) layer_forward(m, kv, li, hidden, scratch);
    kv->pos += 1; /* advance, transformer.rs:508-510 */
    load_norm(m, "model.norm.weight", m->hidden, normw);
    orc_rms_norm(hidden, normw, m->hidden, m->eps);
    lm_head(m, hidden, logits);
    free(hidden); free(scratch); free(normw);
    return 0;
}

/* batch_matmul, turbo.rs:306-343: T independent matvecs (Q4_0 / FP32 / FP16). */
static void batch_matmul(float* y, const uint8_t* w, uint64_t wlen, uint32_t dt, const float* x,
                         size_t n, size_t dim, size_t T) {
    if (dt == DT_Q4_0) {
        size_t total_blocks = (n * dim + 31) / 32;
        int short_buf = wlen < total_blocks * 18;
        #pragma omp parallel for collapse(2) schedule(static)
        for (long long t = 0; t < (long long)T; t++)
            for (long long r = 0; r < (long long)n; r++) {
                if (short_buf) q4_row_scalar(y + t * n + r, w, wlen, x + t * dim, NULL, (size_t)r, dim);
                else q4_row(y + t * n + r, w, wlen, x + t * dim, NULL, (size_t)r, dim);
            }
    } else {
        for (size_t t = 0; t < T; t++) matvec_auto(y + t * n, w, wlen, dt, x + t * dim, n, dim);
    }
}

static inline float silu1(float x) { return x / (1.0f + expf(-x)); } /* turbo.rs:345-348 */

/* batch_forward, turbo.rs:22-281 (col_major = false).  When hidden_out is
 * non-NULL it receives the pre-final-norm hidden states [T, hidden]. */
ORC_API int orc_batch_forward(const orc_model* m, orc_kv* kv, const uint32_t* ids, size_t T, float* logits) {
    size_t hd = m->hidden, im = m->inter, nh = m->nh, nkv = m->nkv, hdim = m->head_dim;
    size_t cache_pos = kv->pos;
    if (cache_pos + T > kv->max_pos) return -1;
    if (T == 0) { memset(logits, 0, m->vocab * 4); return 0; }
    float* hidden = (float*)malloc(T * hd * 4);
    float* residual = (float*)malloc(T * hd * 4);
    float* normed = (float*)malloc(T * hd * 4);
    float* q = (float*)malloc(T * nh * hdim * 4);
    float* k = (float*)malloc(T * nkv * hdim * 4);
    float* v = (float*)malloc(T * nkv * hdim * 4);
    float* attn = (float*)malloc(T * hd * 4);
    float* g = (float*)malloc(T * im * 4);
    float* u = (float*)malloc(T * im * 4);
    float* dn = (float*)malloc(T * hd * 4);
    float* ob = (float*)malloc(T * hd * 4);
    float* scores = (float*)malloc((T + 8) * 4);
    float* nw = (float*)malloc(hd * 4);
    float scale = 1.0f / sqrtf((float)hdim);
    char prefix[64], nm[256];
    const uint8_t* p; uint64_t l; uint32_t dt;

    for (size_t t = 0; t < T; t++) embed_row(m, ids[t], hidden + t * hd);

    for (size_t li = 0; li < m->layers; li++) {
        snprintf(prefix, sizeof prefix, "model.layers.%zu.", li);
        snprintf(nm, sizeof nm, "%sinput_layernorm.weight", prefix);
        load_norm(m, nm, hd, nw);
        for (size_t t = 0; t < T; t++) {
            memcpy(normed + t * hd, hidden + t * hd, hd * 4);
            orc_rms_norm(normed + t * hd, nw, hd, m->eps);
        }
        if (get_w(m, prefix, "self_attn.q_proj.weight", &p, &l, &dt) == 0) batch_matmul(q, p, l, dt, normed, nh * hdim, hd, T);
        if (get_w(m, prefix, "self_attn.k_proj.weight", &p, &l, &dt) == 0) batch_matmul(k, p, l, dt, normed, nkv * hdim, hd, T);
        if (get_w(m, prefix, "self_attn.v_proj.weight", &p, &l, &dt) == 0) batch_matmul(v, p, l, dt, normed, nkv * hdim, hd, T);

        /* RoPE, turbo.rs:113-142 */
        for (size_t t = 0; t < T; t++) {
            size_t pos = cache_pos + t;
            for (size_t h = 0; h < nh; h++) {
                float* qq = q + (t * nh + h) * hdim;
                for (size_t i = 0; i < hdim; i += 2) {
                    float freq = 1.0f / powf(m->theta, (float)i / (float)hdim);
                    float c = cosf((float)pos * freq), s = sinf((float)pos * freq);
                    float q0 = qq[i], q1 = qq[i + 1];
                    qq[i] = q0 * c - q1 * s;
                    qq[i + 1] = q0 * s + q1 * c;
                }
            }
            for (size_t h = 0; h < nkv; h++) {
                float* kk = k + (t * nkv + h) * hdim;
                for (size_t i = 0; i < hdim; i += 2) {
                    float freq = 1.0f / powf(m->theta, (float)i / (float)hdim);
                    float c = cosf((float)pos * freq), s = sinf((float)pos * freq);
                    float k0 = kk[i], k1 = kk[i + 1];
                    kk[i] = k0 * c - k1 * s;
                    kk[i + 1] = k0 * s + k1 * c;
                }
            }
        }

        /* causal attention with the self-exclusion rule, turbo.rs:144-185 */
        memset(attn, 0, T * hd * 4);
        for (size_t t = 0; t < T; t++) {
            for (size_t h = 0; h < nh; h++) {
                size_t kvh = (nkv < nh) ? h * nkv / nh : h;
                float* o = attn + t * hd + h * hdim;
                if (t < 2) {
                    memcpy(o, v + (t * nkv + kvh) * hdim, hdim * 4);
                } else {
                    const float* qq = q + (t * nh + h) * hdim;
                    for (size_t s = 0; s < t; s++) {
                        const float* kp = k + (s * nkv + kvh) * hdim;
                        float dot = 0.0f;
                        for (size_t d = 0; d < hdim; d++) dot += qq[d] * kp[d];
                        scores[s] = dot * scale;
                    }
                    orc_softmax(scores, t);
                    for (size_t d = 0; d < hdim; d++) {
                        float val = 0.0f;
                        for (size_t s = 0; s < t; s++) val += scores[s] * v[(s * nkv + kvh) * hdim + d];
                        o[d] = val;
                    }
                }
            }
        }

        if (get_w(m, prefix, "self_attn.o_proj.weight", &p, &l, &dt) == 0) batch_matmul(ob, p, l, dt, attn, hd, hd, T);
        else memcpy(ob, attn, T * hd * 4);
        memcpy(residual, hidden, T * hd * 4);
        for (size_t i = 0; i < T * hd; i++) hidden[i] = residual[i] + ob[i];

        for (size_t t = 0; t < T; t++) kv_store_at(kv, li, k + t * nkv * hdim, v + t * nkv * hdim, cache_pos + t);

        snprintf(nm, sizeof nm, "%spost_attention_layernorm.weight", prefix);
        load_norm(m, nm, hd, nw);
        for (size_t t = 0; t < T; t++) {
            memcpy(normed + t * hd, hidden + t * hd, hd * 4);
            orc_rms_norm(normed + t * hd, nw, hd, m->eps);
        }
        if (get_w(m, prefix, "mlp.gate_proj.weight", &p, &l, &dt) == 0) batch_matmul(g, p, l, dt, normed, im, hd, T);
        if (get_w(m, prefix, "mlp.up_proj.weight", &p, &l, &dt) == 0) batch_matmul(u, p, l, dt, normed, im, hd, T);
        for (size_t i = 0; i < T * im; i++) g[i] = silu1(g[i]) * u[i];
        if (get_w(m, prefix, "mlp.down_proj.weight", &p, &l, &dt) == 0) batch_matmul(dn, p, l, dt, g, hd, im, T);
        memcpy(residual, hidden, T * hd * 4);
        for (size_t i = 0; i < T * hd; i++) hidden[i] = residual[i] + dn[i];
    }
    kv->pos = cache_pos + T; /* set_pos, turbo.rs:253 */

    float* last = hidden + (T - 1) * hd;
    load_norm(m, "model.norm.weight", hd, nw);
    orc_rms_norm(last, nw, hd, m->eps);
    lm_head(m, last, logits);

    free(hidden); free(residual); free(normed); free(q); free(k); free(v); free(attn);
    free(g); free(u); free(dn); free(ob); free(scores); free(nw);
    return 0;
}

ORC_API int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

ORC_API void orc_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ------------------------------------------------------------------ */
/* Seeded synthetic inputs (test harness, not a reference algorithm)   */
/* ------------------------------------------------------------------ */

/* The benchmark's synthetic weights and activations: element offset+i of the
 * seeded stream (key from seed and stream id) is a 12-term Irwin-Hall sum of
 * 16-bit uniforms taken from three SplitMix64 hashes, centred and scaled by
 * std/65536 with one IEEE multiply, so the CPU reference arm builds the same
 * model bytes as the GPU side without loading the GPU library. */
static inline uint64_t orc_splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

ORC_API void orc_synth_normal(uint64_t seed, uint64_t stream, uint64_t offset, uint64_t n, float std, float* out) {
    const uint64_t key = orc_splitmix64(seed * 0x100000001B3ull ^ orc_splitmix64(stream + 0x51ED270B2ull));
    const float scale = std / 65536.0f;
    #pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; i++) {
        const uint64_t idx = offset + (uint64_t)i;
        uint32_t s = 0;
        for (int j = 0; j < 3; j++) {
            const uint64_t h = orc_splitmix64(key + 3ull * idx + (uint64_t)j);
            s += (uint32_t)(h & 0xFFFF) + (uint32_t)((h >> 16) & 0xFFFF) + (uint32_t)((h >> 32) & 0xFFFF) +
                 (uint32_t)(h >> 48);
        }
        const int32_t z = (int32_t)s - 393210;
        out[i] = (float)z * scale;
    }
}

/* ------------------------------------------------------------------ */
/* Sampling — run.rs:203-278                                           */
/* ------------------------------------------------------------------ */

/* XorShift64::next / next_f32, run.rs:267-278 (seed.max(1) at creation). */
ORC_API uint64_t orc_xorshift_next(uint64_t* state) {
    uint64_t x = *state;
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    *state = x;
    return x;
}

ORC_API float orc_xorshift_next_f32(uint64_t* state) { return (float)(orc_xorshift_next(state) >> 40) / 16777216.0f; }

typedef struct { size_t i; float v; } orc_iv;

/* sort_unstable_by(|a, b| b.1.partial_cmp(&a.1).unwrap_or(Equal)): descending;
 * NaN compares Equal (its position is unspecified in the reference). */
static int orc_cmp_desc(const void* a, const void* b) {
    float x = ((const orc_iv*)a)->v, y = ((const orc_iv*)b)->v;
    if (y > x) return 1;
    if (y < x) return -1;
    return 0;
}

/* Iterator::max_by with partial_cmp().unwrap_or(Equal): the last maximal
 * element; an incomparable pair counts as Equal, so the later one wins. */
static uint32_t orc_max_by_last(const float* v, size_t n) {
    if (n == 0) return 0;
    size_t bi = 0;
    float best = v[0];
    for (size_t i = 1; i < n; i++) {
        float x = v[i];
        int less = x < best;  /* partial_cmp(best, x) == Greater keeps best */
        if (!less) { best = x; bi = i; }
    }
    return (uint32_t)bi;
}

/* sample_token, run.rs:203-251, step by step in f32 (sequential sums in index
 * order, libm expf). */
ORC_API uint32_t orc_sample_token(const float* logits, size_t n, float temperature, float top_p, size_t top_k,
                                  uint64_t* rng_state) {
    float* probs = (float*)malloc(n * sizeof(float));
    orc_iv* idx = (orc_iv*)malloc((n ? n : 1) * sizeof(orc_iv));
    memcpy(probs, logits, n * sizeof(float));
    if (temperature > 0.0f) {
        float inv_temp = 1.0f / temperature;
        for (size_t i = 0; i < n; i++) probs[i] = expf(probs[i] * inv_temp);
    }
    if (top_k > 0 && top_k < n) {
        for (size_t i = 0; i < n; i++) { idx[i].i = i; idx[i].v = probs[i]; }
        qsort(idx, n, sizeof(orc_iv), orc_cmp_desc);
        float threshold = idx[top_k - 1].v;
        for (size_t i = 0; i < n; i++) if (probs[i] < threshold) probs[i] = 0.0f;
    }
    if (top_p < 1.0f) {
        for (size_t i = 0; i < n; i++) { idx[i].i = i; idx[i].v = probs[i]; }
        qsort(idx, n, sizeof(orc_iv), orc_cmp_desc);
        float sum = 0.0f;
        for (size_t i = 0; i < n; i++) sum += probs[i];
        if (sum > 0.0f) {
            float cumsum = 0.0f, threshold = 3.40282347e38f; /* f32::MAX */
            for (size_t i = 0; i < n; i++) {
                cumsum += idx[i].v / sum;
                if (cumsum > top_p) { threshold = idx[i].v; break; }
            }
            for (size_t i = 0; i < n; i++) if (probs[i] < threshold) probs[i] = 0.0f;
        }
    }
    float sum = 0.0f;
    for (size_t i = 0; i < n; i++) sum += probs[i];
    uint32_t out;
    if (sum <= 0.0f) {
        out = orc_max_by_last(logits, n);
    } else {
        float r = orc_xorshift_next_f32(rng_state);
        float cumsum = 0.0f;
        out = UINT32_MAX;
        for (size_t i = 0; i < n; i++) {
            cumsum += probs[i] / sum;
            if (r < cumsum) { out = (uint32_t)i; break; }
        }
        if (out == UINT32_MAX) out = orc_max_by_last(probs, n);
    }
    free(probs);
    free(idx);
    return out;
}
