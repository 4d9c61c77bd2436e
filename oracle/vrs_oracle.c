/*
 * vrs_oracle.c -- TEST INFRASTRUCTURE ONLY (parity checker and timed CPU
 * baseline). Nothing in the product links, loads or calls this file; only
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg do.
 *
 * A plain-C restatement of VectorRS's CPU paths for exact flat kNN and Lloyd
 * k-means, i.e. the paths the reference runs when no GPU is present:
 *
 *   - pair distances: crates/vector-simd/src/avx512.rs (the backend that
 *     DistanceEngine::auto() selects on an AVX-512 host,
 *     crates/vector-simd/src/lib.rs:292-310); semantics and guards from
 *     crates/vector-simd/src/scalar.rs:14-263.
 *   - batch flat search: CudaKnnEngine::search_batch_cpu,
 *     crates/vector-cuda/src/knn.rs:312-377 (bounded max-heap, strict `<`
 *     replacement, output best-first; similarity metrics negated,
 *     knn.rs:345-349).
 *   - shard merge: CollectiveOps::top_k_reduce,
 *     crates/vector-cuda/src/ddp/collective.rs:115-159.
 *   - Lloyd k-means: CudaKMeansEngine::fit_cpu + find_nearest,
 *     crates/vector-cuda/src/kmeans.rs:240-407.
 *
 * Every AVX-512 kernel exists twice: with intrinsics (fast; timed CPU
 * baseline) and as a 16-lane array emulation with the same operation order
 * (runs on any x86-64 host). Both give identical bits; a test checks it.
 *
 * Arithmetic-order facts restated from avx512.rs:
 *   - dot/L2: four 16-lane FMA accumulators over 64-wide chunks (:23-76,
 *     :87-148), a 16-wide tail into accumulator 0, (s0+s1)+(s2+s3), a
 *     halving-tree horizontal add, then a scalar tail with separate multiply
 *     and add (Rust never contracts a*b+c).
 *   - cosine: two accumulator sets over 32-wide chunks (:161-223).
 *   - L1: two add accumulators over 32-wide chunks (:234-280).
 *   - Minkowski p=3: two FMA accumulators over 32-wide chunks, no 16-wide
 *     tail, scalar remainder, cbrt (:300-340).
 *   - Chebyshev: one 16-lane max over 16-wide chunks (:354-390).
 *   - Hamming: per-16-chunk popcount of |d|>1e-6 (:401-433).
 *   - Jaccard: one min and one max accumulator over 16-wide chunks, separate
 *     remainder sum for min (:520-568).
 *   - Hellinger: one FMA accumulator of (sqrt|a|-sqrt|b|)^2 (:581-610).
 *   - _mm512_reduce_add_ps is the halving tree lanes i+8, i+4, i+2, i+1.
 *
 * Deliberate deviations (the GPU path makes the same ones):
 *   - k-means starts from caller-supplied centroids instead of the unseeded
 *     k-means++ (kmeans.rs:409-460), which cannot be reproduced;
 *   - an empty cluster keeps its centroid (as the reference GPU kernel,
 *     crates/vector-cuda/src/kernels/kmeans.cu:350-356) instead of a
 *     thread_rng reseed (kmeans.rs:334-339);
 *   - per-cluster sums and the inertia are accumulated in f64 in point
 *     order; the new centroid is (float)(sum / count);
 *   - the kNN heap orders by (score, id), so among exactly equal scores the
 *     lower id is kept and listed first (the reference's BinaryHeap leaves
 *     that order unspecified).
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off -pthread).
 */
#include <immintrin.h>
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

enum {
    M_L2 = 0, M_DOT = 1, M_COS = 2, M_L1 = 3, M_MINK = 4,
    M_CHEB = 5, M_HAM = 6, M_MAHA = 7, M_JAC = 8, M_HELL = 9
};

/* DistanceMetric::higher_is_better, crates/vector-index/src/lib.rs:85-94 */
int orc_higher_is_better(int metric) { return metric == M_DOT || metric == M_COS; }

/* ---------------------------------------------------------------------- */
/* 16-lane emulation (portable; bit-identical to the intrinsics below)     */
/* ---------------------------------------------------------------------- */

static float tree16(const float* v) {
    float t8[8], t4[4], t2[2];
    for (int i = 0; i < 8; i++) t8[i] = v[i] + v[i + 8];
    for (int i = 0; i < 4; i++) t4[i] = t8[i] + t8[i + 4];
    for (int i = 0; i < 2; i++) t2[i] = t4[i] + t4[i + 2];
    return t2[0] + t2[1];
}

static float tree16_max(const float* v) {
    float t8[8], t4[4], t2[2];
    for (int i = 0; i < 8; i++) t8[i] = v[i] > v[i + 8] ? v[i] : v[i + 8];
    for (int i = 0; i < 4; i++) t4[i] = t8[i] > t8[i + 4] ? t8[i] : t8[i + 4];
    for (int i = 0; i < 2; i++) t2[i] = t4[i] > t4[i + 2] ? t4[i] : t4[i + 2];
    return t2[0] > t2[1] ? t2[0] : t2[1];
}

static float emu_dot(const float* a, const float* b, int n) {
    float s0[16] = {0}, s1[16] = {0}, s2[16] = {0}, s3[16] = {0};
    int chunks = n / 64;
    for (int c = 0; c < chunks; c++) {
        int base = c * 64;
        for (int l = 0; l < 16; l++) {
            s0[l] = fmaf(a[base + l], b[base + l], s0[l]);
            s1[l] = fmaf(a[base + 16 + l], b[base + 16 + l], s1[l]);
            s2[l] = fmaf(a[base + 32 + l], b[base + 32 + l], s2[l]);
            s3[l] = fmaf(a[base + 48 + l], b[base + 48 + l], s3[l]);
        }
    }
    int i = chunks * 64;
    while (i + 16 <= n) {
        for (int l = 0; l < 16; l++) s0[l] = fmaf(a[i + l], b[i + l], s0[l]);
        i += 16;
    }
    for (int l = 0; l < 16; l++) {
        s0[l] = s0[l] + s1[l];
        s2[l] = s2[l] + s3[l];
        s0[l] = s0[l] + s2[l];
    }
    float r = tree16(s0);
    for (; i < n; i++) r += a[i] * b[i];
    return r;
}

static float emu_l2(const float* a, const float* b, int n) {
    float s0[16] = {0}, s1[16] = {0}, s2[16] = {0}, s3[16] = {0};
    int chunks = n / 64;
    for (int c = 0; c < chunks; c++) {
        int base = c * 64;
        for (int l = 0; l < 16; l++) {
            float d0 = a[base + l] - b[base + l];
            float d1 = a[base + 16 + l] - b[base + 16 + l];
            float d2 = a[base + 32 + l] - b[base + 32 + l];
            float d3 = a[base + 48 + l] - b[base + 48 + l];
            s0[l] = fmaf(d0, d0, s0[l]);
            s1[l] = fmaf(d1, d1, s1[l]);
            s2[l] = fmaf(d2, d2, s2[l]);
            s3[l] = fmaf(d3, d3, s3[l]);
        }
    }
    int i = chunks * 64;
    while (i + 16 <= n) {
        for (int l = 0; l < 16; l++) {
            float d = a[i + l] - b[i + l];
            s0[l] = fmaf(d, d, s0[l]);
        }
        i += 16;
    }
    for (int l = 0; l < 16; l++) {
        s0[l] = s0[l] + s1[l];
        s2[l] = s2[l] + s3[l];
        s0[l] = s0[l] + s2[l];
    }
    float r = tree16(s0);
    for (; i < n; i++) {
        float d = a[i] - b[i];
        r += d * d;
    }
    return r;
}

static float emu_cos(const float* a, const float* b, int n) {
    float d0[16] = {0}, d1[16] = {0}, a0[16] = {0}, a1[16] = {0}, b0[16] = {0}, b1[16] = {0};
    int chunks = n / 32;
    for (int c = 0; c < chunks; c++) {
        int base = c * 32;
        for (int l = 0; l < 16; l++) {
            float x0 = a[base + l], y0 = b[base + l];
            d0[l] = fmaf(x0, y0, d0[l]);
            a0[l] = fmaf(x0, x0, a0[l]);
            b0[l] = fmaf(y0, y0, b0[l]);
            float x1 = a[base + 16 + l], y1 = b[base + 16 + l];
            d1[l] = fmaf(x1, y1, d1[l]);
            a1[l] = fmaf(x1, x1, a1[l]);
            b1[l] = fmaf(y1, y1, b1[l]);
        }
    }
    int i = chunks * 32;
    while (i + 16 <= n) {
        for (int l = 0; l < 16; l++) {
            float x = a[i + l], y = b[i + l];
            d0[l] = fmaf(x, y, d0[l]);
            a0[l] = fmaf(x, x, a0[l]);
            b0[l] = fmaf(y, y, b0[l]);
        }
        i += 16;
    }
    for (int l = 0; l < 16; l++) {
        d0[l] = d0[l] + d1[l];
        a0[l] = a0[l] + a1[l];
        b0[l] = b0[l] + b1[l];
    }
    float dot = tree16(d0), na = tree16(a0), nb = tree16(b0);
    for (; i < n; i++) {
        dot += a[i] * b[i];
        na += a[i] * a[i];
        nb += b[i] * b[i];
    }
    float den = sqrtf(na) * sqrtf(nb);
    return den <= 1e-9f ? 0.0f : dot / den;
}

static float emu_l1(const float* a, const float* b, int n) {
    float s0[16] = {0}, s1[16] = {0};
    int chunks = n / 32;
    for (int c = 0; c < chunks; c++) {
        int base = c * 32;
        for (int l = 0; l < 16; l++) {
            s0[l] = s0[l] + fabsf(a[base + l] - b[base + l]);
            s1[l] = s1[l] + fabsf(a[base + 16 + l] - b[base + 16 + l]);
        }
    }
    int i = chunks * 32;
    while (i + 16 <= n) {
        for (int l = 0; l < 16; l++) s0[l] = s0[l] + fabsf(a[i + l] - b[i + l]);
        i += 16;
    }
    for (int l = 0; l < 16; l++) s0[l] = s0[l] + s1[l];
    float r = tree16(s0);
    for (; i < n; i++) r += fabsf(a[i] - b[i]);
    return r;
}

/* Minkowski p=3 before the cube root (the root is monotone). */
static float emu_mink3_sum(const float* a, const float* b, int n) {
    float s0[16] = {0}, s1[16] = {0};
    int chunks = n / 32;
    for (int c = 0; c < chunks; c++) {
        int base = c * 32;
        for (int l = 0; l < 16; l++) {
            float x0 = fabsf(a[base + l] - b[base + l]);
            float x1 = fabsf(a[base + 16 + l] - b[base + 16 + l]);
            float q0 = x0 * x0, q1 = x1 * x1;
            s0[l] = fmaf(q0, x0, s0[l]);
            s1[l] = fmaf(q1, x1, s1[l]);
        }
    }
    for (int l = 0; l < 16; l++) s0[l] = s0[l] + s1[l];
    float r = tree16(s0);
    for (int i = chunks * 32; i < n; i++) {
        float x = fabsf(a[i] - b[i]);
        r += x * x * x;
    }
    return r;
}

static float emu_cheb(const float* a, const float* b, int n) {
    if (n == 0) return 0.0f;
    float m[16] = {0};
    int chunks = n / 16;
    for (int c = 0; c < chunks; c++)
        for (int l = 0; l < 16; l++) {
            float x = fabsf(a[c * 16 + l] - b[c * 16 + l]);
            m[l] = m[l] > x ? m[l] : x; /* MAXPS returns the 2nd operand unless 1st > 2nd */
        }
    float r = tree16_max(m);
    for (int i = chunks * 16; i < n; i++) {
        float x = fabsf(a[i] - b[i]);
        if (x > r) r = x;
    }
    return r;
}

static float emu_ham(const float* a, const float* b, int n) {
    float count = 0.0f;
    int chunks = n / 16;
    for (int c = 0; c < chunks; c++) {
        int pc = 0;
        for (int l = 0; l < 16; l++) pc += fabsf(a[c * 16 + l] - b[c * 16 + l]) > 1e-6f;
        count += (float)pc;
    }
    for (int i = chunks * 16; i < n; i++)
        if (fabsf(a[i] - b[i]) > 1e-6f) count += 1.0f;
    return count;
}

static float emu_jac(const float* a, const float* b, int n) {
    float mn[16] = {0}, mx[16] = {0};
    int chunks = n / 16;
    for (int c = 0; c < chunks; c++)
        for (int l = 0; l < 16; l++) {
            float x = fabsf(a[c * 16 + l]), y = fabsf(b[c * 16 + l]);
            mn[l] = mn[l] + (x < y ? x : y);
            mx[l] = mx[l] + (x > y ? x : y);
        }
    float smin = tree16(mn), smax = tree16(mx), rem = 0.0f;
    for (int i = chunks * 16; i < n; i++) {
        float x = fabsf(a[i]), y = fabsf(b[i]);
        rem += (x < y ? x : y);
        smax += (x > y ? x : y);
    }
    float tmin = smin + rem;
    return smax <= 1e-9f ? 0.0f : 1.0f - tmin / smax;
}

/* Hellinger before the final sqrt(0.5*s) (monotone). */
static float emu_hell_sum(const float* a, const float* b, int n) {
    float s[16] = {0};
    int chunks = n / 16;
    for (int c = 0; c < chunks; c++)
        for (int l = 0; l < 16; l++) {
            float d = sqrtf(fabsf(a[c * 16 + l])) - sqrtf(fabsf(b[c * 16 + l]));
            s[l] = fmaf(d, d, s[l]);
        }
    float r = tree16(s);
    for (int i = chunks * 16; i < n; i++) {
        float d = sqrtf(fabsf(a[i])) - sqrtf(fabsf(b[i]));
        r += d * d;
    }
    return r;
}

/* ---------------------------------------------------------------------- */
/* AVX-512 intrinsics (same operation order as above)                      */
/* ---------------------------------------------------------------------- */
#define AVX512 __attribute__((target("avx512f")))

/* |x| by clearing the sign bit (the reference's and-with-0x7fffffff mask);
 * done on the integer view so only AVX-512F is required. */
AVX512 static inline __m512 vabs(__m512 x) {
    return _mm512_castsi512_ps(_mm512_and_si512(_mm512_castps_si512(x), _mm512_set1_epi32(0x7fffffff)));
}

AVX512 static inline float hsum(__m512 v) {
    __m256 lo = _mm512_castps512_ps256(v);
    __m256 hi = _mm256_castpd_ps(_mm512_extractf64x4_pd(_mm512_castps_pd(v), 1));
    __m256 t8 = _mm256_add_ps(lo, hi);
    __m128 t4 = _mm_add_ps(_mm256_castps256_ps128(t8), _mm256_extractf128_ps(t8, 1));
    __m128 t2 = _mm_add_ps(t4, _mm_shuffle_ps(t4, t4, _MM_SHUFFLE(1, 0, 3, 2)));
    return _mm_cvtss_f32(t2) + _mm_cvtss_f32(_mm_shuffle_ps(t2, t2, 1));
}

AVX512 static inline float hmax(__m512 v) {
    __m256 lo = _mm512_castps512_ps256(v);
    __m256 hi = _mm256_castpd_ps(_mm512_extractf64x4_pd(_mm512_castps_pd(v), 1));
    __m256 t8 = _mm256_max_ps(lo, hi);
    __m128 t4 = _mm_max_ps(_mm256_castps256_ps128(t8), _mm256_extractf128_ps(t8, 1));
    __m128 t2 = _mm_max_ps(t4, _mm_shuffle_ps(t4, t4, _MM_SHUFFLE(1, 0, 3, 2)));
    float x = _mm_cvtss_f32(t2), y = _mm_cvtss_f32(_mm_shuffle_ps(t2, t2, 1));
    return x > y ? x : y;
}

AVX512 static float v_dot(const float* a, const float* b, int n) {
    __m512 s0 = _mm512_setzero_ps(), s1 = s0, s2 = s0, s3 = s0;
    int chunks = n / 64;
    for (int c = 0; c < chunks; c++) {
        const float *pa = a + c * 64, *pb = b + c * 64;
        s0 = _mm512_fmadd_ps(_mm512_loadu_ps(pa), _mm512_loadu_ps(pb), s0);
        s1 = _mm512_fmadd_ps(_mm512_loadu_ps(pa + 16), _mm512_loadu_ps(pb + 16), s1);
        s2 = _mm512_fmadd_ps(_mm512_loadu_ps(pa + 32), _mm512_loadu_ps(pb + 32), s2);
        s3 = _mm512_fmadd_ps(_mm512_loadu_ps(pa + 48), _mm512_loadu_ps(pb + 48), s3);
    }
    int i = chunks * 64;
    for (; i + 16 <= n; i += 16) s0 = _mm512_fmadd_ps(_mm512_loadu_ps(a + i), _mm512_loadu_ps(b + i), s0);
    s0 = _mm512_add_ps(s0, s1);
    s2 = _mm512_add_ps(s2, s3);
    s0 = _mm512_add_ps(s0, s2);
    float r = hsum(s0);
    for (; i < n; i++) r += a[i] * b[i];
    return r;
}

AVX512 static float v_l2(const float* a, const float* b, int n) {
    __m512 s0 = _mm512_setzero_ps(), s1 = s0, s2 = s0, s3 = s0;
    int chunks = n / 64;
    for (int c = 0; c < chunks; c++) {
        const float *pa = a + c * 64, *pb = b + c * 64;
        __m512 d0 = _mm512_sub_ps(_mm512_loadu_ps(pa), _mm512_loadu_ps(pb));
        s0 = _mm512_fmadd_ps(d0, d0, s0);
        __m512 d1 = _mm512_sub_ps(_mm512_loadu_ps(pa + 16), _mm512_loadu_ps(pb + 16));
        s1 = _mm512_fmadd_ps(d1, d1, s1);
        __m512 d2 = _mm512_sub_ps(_mm512_loadu_ps(pa + 32), _mm512_loadu_ps(pb + 32));
        s2 = _mm512_fmadd_ps(d2, d2, s2);
        __m512 d3 = _mm512_sub_ps(_mm512_loadu_ps(pa + 48), _mm512_loadu_ps(pb + 48));
        s3 = _mm512_fmadd_ps(d3, d3, s3);
    }
    int i = chunks * 64;
    for (; i + 16 <= n; i += 16) {
        __m512 d = _mm512_sub_ps(_mm512_loadu_ps(a + i), _mm512_loadu_ps(b + i));
        s0 = _mm512_fmadd_ps(d, d, s0);
    }
    s0 = _mm512_add_ps(s0, s1);
    s2 = _mm512_add_ps(s2, s3);
    s0 = _mm512_add_ps(s0, s2);
    float r = hsum(s0);
    for (; i < n; i++) {
        float d = a[i] - b[i];
        r += d * d;
    }
    return r;
}

AVX512 static float v_cos(const float* a, const float* b, int n) {
    __m512 d0 = _mm512_setzero_ps(), d1 = d0, a0 = d0, a1 = d0, b0 = d0, b1 = d0;
    int chunks = n / 32;
    for (int c = 0; c < chunks; c++) {
        const float *pa = a + c * 32, *pb = b + c * 32;
        __m512 x0 = _mm512_loadu_ps(pa), y0 = _mm512_loadu_ps(pb);
        d0 = _mm512_fmadd_ps(x0, y0, d0);
        a0 = _mm512_fmadd_ps(x0, x0, a0);
        b0 = _mm512_fmadd_ps(y0, y0, b0);
        __m512 x1 = _mm512_loadu_ps(pa + 16), y1 = _mm512_loadu_ps(pb + 16);
        d1 = _mm512_fmadd_ps(x1, y1, d1);
        a1 = _mm512_fmadd_ps(x1, x1, a1);
        b1 = _mm512_fmadd_ps(y1, y1, b1);
    }
    int i = chunks * 32;
    for (; i + 16 <= n; i += 16) {
        __m512 x = _mm512_loadu_ps(a + i), y = _mm512_loadu_ps(b + i);
        d0 = _mm512_fmadd_ps(x, y, d0);
        a0 = _mm512_fmadd_ps(x, x, a0);
        b0 = _mm512_fmadd_ps(y, y, b0);
    }
    d0 = _mm512_add_ps(d0, d1);
    a0 = _mm512_add_ps(a0, a1);
    b0 = _mm512_add_ps(b0, b1);
    float dot = hsum(d0), na = hsum(a0), nb = hsum(b0);
    for (; i < n; i++) {
        dot += a[i] * b[i];
        na += a[i] * a[i];
        nb += b[i] * b[i];
    }
    float den = sqrtf(na) * sqrtf(nb);
    return den <= 1e-9f ? 0.0f : dot / den;
}

AVX512 static float v_l1(const float* a, const float* b, int n) {
    __m512 s0 = _mm512_setzero_ps(), s1 = s0;
    int chunks = n / 32;
    for (int c = 0; c < chunks; c++) {
        const float *pa = a + c * 32, *pb = b + c * 32;
        s0 = _mm512_add_ps(s0, vabs(_mm512_sub_ps(_mm512_loadu_ps(pa), _mm512_loadu_ps(pb))));
        s1 = _mm512_add_ps(s1, vabs(_mm512_sub_ps(_mm512_loadu_ps(pa + 16), _mm512_loadu_ps(pb + 16))));
    }
    int i = chunks * 32;
    for (; i + 16 <= n; i += 16)
        s0 = _mm512_add_ps(s0, vabs(_mm512_sub_ps(_mm512_loadu_ps(a + i), _mm512_loadu_ps(b + i))));
    s0 = _mm512_add_ps(s0, s1);
    float r = hsum(s0);
    for (; i < n; i++) r += fabsf(a[i] - b[i]);
    return r;
}

AVX512 static float v_mink3_sum(const float* a, const float* b, int n) {
    __m512 s0 = _mm512_setzero_ps(), s1 = s0;
    int chunks = n / 32;
    for (int c = 0; c < chunks; c++) {
        const float *pa = a + c * 32, *pb = b + c * 32;
        __m512 x0 = vabs(_mm512_sub_ps(_mm512_loadu_ps(pa), _mm512_loadu_ps(pb)));
        s0 = _mm512_fmadd_ps(_mm512_mul_ps(x0, x0), x0, s0);
        __m512 x1 = vabs(_mm512_sub_ps(_mm512_loadu_ps(pa + 16), _mm512_loadu_ps(pb + 16)));
        s1 = _mm512_fmadd_ps(_mm512_mul_ps(x1, x1), x1, s1);
    }
    s0 = _mm512_add_ps(s0, s1);
    float r = hsum(s0);
    for (int i = chunks * 32; i < n; i++) {
        float x = fabsf(a[i] - b[i]);
        r += x * x * x;
    }
    return r;
}

AVX512 static float v_cheb(const float* a, const float* b, int n) {
    if (n == 0) return 0.0f;
    __m512 m = _mm512_setzero_ps();
    int chunks = n / 16;
    for (int c = 0; c < chunks; c++)
        m = _mm512_max_ps(m, vabs(_mm512_sub_ps(_mm512_loadu_ps(a + c * 16), _mm512_loadu_ps(b + c * 16))));
    float r = hmax(m);
    for (int i = chunks * 16; i < n; i++) {
        float x = fabsf(a[i] - b[i]);
        if (x > r) r = x;
    }
    return r;
}

AVX512 static float v_ham(const float* a, const float* b, int n) {
    const __m512 eps = _mm512_set1_ps(1e-6f);
    float count = 0.0f;
    int chunks = n / 16;
    for (int c = 0; c < chunks; c++) {
        __m512 x = vabs(_mm512_sub_ps(_mm512_loadu_ps(a + c * 16), _mm512_loadu_ps(b + c * 16)));
        __mmask16 k = _mm512_cmp_ps_mask(x, eps, _CMP_GT_OQ);
        count += (float)__builtin_popcount((unsigned)k);
    }
    for (int i = chunks * 16; i < n; i++)
        if (fabsf(a[i] - b[i]) > 1e-6f) count += 1.0f;
    return count;
}

AVX512 static float v_jac(const float* a, const float* b, int n) {
    __m512 mn = _mm512_setzero_ps(), mx = mn;
    int chunks = n / 16;
    for (int c = 0; c < chunks; c++) {
        __m512 x = vabs(_mm512_loadu_ps(a + c * 16));
        __m512 y = vabs(_mm512_loadu_ps(b + c * 16));
        mn = _mm512_add_ps(mn, _mm512_min_ps(x, y));
        mx = _mm512_add_ps(mx, _mm512_max_ps(x, y));
    }
    float smin = hsum(mn), smax = hsum(mx), rem = 0.0f;
    for (int i = chunks * 16; i < n; i++) {
        float x = fabsf(a[i]), y = fabsf(b[i]);
        rem += (x < y ? x : y);
        smax += (x > y ? x : y);
    }
    float tmin = smin + rem;
    return smax <= 1e-9f ? 0.0f : 1.0f - tmin / smax;
}

AVX512 static float v_hell_sum(const float* a, const float* b, int n) {
    __m512 s = _mm512_setzero_ps();
    int chunks = n / 16;
    for (int c = 0; c < chunks; c++) {
        __m512 x = _mm512_sqrt_ps(vabs(_mm512_loadu_ps(a + c * 16)));
        __m512 y = _mm512_sqrt_ps(vabs(_mm512_loadu_ps(b + c * 16)));
        __m512 d = _mm512_sub_ps(x, y);
        s = _mm512_fmadd_ps(d, d, s);
    }
    float r = hsum(s);
    for (int i = chunks * 16; i < n; i++) {
        float d = sqrtf(fabsf(a[i])) - sqrtf(fabsf(b[i]));
        r += d * d;
    }
    return r;
}

/* ---------------------------------------------------------------------- */
/* Dispatch                                                               */
/* ---------------------------------------------------------------------- */

int orc_has_avx512(void) { return __builtin_cpu_supports("avx512f") ? 1 : 0; }

/* "Rank key": the value whose order equals the metric's order before the
 * final monotone map (cube root for Minkowski, sqrt(0.5*s) for Hellinger,
 * sqrt for Mahalanobis), so ranking never depends on libm's cbrtf. */
static float rank_key(int metric, const float* a, const float* b, int n, int simd) {
    switch (metric) {
    case M_L2: case M_MAHA: return simd ? v_l2(a, b, n) : emu_l2(a, b, n);
    case M_DOT: return simd ? v_dot(a, b, n) : emu_dot(a, b, n);
    case M_COS: return simd ? v_cos(a, b, n) : emu_cos(a, b, n);
    case M_L1: return simd ? v_l1(a, b, n) : emu_l1(a, b, n);
    case M_MINK: return simd ? v_mink3_sum(a, b, n) : emu_mink3_sum(a, b, n);
    case M_CHEB: return simd ? v_cheb(a, b, n) : emu_cheb(a, b, n);
    case M_HAM: return simd ? v_ham(a, b, n) : emu_ham(a, b, n);
    case M_JAC: return simd ? v_jac(a, b, n) : emu_jac(a, b, n);
    case M_HELL: return simd ? v_hell_sum(a, b, n) : emu_hell_sum(a, b, n);
    }
    return NAN;
}

/* Final value reported as the distance, from the rank key. Rust's
 * f32::cbrt is glibc cbrtf (crates/vector-simd/src/avx512.rs:338). */
static float finish(int metric, float key) {
    switch (metric) {
    case M_MINK: return cbrtf(key);
    case M_MAHA: return sqrtf(key);
    case M_HELL: return sqrtf(0.5f * key);
    default: return key;
    }
}

static int pick_simd(int use_simd) {
    if (use_simd < 0) return orc_has_avx512();
    return use_simd && orc_has_avx512();
}

/* Reference distance for one pair; use_simd: 1 intrinsics, 0 emulation, -1 auto. */
float orc_distance(int metric, const float* a, const float* b, int n, int use_simd) {
    return finish(metric, rank_key(metric, a, b, n, pick_simd(use_simd)));
}

float orc_rank_key(int metric, const float* a, const float* b, int n, int use_simd) {
    return rank_key(metric, a, b, n, pick_simd(use_simd));
}

/* ---------------------------------------------------------------------- */
/* Batch flat kNN: CudaKnnEngine::search_batch_cpu (knn.rs:312-377)        */
/* ---------------------------------------------------------------------- */

typedef struct { float hs; float dist; uint32_t id; } cand_t;

static int cand_less(const cand_t* x, const cand_t* y) {
    return x->hs < y->hs || (x->hs == y->hs && x->id < y->id);
}

static void sift_down(cand_t* h, int n, int i) {
    for (;;) {
        int l = 2 * i + 1, r = l + 1, m = i;
        if (l < n && cand_less(&h[m], &h[l])) m = l;
        if (r < n && cand_less(&h[m], &h[r])) m = r;
        if (m == i) return;
        cand_t t = h[i]; h[i] = h[m]; h[m] = t;
        i = m;
    }
}

static void sift_up(cand_t* h, int i) {
    while (i > 0) {
        int p = (i - 1) / 2;
        if (!cand_less(&h[p], &h[i])) return;
        cand_t t = h[i]; h[i] = h[p]; h[p] = t;
        i = p;
    }
}

static int cmp_cand(const void* x, const void* y) {
    const cand_t *a = x, *b = y;
    if (cand_less(a, b)) return -1;
    if (cand_less(b, a)) return 1;
    return 0;
}

typedef struct {
    const float* base; int64_t n; int d;
    const float* q; int64_t q0, q1;
    int k; int metric; int simd;
    float* out_dist; uint32_t* out_id;
} knn_job_t;

static void* knn_worker(void* arg) {
    knn_job_t* j = arg;
    int hib = orc_higher_is_better(j->metric);
    cand_t* heap = malloc(sizeof(cand_t) * (size_t)(j->k + 1));
    for (int64_t qi = j->q0; qi < j->q1; qi++) {
        const float* qv = j->q + qi * j->d;
        int hn = 0;
        for (int64_t x = 0; x < j->n; x++) {
            float key = rank_key(j->metric, qv, j->base + x * j->d, j->d, j->simd);
            cand_t c = { hib ? -key : key, 0.0f, (uint32_t)x };
            if (hn < j->k) {
                c.dist = finish(j->metric, key);
                heap[hn++] = c;
                sift_up(heap, hn - 1);
            } else if (c.hs < heap[0].hs) {
                c.dist = finish(j->metric, key);
                heap[0] = c;
                sift_down(heap, hn, 0);
            }
        }
        qsort(heap, hn, sizeof(cand_t), cmp_cand);
        for (int r = 0; r < hn; r++) {
            j->out_dist[qi * j->k + r] = heap[r].dist;
            j->out_id[qi * j->k + r] = heap[r].id;
        }
    }
    free(heap);
    return NULL;
}

/* out_dist/out_id: nq x k' (k' = min(k, n), written to *out_k), best first. */
int orc_knn_search(const float* base, int64_t n, int d, const float* q, int64_t nq,
                   int k, int metric, int nthreads, int use_simd,
                   float* out_dist, uint32_t* out_id, int* out_k) {
    int kk = (int)(k < n ? k : n);
    if (kk < 0) kk = 0;
    *out_k = kk;
    if (nq <= 0 || kk == 0) return 0;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > nq) nthreads = (int)nq;
    int simd = pick_simd(use_simd);
    pthread_t th[256];
    knn_job_t jobs[256];
    if (nthreads > 256) nthreads = 256;
    int64_t per = (nq + nthreads - 1) / nthreads;
    int started = 0;
    for (int t = 0; t < nthreads; t++) {
        int64_t q0 = t * per, q1 = q0 + per < nq ? q0 + per : nq;
        if (q0 >= q1) break;
        jobs[t] = (knn_job_t){ base, n, d, q, q0, q1, kk, metric, simd, out_dist, out_id };
        pthread_create(&th[t], NULL, knn_worker, &jobs[t]);
        started++;
    }
    for (int t = 0; t < started; t++) pthread_join(th[t], NULL);
    return 0;
}

/* The same search for a few queries over many rows: threads split the ROWS
 * (each keeps k' per query over its row range, reading every row once for
 * all queries), then the per-thread lists are merged per query in
 * (heap score, id) order. The sequential heap above keeps exactly the k'
 * smallest (heap score, id) pairs -- a later row with an equal score has a
 * larger id and never displaces the root -- so the merged result is the
 * same. Ids are row index + id_offset (for a base fed in chunks). */
typedef struct {
    const float* base; int64_t r0, r1; int d;
    const float* q; int nq; int k; int metric; int simd; uint32_t id_offset;
    cand_t* heaps; int* counts;
} knn_rows_job_t;

static void* knn_rows_worker(void* arg) {
    knn_rows_job_t* j = arg;
    int hib = orc_higher_is_better(j->metric);
    for (int64_t x = j->r0; x < j->r1; x++) {
        const float* xv = j->base + x * j->d;
        for (int qi = 0; qi < j->nq; qi++) {
            cand_t* heap = j->heaps + (size_t)qi * j->k;
            int hn = j->counts[qi];
            float key = rank_key(j->metric, j->q + (int64_t)qi * j->d, xv, j->d, j->simd);
            cand_t c = { hib ? -key : key, 0.0f, (uint32_t)x + j->id_offset };
            if (hn < j->k) {
                c.dist = finish(j->metric, key);
                heap[hn++] = c;
                sift_up(heap, hn - 1);
                j->counts[qi] = hn;
            } else if (cand_less(&c, &heap[0])) {
                c.dist = finish(j->metric, key);
                heap[0] = c;
                sift_down(heap, hn, 0);
            }
        }
    }
    return NULL;
}

int orc_knn_search_rows(const float* base, int64_t n, int d, const float* q, int nq, int k, int metric,
                        int nthreads, int use_simd, uint32_t id_offset, float* out_dist, uint32_t* out_id,
                        int* out_k) {
    int kk = (int)(k < n ? k : n);
    if (kk < 0) kk = 0;
    *out_k = kk;
    if (nq <= 0 || kk == 0) return 0;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if (n < (int64_t)nthreads * 64) nthreads = 1;
    int simd = pick_simd(use_simd);
    cand_t* heaps = malloc(sizeof(cand_t) * (size_t)nthreads * nq * kk);
    int* counts = calloc((size_t)nthreads * nq, sizeof(int));
    pthread_t th[256];
    knn_rows_job_t jobs[256];
    int64_t per = (n + nthreads - 1) / nthreads;
    int started = 0;
    for (int t = 0; t < nthreads; t++) {
        int64_t r0 = t * per, r1 = r0 + per < n ? r0 + per : n;
        jobs[t] = (knn_rows_job_t){ base, r0 < n ? r0 : n, r1 > r0 ? r1 : r0, d, q, nq, kk, metric, simd,
                                    id_offset, heaps + (size_t)t * nq * kk, counts + (size_t)t * nq };
        pthread_create(&th[t], NULL, knn_rows_worker, &jobs[t]);
        started++;
    }
    for (int t = 0; t < started; t++) pthread_join(th[t], NULL);
    cand_t* all = malloc(sizeof(cand_t) * (size_t)nthreads * kk);
    for (int qi = 0; qi < nq; qi++) {
        int m = 0;
        for (int t = 0; t < started; t++) {
            const cand_t* h = heaps + ((size_t)t * nq + qi) * kk;
            int c = counts[(size_t)t * nq + qi];
            memcpy(all + m, h, sizeof(cand_t) * (size_t)c);
            m += c;
        }
        qsort(all, m, sizeof(cand_t), cmp_cand);
        for (int r = 0; r < kk && r < m; r++) {
            out_dist[(int64_t)qi * kk + r] = all[r].dist;
            out_id[(int64_t)qi * kk + r] = all[r].id;
        }
    }
    free(all);
    free(heaps);
    free(counts);
    return 0;
}

/* CollectiveOps::top_k_reduce (collective.rs:115-159): lists concatenated in
 * rank order, same strict heap rule, output best-first. lens[r] entries per
 * list; returns the merged count. */
int orc_topk_reduce(const float* dists, const uint32_t* ids, const int* lens, int nlists,
                    int k, int metric, float* out_dist, uint32_t* out_id) {
    if (nlists <= 0 || k <= 0) return 0;
    int hib = orc_higher_is_better(metric);
    cand_t* heap = malloc(sizeof(cand_t) * (size_t)(k + 1));
    int hn = 0, off = 0;
    for (int r = 0; r < nlists; r++) {
        for (int i = 0; i < lens[r]; i++) {
            float dist = dists[off + i];
            cand_t c = { hib ? -dist : dist, dist, ids[off + i] };
            if (hn < k) { heap[hn++] = c; sift_up(heap, hn - 1); }
            else if (c.hs < heap[0].hs) { heap[0] = c; sift_down(heap, hn, 0); }
        }
        off += lens[r];
    }
    qsort(heap, hn, sizeof(cand_t), cmp_cand);
    for (int i = 0; i < hn; i++) { out_dist[i] = heap[i].dist; out_id[i] = heap[i].id; }
    free(heap);
    return hn;
}

/* ---------------------------------------------------------------------- */
/* Lloyd k-means: CudaKMeansEngine::fit_cpu (kmeans.rs:240-357)            */
/* ---------------------------------------------------------------------- */

typedef struct {
    const float* x; int64_t i0, i1; int d; int k; int metric; int simd;
    const float* cent; int32_t* assign; float* dist;
} assign_job_t;

/* find_nearest, kmeans.rs:361-407: strict comparison, lowest index wins. */
static void* assign_worker(void* arg) {
    assign_job_t* j = arg;
    int hib = orc_higher_is_better(j->metric);
    for (int64_t i = j->i0; i < j->i1; i++) {
        const float* v = j->x + i * j->d;
        int best = 0;
        float best_key = hib ? -INFINITY : INFINITY;
        for (int c = 0; c < j->k; c++) {
            float key = rank_key(j->metric, v, j->cent + (int64_t)c * j->d, j->d, j->simd);
            if (hib ? key > best_key : key < best_key) { best_key = key; best = c; }
        }
        j->assign[i] = best;
        j->dist[i] = finish(j->metric, best_key);
    }
    return NULL;
}

static void assign_all(const float* x, int64_t n, int d, int k, int metric, int simd,
                       int nthreads, const float* cent, int32_t* assign, float* dist) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    pthread_t th[256];
    assign_job_t jobs[256];
    int64_t per = (n + nthreads - 1) / nthreads;
    int started = 0;
    for (int t = 0; t < nthreads; t++) {
        int64_t i0 = t * per, i1 = i0 + per < n ? i0 + per : n;
        if (i0 >= i1) break;
        jobs[t] = (assign_job_t){ x, i0, i1, d, k, metric, simd, cent, assign, dist };
        pthread_create(&th[t], NULL, assign_worker, &jobs[t]);
        started++;
    }
    for (int t = 0; t < started; t++) pthread_join(th[t], NULL);
}

/* One rank's share of a Lloyd iteration: assign the rank's rows to their
 * nearest centroid, then per-cluster f64 sums of the rows (row order),
 * counts and the summed distances (distributed_kmeans.rs:377-409, with f64
 * sums in place of the reference's f32 ones). The sums of all ranks are
 * added by an all-reduce before orc_kmeans_update. */
void orc_kmeans_local(const float* x, int64_t n, int d, int kk, const float* cent, int metric,
                      int nthreads, int use_simd, int32_t* out_assign, double* out_sums,
                      int64_t* out_counts, double* out_inertia) {
    int simd = pick_simd(use_simd);
    float* dist = malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
    memset(out_sums, 0, sizeof(double) * (size_t)kk * d);
    memset(out_counts, 0, sizeof(int64_t) * (size_t)kk);
    double inertia = 0.0;
    if (n > 0) assign_all(x, n, d, kk, metric, simd, nthreads, cent, out_assign, dist);
    for (int64_t i = 0; i < n; i++) {
        int c = out_assign[i];
        out_counts[c]++;
        const float* v = x + i * d;
        double* s = out_sums + (int64_t)c * d;
        for (int e = 0; e < d; e++) s[e] += (double)v[e];
        inertia += (double)dist[i];
    }
    *out_inertia = inertia;
    free(dist);
}

/* Centroid update from the global sums and counts: mean = (float)(sum /
 * count), squared shift accumulated in f32 per cluster, the largest shift
 * returned; an empty cluster keeps its centroid (distributed_kmeans.rs:433-461
 * reseeds it from a random row instead). */
float orc_kmeans_update(const double* sums, const int64_t* counts, int kk, int d, float* cent) {
    float max_shift = 0.0f;
    for (int c = 0; c < kk; c++) {
        if (counts[c] == 0) continue;
        float shift = 0.0f;
        for (int e = 0; e < d; e++) {
            float val = (float)(sums[(int64_t)c * d + e] / (double)counts[c]);
            float diff = val - cent[(int64_t)c * d + e];
            shift += diff * diff;
            cent[(int64_t)c * d + e] = val;
        }
        if (shift > max_shift) max_shift = shift;
    }
    return max_shift;
}

/* Returns the effective k (min(k, n); 0 when n == 0 or k == 0).
 * init: k_eff x d initial centroids (required). out_assign may be NULL.
 * out_inertia: f64 sum, in point order, of the last assignment step's
 * per-point metric values (kmeans.rs:293-297). */
int orc_kmeans_fit(const float* x, int64_t n, int d, int k, const float* init,
                   int max_iters, float tol, int metric, int nthreads, int use_simd,
                   float* out_centroids, int32_t* out_assign, int* out_iters,
                   double* out_inertia) {
    *out_iters = 0;
    *out_inertia = 0.0;
    if (n <= 0 || k <= 0) return 0;
    int kk = (int)(k < n ? k : n);
    float* cent = malloc(sizeof(float) * (size_t)kk * d);
    memcpy(cent, init, sizeof(float) * (size_t)kk * d);
    int32_t* assign = malloc(sizeof(int32_t) * (size_t)n);
    double* sums = malloc(sizeof(double) * (size_t)kk * d);
    int64_t* counts = malloc(sizeof(int64_t) * (size_t)kk);
    double inertia = 0.0;
    int iters = 0;
    for (int it = 0; it < max_iters; it++) {
        iters = it + 1;
        orc_kmeans_local(x, n, d, kk, cent, metric, nthreads, use_simd, assign, sums, counts,
                         &inertia);
        if (orc_kmeans_update(sums, counts, kk, d, cent) <= tol) break;
    }
    memcpy(out_centroids, cent, sizeof(float) * (size_t)kk * d);
    if (out_assign) memcpy(out_assign, assign, sizeof(int32_t) * (size_t)n);
    *out_iters = iters;
    *out_inertia = inertia;
    free(cent); free(assign); free(sums); free(counts);
    return kk;
}

/* ---------------------------------------------------------------------- */
/* IVF-PQ ADC search on a trained index: IvfPqIndex::search               */
/* (crates/vector-index/src/ivf/mod.rs:265-345) with ProductQuantizer's    */
/* compute_adc_lut and compute_distance_with_lut (ivf/pq.rs:233-296). The  */
/* k best candidates live in a restatement of std's BinaryHeap compared on */
/* the heap score alone (mod.rs:28-54): push = append + sift_up; pop =     */
/* last element into the root, sift_down_to_bottom (towards the larger     */
/* child, the right one when left <= right), then sift_up. Inverted list c */
/* holds entries [list_off[c], list_off[c+1]) of ids and M-byte codes.     */
/* Finite scores assumed (the reference's comparator maps NaN to Equal).   */
/* ---------------------------------------------------------------------- */

typedef struct { float hs; float dist; uint32_t id; } pq_cand_t;
typedef struct { float v; int idx; int desc; } pq_rank_t;

static int pq_le(float a, float b) { return !(a > b); } /* partial_cmp != Greater */

static void pq_sift_up(pq_cand_t* h, int start, int pos) {
    pq_cand_t e = h[pos];
    while (pos > start) {
        int parent = (pos - 1) / 2;
        if (pq_le(e.hs, h[parent].hs)) break;
        h[pos] = h[parent];
        pos = parent;
    }
    h[pos] = e;
}

static void pq_sift_down_to_bottom(pq_cand_t* h, int end, int pos) {
    const int start = pos;
    pq_cand_t e = h[pos];
    int child = 2 * pos + 1;
    while (child <= end - 2) {
        if (pq_le(h[child].hs, h[child + 1].hs)) child++;
        h[pos] = h[child];
        pos = child;
        child = 2 * pos + 1;
    }
    if (child == end - 1) {
        h[pos] = h[child];
        pos = child;
    }
    h[pos] = e;
    pq_sift_up(h, start, pos);
}

/* Stable order of find_top_centroids (kmeans.rs:345-350): by value (descending
 * for similarities), equal values by index. */
static int pq_rank_cmp(const void* pa, const void* pb) {
    const pq_rank_t* a = (const pq_rank_t*)pa;
    const pq_rank_t* b = (const pq_rank_t*)pb;
    float x = a->desc ? b->v : a->v, y = a->desc ? a->v : b->v;
    if (x < y) return -1;
    if (x > y) return 1;
    return (a->idx > b->idx) - (a->idx < b->idx);
}

int orc_ivfpq_search(const float* q, int d, int k, int nprobe, const float* coarse, int nlist,
                     const int64_t* list_off, const uint32_t* ids, const uint8_t* codes,
                     const float* codebooks, int M, int ksub, int metric, int use_simd,
                     float* out_dist, uint32_t* out_id) {
    if (k <= 0 || nlist <= 0) return 0;
    const int simd = pick_simd(use_simd);
    const int hib = orc_higher_is_better(metric);
    const int ds = d / M;
    int eff = nprobe < nlist ? nprobe : nlist;
    if (eff < 1) eff = 1;
    pq_rank_t* rk = (pq_rank_t*)malloc(sizeof(pq_rank_t) * (size_t)nlist);
    for (int c = 0; c < nlist; c++) {
        rk[c].v = finish(metric, rank_key(metric, q, coarse + (size_t)c * d, d, simd));
        rk[c].idx = c;
        rk[c].desc = hib;
    }
    qsort(rk, (size_t)nlist, sizeof(pq_rank_t), pq_rank_cmp);
    float* resid = (float*)malloc(sizeof(float) * (size_t)d);
    float* lut = (float*)malloc(sizeof(float) * (size_t)M * ksub);
    pq_cand_t* heap = (pq_cand_t*)malloc(sizeof(pq_cand_t) * ((size_t)k + 1));
    int hn = 0;
    for (int t = 0; t < eff; t++) {
        const int c = rk[t].idx;
        const int64_t b = list_off[c], e = list_off[c + 1];
        if (e <= b) continue;
        for (int j = 0; j < d; j++) resid[j] = q[j] - coarse[(size_t)c * d + j];
        for (int m = 0; m < M; m++)
            for (int s = 0; s < ksub; s++)
                lut[m * ksub + s] = finish(metric, rank_key(metric, resid + m * ds,
                                                            codebooks + ((size_t)m * ksub + s) * ds, ds, simd));
        for (int64_t i = b; i < e; i++) {
            const uint8_t* code = codes + (size_t)i * M;
            float total = 0.0f;
            int m = 0;
            for (; m + 4 <= M; m += 4) {
                const float d0 = lut[m * ksub + code[m]], d1 = lut[(m + 1) * ksub + code[m + 1]];
                const float d2 = lut[(m + 2) * ksub + code[m + 2]], d3 = lut[(m + 3) * ksub + code[m + 3]];
                total = total + ((d0 + d1) + (d2 + d3));
            }
            for (; m < M; m++) total = total + lut[m * ksub + code[m]];
            const float hs = hib ? -total : total;
            pq_cand_t cand = {hs, total, ids[i]};
            if (hn < k) {
                heap[hn] = cand;
                pq_sift_up(heap, 0, hn);
                hn++;
            } else if (hs < heap[0].hs) {
                /* pop the worst, then push */
                pq_cand_t last = heap[--hn];
                if (hn > 0) {
                    heap[0] = last;
                    pq_sift_down_to_bottom(heap, hn, 0);
                }
                heap[hn] = cand;
                pq_sift_up(heap, 0, hn);
                hn++;
            }
        }
    }
    /* pop worst to best, written back to front: best first */
    const int count = hn;
    while (hn > 0) {
        pq_cand_t top = heap[0];
        pq_cand_t last = heap[--hn];
        if (hn > 0) {
            heap[0] = last;
            pq_sift_down_to_bottom(heap, hn, 0);
        }
        out_dist[hn] = top.dist;
        out_id[hn] = top.id;
    }
    free(rk); free(resid); free(lut); free(heap);
    return count;
}
