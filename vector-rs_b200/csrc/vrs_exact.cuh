// vrs_exact.cuh -- per-pair distances in the exact arithmetic order of
// VectorRS's AVX-512 CPU kernels (crates/vector-simd/src/avx512.rs), usable
// on host and device. The GPU uses these to re-rank candidates, so the final
// distances are bit-identical to the reference's CPU path:
//   * 16 "SIMD lanes" are 16-element register arrays;
//   * _mm512_fmadd_ps is one fused multiply-add (VRS_FMA);
//   * _mm512_reduce_add_ps is the halving tree i+8, i+4, i+2, i+1;
//   * scalar tails multiply and add separately, as Rust does not contract.
// Device code uses the _rn intrinsics so nvcc cannot contract or reorder;
// host code is compiled with -ffp-contract=off.
#pragma once
#include <math.h>
#include <stdint.h>

#if defined(__CUDACC__)
#define VX_HD __host__ __device__ __forceinline__
#else
#define VX_HD inline
#endif

#if defined(__CUDA_ARCH__)
#define VX_ADD(a, b) __fadd_rn((a), (b))
#define VX_SUB(a, b) __fsub_rn((a), (b))
#define VX_MUL(a, b) __fmul_rn((a), (b))
#define VX_FMA(a, b, c) __fmaf_rn((a), (b), (c))
#define VX_DIV(a, b) __fdiv_rn((a), (b))
#define VX_SQRT(a) __fsqrt_rn(a)
#define VX_CBRT(a) cbrtf(a)
#else
#define VX_ADD(a, b) ((a) + (b))
#define VX_SUB(a, b) ((a) - (b))
#define VX_MUL(a, b) ((a) * (b))
#define VX_FMA(a, b, c) fmaf((a), (b), (c))
#define VX_DIV(a, b) ((a) / (b))
#define VX_SQRT(a) sqrtf(a)
#define VX_CBRT(a) cbrtf(a)
#endif

namespace vrs_exact {

// Metric codes: the reference's launch codes, crates/vector-cuda/src/knn.rs:235-246.
enum Metric : int {
  kL2 = 0, kDot = 1, kCos = 2, kL1 = 3, kMink = 4,
  kCheb = 5, kHam = 6, kMaha = 7, kJac = 8, kHell = 9
};

VX_HD bool higher_is_better(int m) { return m == kDot || m == kCos; }

VX_HD float fabs_(float x) { return fabsf(x); }
VX_HD float max_(float a, float b) { return a > b ? a : b; }
VX_HD float min_(float a, float b) { return a < b ? a : b; }

VX_HD float tree16(const float* v) {
  float t8[8], t4[4];
#pragma unroll
  for (int i = 0; i < 8; i++) t8[i] = VX_ADD(v[i], v[i + 8]);
#pragma unroll
  for (int i = 0; i < 4; i++) t4[i] = VX_ADD(t8[i], t8[i + 4]);
  float a = VX_ADD(t4[0], t4[2]), b = VX_ADD(t4[1], t4[3]);
  return VX_ADD(a, b);
}

VX_HD float tree16_max(const float* v) {
  float t8[8], t4[4];
#pragma unroll
  for (int i = 0; i < 8; i++) t8[i] = max_(v[i], v[i + 8]);
#pragma unroll
  for (int i = 0; i < 4; i++) t4[i] = max_(t8[i], t8[i + 4]);
  return max_(max_(t4[0], t4[2]), max_(t4[1], t4[3]));
}

// avx512::dot_product, avx512.rs:23-76
VX_HD float dot(const float* a, const float* b, int n) {
  float s0[16], s1[16], s2[16], s3[16];
#pragma unroll
  for (int l = 0; l < 16; l++) s0[l] = s1[l] = s2[l] = s3[l] = 0.0f;
  int chunks = n / 64;
  for (int c = 0; c < chunks; c++) {
    const float* pa = a + c * 64;
    const float* pb = b + c * 64;
#pragma unroll
    for (int l = 0; l < 16; l++) {
      s0[l] = VX_FMA(pa[l], pb[l], s0[l]);
      s1[l] = VX_FMA(pa[16 + l], pb[16 + l], s1[l]);
      s2[l] = VX_FMA(pa[32 + l], pb[32 + l], s2[l]);
      s3[l] = VX_FMA(pa[48 + l], pb[48 + l], s3[l]);
    }
  }
  int i = chunks * 64;
  for (; i + 16 <= n; i += 16) {
#pragma unroll
    for (int l = 0; l < 16; l++) s0[l] = VX_FMA(a[i + l], b[i + l], s0[l]);
  }
#pragma unroll
  for (int l = 0; l < 16; l++) s0[l] = VX_ADD(VX_ADD(s0[l], s1[l]), VX_ADD(s2[l], s3[l]));
  float r = tree16(s0);
  for (; i < n; i++) r = VX_ADD(r, VX_MUL(a[i], b[i]));
  return r;
}

// avx512::l2_squared, avx512.rs:87-148
VX_HD float l2(const float* a, const float* b, int n) {
  float s0[16], s1[16], s2[16], s3[16];
#pragma unroll
  for (int l = 0; l < 16; l++) s0[l] = s1[l] = s2[l] = s3[l] = 0.0f;
  int chunks = n / 64;
  for (int c = 0; c < chunks; c++) {
    const float* pa = a + c * 64;
    const float* pb = b + c * 64;
#pragma unroll
    for (int l = 0; l < 16; l++) {
      float d0 = VX_SUB(pa[l], pb[l]), d1 = VX_SUB(pa[16 + l], pb[16 + l]);
      float d2 = VX_SUB(pa[32 + l], pb[32 + l]), d3 = VX_SUB(pa[48 + l], pb[48 + l]);
      s0[l] = VX_FMA(d0, d0, s0[l]);
      s1[l] = VX_FMA(d1, d1, s1[l]);
      s2[l] = VX_FMA(d2, d2, s2[l]);
      s3[l] = VX_FMA(d3, d3, s3[l]);
    }
  }
  int i = chunks * 64;
  for (; i + 16 <= n; i += 16) {
#pragma unroll
    for (int l = 0; l < 16; l++) {
      float d = VX_SUB(a[i + l], b[i + l]);
      s0[l] = VX_FMA(d, d, s0[l]);
    }
  }
#pragma unroll
  for (int l = 0; l < 16; l++) s0[l] = VX_ADD(VX_ADD(s0[l], s1[l]), VX_ADD(s2[l], s3[l]));
  float r = tree16(s0);
  for (; i < n; i++) {
    float d = VX_SUB(a[i], b[i]);
    r = VX_ADD(r, VX_MUL(d, d));
  }
  return r;
}

// Sum of squares in the cosine kernel's order (two accumulator sets over
// 32-wide chunks, avx512.rs:161-223); `na` and `nb` there are this value of
// each operand, so it can be computed once per vector.
VX_HD float cos_norm_sq(const float* a, int n) {
  float s0[16], s1[16];
#pragma unroll
  for (int l = 0; l < 16; l++) s0[l] = s1[l] = 0.0f;
  int chunks = n / 32;
  for (int c = 0; c < chunks; c++) {
    const float* pa = a + c * 32;
#pragma unroll
    for (int l = 0; l < 16; l++) {
      s0[l] = VX_FMA(pa[l], pa[l], s0[l]);
      s1[l] = VX_FMA(pa[16 + l], pa[16 + l], s1[l]);
    }
  }
  int i = chunks * 32;
  for (; i + 16 <= n; i += 16) {
#pragma unroll
    for (int l = 0; l < 16; l++) s0[l] = VX_FMA(a[i + l], a[i + l], s0[l]);
  }
#pragma unroll
  for (int l = 0; l < 16; l++) s0[l] = VX_ADD(s0[l], s1[l]);
  float r = tree16(s0);
  for (; i < n; i++) r = VX_ADD(r, VX_MUL(a[i], a[i]));
  return r;
}

// Dot product in the cosine kernel's order.
VX_HD float cos_dot(const float* a, const float* b, int n) {
  float s0[16], s1[16];
#pragma unroll
  for (int l = 0; l < 16; l++) s0[l] = s1[l] = 0.0f;
  int chunks = n / 32;
  for (int c = 0; c < chunks; c++) {
    const float* pa = a + c * 32;
    const float* pb = b + c * 32;
#pragma unroll
    for (int l = 0; l < 16; l++) {
      s0[l] = VX_FMA(pa[l], pb[l], s0[l]);
      s1[l] = VX_FMA(pa[16 + l], pb[16 + l], s1[l]);
    }
  }
  int i = chunks * 32;
  for (; i + 16 <= n; i += 16) {
#pragma unroll
    for (int l = 0; l < 16; l++) s0[l] = VX_FMA(a[i + l], b[i + l], s0[l]);
  }
#pragma unroll
  for (int l = 0; l < 16; l++) s0[l] = VX_ADD(s0[l], s1[l]);
  float r = tree16(s0);
  for (; i < n; i++) r = VX_ADD(r, VX_MUL(a[i], b[i]));
  return r;
}

// Cosine tail of avx512.rs:215-222 from the three reductions.
VX_HD float cos_finish(float dotv, float na, float nb) {
  float den = VX_MUL(VX_SQRT(na), VX_SQRT(nb));
  return den <= 1e-9f ? 0.0f : VX_DIV(dotv, den);
}

// avx512::manhattan, avx512.rs:234-280
VX_HD float l1(const float* a, const float* b, int n) {
  float s0[16], s1[16];
#pragma unroll
  for (int l = 0; l < 16; l++) s0[l] = s1[l] = 0.0f;
  int chunks = n / 32;
  for (int c = 0; c < chunks; c++) {
    const float* pa = a + c * 32;
    const float* pb = b + c * 32;
#pragma unroll
    for (int l = 0; l < 16; l++) {
      s0[l] = VX_ADD(s0[l], fabs_(VX_SUB(pa[l], pb[l])));
      s1[l] = VX_ADD(s1[l], fabs_(VX_SUB(pa[16 + l], pb[16 + l])));
    }
  }
  int i = chunks * 32;
  for (; i + 16 <= n; i += 16) {
#pragma unroll
    for (int l = 0; l < 16; l++) s0[l] = VX_ADD(s0[l], fabs_(VX_SUB(a[i + l], b[i + l])));
  }
#pragma unroll
  for (int l = 0; l < 16; l++) s0[l] = VX_ADD(s0[l], s1[l]);
  float r = tree16(s0);
  for (; i < n; i++) r = VX_ADD(r, fabs_(VX_SUB(a[i], b[i])));
  return r;
}

// avx512::minkowski p=3 before the cube root, avx512.rs:300-340
VX_HD float mink3_sum(const float* a, const float* b, int n) {
  float s0[16], s1[16];
#pragma unroll
  for (int l = 0; l < 16; l++) s0[l] = s1[l] = 0.0f;
  int chunks = n / 32;
  for (int c = 0; c < chunks; c++) {
    const float* pa = a + c * 32;
    const float* pb = b + c * 32;
#pragma unroll
    for (int l = 0; l < 16; l++) {
      float x0 = fabs_(VX_SUB(pa[l], pb[l])), x1 = fabs_(VX_SUB(pa[16 + l], pb[16 + l]));
      s0[l] = VX_FMA(VX_MUL(x0, x0), x0, s0[l]);
      s1[l] = VX_FMA(VX_MUL(x1, x1), x1, s1[l]);
    }
  }
#pragma unroll
  for (int l = 0; l < 16; l++) s0[l] = VX_ADD(s0[l], s1[l]);
  float r = tree16(s0);
  for (int i = chunks * 32; i < n; i++) {
    float x = fabs_(VX_SUB(a[i], b[i]));
    r = VX_ADD(r, VX_MUL(VX_MUL(x, x), x));
  }
  return r;
}

// avx512::chebyshev, avx512.rs:354-390
VX_HD float cheb(const float* a, const float* b, int n) {
  if (n == 0) return 0.0f;
  float m[16];
#pragma unroll
  for (int l = 0; l < 16; l++) m[l] = 0.0f;
  int chunks = n / 16;
  for (int c = 0; c < chunks; c++) {
#pragma unroll
    for (int l = 0; l < 16; l++) m[l] = max_(m[l], fabs_(VX_SUB(a[c * 16 + l], b[c * 16 + l])));
  }
  float r = tree16_max(m);
  for (int i = chunks * 16; i < n; i++) {
    float x = fabs_(VX_SUB(a[i], b[i]));
    if (x > r) r = x;
  }
  return r;
}

// avx512::hamming, avx512.rs:401-433
VX_HD float ham(const float* a, const float* b, int n) {
  float count = 0.0f;
  int chunks = n / 16;
  for (int c = 0; c < chunks; c++) {
    int pc = 0;
#pragma unroll
    for (int l = 0; l < 16; l++) pc += fabs_(VX_SUB(a[c * 16 + l], b[c * 16 + l])) > 1e-6f ? 1 : 0;
    count = VX_ADD(count, (float)pc);
  }
  for (int i = chunks * 16; i < n; i++)
    if (fabs_(VX_SUB(a[i], b[i])) > 1e-6f) count = VX_ADD(count, 1.0f);
  return count;
}

// avx512::jaccard, avx512.rs:520-568
VX_HD float jac(const float* a, const float* b, int n) {
  float mn[16], mx[16];
#pragma unroll
  for (int l = 0; l < 16; l++) mn[l] = mx[l] = 0.0f;
  int chunks = n / 16;
  for (int c = 0; c < chunks; c++) {
#pragma unroll
    for (int l = 0; l < 16; l++) {
      float x = fabs_(a[c * 16 + l]), y = fabs_(b[c * 16 + l]);
      mn[l] = VX_ADD(mn[l], min_(x, y));
      mx[l] = VX_ADD(mx[l], max_(x, y));
    }
  }
  float smin = tree16(mn), smax = tree16(mx), rem = 0.0f;
  for (int i = chunks * 16; i < n; i++) {
    float x = fabs_(a[i]), y = fabs_(b[i]);
    rem = VX_ADD(rem, min_(x, y));
    smax = VX_ADD(smax, max_(x, y));
  }
  float tmin = VX_ADD(smin, rem);
  return smax <= 1e-9f ? 0.0f : VX_SUB(1.0f, VX_DIV(tmin, smax));
}

// Hellinger sum on operands that already hold sqrt(|v|) per element
// (avx512.rs:581-610 takes the roots inside; the roots are per-vector, so
// they are taken once per vector). The caller applies sqrt(0.5 * sum).
VX_HD float hell_sum_roots(const float* ra, const float* rb, int n) {
  float s[16];
#pragma unroll
  for (int l = 0; l < 16; l++) s[l] = 0.0f;
  int chunks = n / 16;
  for (int c = 0; c < chunks; c++) {
#pragma unroll
    for (int l = 0; l < 16; l++) {
      float d = VX_SUB(ra[c * 16 + l], rb[c * 16 + l]);
      s[l] = VX_FMA(d, d, s[l]);
    }
  }
  float r = tree16(s);
  for (int i = chunks * 16; i < n; i++) {
    float d = VX_SUB(ra[i], rb[i]);
    r = VX_ADD(r, VX_MUL(d, d));
  }
  return r;
}

VX_HD float root_abs(float v) { return VX_SQRT(fabs_(v)); }

// Rank key: orders like the metric, before the monotone final map.
// For kHell the operands must be the per-element roots (see above); for
// kCos the caller passes the two cos_norm_sq values.
VX_HD float rank_key(int metric, const float* a, const float* b, int n, float na, float nb) {
  switch (metric) {
    case kL2: case kMaha: return l2(a, b, n);
    case kDot: return dot(a, b, n);
    case kCos: return cos_finish(cos_dot(a, b, n), na, nb);
    case kL1: return l1(a, b, n);
    case kMink: return mink3_sum(a, b, n);
    case kCheb: return cheb(a, b, n);
    case kHam: return ham(a, b, n);
    case kJac: return jac(a, b, n);
    case kHell: return hell_sum_roots(a, b, n);
  }
  return 0.0f;
}

// Reported distance from a rank key (the reference's final map).
VX_HD float finish(int metric, float key) {
  switch (metric) {
    case kMink: return VX_CBRT(key);
    case kMaha: return VX_SQRT(key);
    case kHell: return VX_SQRT(VX_MUL(0.5f, key));
  }
  return key;
}

// Heap score: smaller is better (knn.rs:345-349 negates similarities).
VX_HD float heap_score(int metric, float key) { return higher_is_better(metric) ? -key : key; }

}  // namespace vrs_exact
