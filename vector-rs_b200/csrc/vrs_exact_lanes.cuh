// vrs_exact_lanes.cuh -- the reference's AVX-512 pair arithmetic computed by
// a half-warp: lane l (0..15) plays SIMD lane l, loads are coalesced, and the
// horizontal add is a shuffle halving tree (xor 8, 4, 2, 1), which pairs the
// same elements as _mm512_reduce_add_ps. Results are bit-identical to
// vrs_exact.cuh (and to crates/vector-simd/src/avx512.rs). Every lane of the
// half-warp returns the same value; all 16 lanes must call together.
#pragma once
#include "vrs_exact.cuh"

namespace vrs_exact {
namespace lanes {

// `mask` names the lanes taking part: the full warp, or one half-warp when
// the two halves run independently.
__device__ __forceinline__ float hsum16(float v, unsigned mask = 0xffffffffu) {
  v = __fadd_rn(v, __shfl_xor_sync(mask, v, 8, 16));
  v = __fadd_rn(v, __shfl_xor_sync(mask, v, 4, 16));
  v = __fadd_rn(v, __shfl_xor_sync(mask, v, 2, 16));
  v = __fadd_rn(v, __shfl_xor_sync(mask, v, 1, 16));
  return v;
}

// avx512::dot_product (avx512.rs:23-76)
__device__ __forceinline__ float dot(const float* __restrict__ a, const float* __restrict__ b, int n,
                                     int l, unsigned mask = 0xffffffffu) {
  float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
  const int chunks = n / 64;
  for (int c = 0; c < chunks; c++) {
    const float* pa = a + c * 64 + l;
    const float* pb = b + c * 64 + l;
    s0 = __fmaf_rn(pa[0], pb[0], s0);
    s1 = __fmaf_rn(pa[16], pb[16], s1);
    s2 = __fmaf_rn(pa[32], pb[32], s2);
    s3 = __fmaf_rn(pa[48], pb[48], s3);
  }
  int i = chunks * 64;
  for (; i + 16 <= n; i += 16) s0 = __fmaf_rn(a[i + l], b[i + l], s0);
  float r = hsum16(__fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3)), mask);
  for (; i < n; i++) r = __fadd_rn(r, __fmul_rn(a[i], b[i]));
  return r;
}

// avx512::l2_squared (avx512.rs:87-148)
__device__ __forceinline__ float l2(const float* __restrict__ a, const float* __restrict__ b, int n,
                                    int l, unsigned mask = 0xffffffffu) {
  float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
  const int chunks = n / 64;
  for (int c = 0; c < chunks; c++) {
    const float* pa = a + c * 64 + l;
    const float* pb = b + c * 64 + l;
    float d0 = __fsub_rn(pa[0], pb[0]), d1 = __fsub_rn(pa[16], pb[16]);
    float d2 = __fsub_rn(pa[32], pb[32]), d3 = __fsub_rn(pa[48], pb[48]);
    s0 = __fmaf_rn(d0, d0, s0);
    s1 = __fmaf_rn(d1, d1, s1);
    s2 = __fmaf_rn(d2, d2, s2);
    s3 = __fmaf_rn(d3, d3, s3);
  }
  int i = chunks * 64;
  for (; i + 16 <= n; i += 16) {
    float d = __fsub_rn(a[i + l], b[i + l]);
    s0 = __fmaf_rn(d, d, s0);
  }
  float r = hsum16(__fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3)), mask);
  for (; i < n; i++) {
    float d = __fsub_rn(a[i], b[i]);
    r = __fadd_rn(r, __fmul_rn(d, d));
  }
  return r;
}

// Dot product in the cosine kernel's order (avx512.rs:161-223).
__device__ __forceinline__ float cos_dot(const float* __restrict__ a, const float* __restrict__ b,
                                         int n, int l, unsigned mask = 0xffffffffu) {
  float s0 = 0.0f, s1 = 0.0f;
  const int chunks = n / 32;
  for (int c = 0; c < chunks; c++) {
    const float* pa = a + c * 32 + l;
    const float* pb = b + c * 32 + l;
    s0 = __fmaf_rn(pa[0], pb[0], s0);
    s1 = __fmaf_rn(pa[16], pb[16], s1);
  }
  int i = chunks * 32;
  for (; i + 16 <= n; i += 16) s0 = __fmaf_rn(a[i + l], b[i + l], s0);
  float r = hsum16(__fadd_rn(s0, s1), mask);
  for (; i < n; i++) r = __fadd_rn(r, __fmul_rn(a[i], b[i]));
  return r;
}

// Two rows against one query in one pass (row loads of both in flight);
// each result is bit-identical to the single-row function.
__device__ __forceinline__ void dot2(const float* __restrict__ a, const float* __restrict__ b0,
                                     const float* __restrict__ b1, int n, int l, unsigned mask,
                                     float* r0, float* r1) {
  float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
  float t0 = 0.0f, t1 = 0.0f, t2 = 0.0f, t3 = 0.0f;
  const int chunks = n / 64;
  for (int c = 0; c < chunks; c++) {
    const float* pa = a + c * 64 + l;
    const float* p0 = b0 + c * 64 + l;
    const float* p1 = b1 + c * 64 + l;
    const float a0 = pa[0], a1 = pa[16], a2 = pa[32], a3 = pa[48];
    const float x0 = p0[0], x1 = p0[16], x2 = p0[32], x3 = p0[48];
    const float y0 = p1[0], y1 = p1[16], y2 = p1[32], y3 = p1[48];
    s0 = __fmaf_rn(a0, x0, s0);
    s1 = __fmaf_rn(a1, x1, s1);
    s2 = __fmaf_rn(a2, x2, s2);
    s3 = __fmaf_rn(a3, x3, s3);
    t0 = __fmaf_rn(a0, y0, t0);
    t1 = __fmaf_rn(a1, y1, t1);
    t2 = __fmaf_rn(a2, y2, t2);
    t3 = __fmaf_rn(a3, y3, t3);
  }
  int i = chunks * 64;
  for (; i + 16 <= n; i += 16) {
    const float av = a[i + l];
    s0 = __fmaf_rn(av, b0[i + l], s0);
    t0 = __fmaf_rn(av, b1[i + l], t0);
  }
  float u0 = hsum16(__fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3)), mask);
  float u1 = hsum16(__fadd_rn(__fadd_rn(t0, t1), __fadd_rn(t2, t3)), mask);
  for (; i < n; i++) {
    u0 = __fadd_rn(u0, __fmul_rn(a[i], b0[i]));
    u1 = __fadd_rn(u1, __fmul_rn(a[i], b1[i]));
  }
  *r0 = u0;
  *r1 = u1;
}

__device__ __forceinline__ void l2_2(const float* __restrict__ a, const float* __restrict__ b0,
                                     const float* __restrict__ b1, int n, int l, unsigned mask,
                                     float* r0, float* r1) {
  float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
  float t0 = 0.0f, t1 = 0.0f, t2 = 0.0f, t3 = 0.0f;
  const int chunks = n / 64;
  for (int c = 0; c < chunks; c++) {
    const float* pa = a + c * 64 + l;
    const float* p0 = b0 + c * 64 + l;
    const float* p1 = b1 + c * 64 + l;
    const float a0 = pa[0], a1 = pa[16], a2 = pa[32], a3 = pa[48];
    const float x0 = __fsub_rn(a0, p0[0]), x1 = __fsub_rn(a1, p0[16]);
    const float x2 = __fsub_rn(a2, p0[32]), x3 = __fsub_rn(a3, p0[48]);
    const float y0 = __fsub_rn(a0, p1[0]), y1 = __fsub_rn(a1, p1[16]);
    const float y2 = __fsub_rn(a2, p1[32]), y3 = __fsub_rn(a3, p1[48]);
    s0 = __fmaf_rn(x0, x0, s0);
    s1 = __fmaf_rn(x1, x1, s1);
    s2 = __fmaf_rn(x2, x2, s2);
    s3 = __fmaf_rn(x3, x3, s3);
    t0 = __fmaf_rn(y0, y0, t0);
    t1 = __fmaf_rn(y1, y1, t1);
    t2 = __fmaf_rn(y2, y2, t2);
    t3 = __fmaf_rn(y3, y3, t3);
  }
  int i = chunks * 64;
  for (; i + 16 <= n; i += 16) {
    const float av = a[i + l];
    const float x = __fsub_rn(av, b0[i + l]), y = __fsub_rn(av, b1[i + l]);
    s0 = __fmaf_rn(x, x, s0);
    t0 = __fmaf_rn(y, y, t0);
  }
  float u0 = hsum16(__fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3)), mask);
  float u1 = hsum16(__fadd_rn(__fadd_rn(t0, t1), __fadd_rn(t2, t3)), mask);
  for (; i < n; i++) {
    const float x = __fsub_rn(a[i], b0[i]), y = __fsub_rn(a[i], b1[i]);
    u0 = __fadd_rn(u0, __fmul_rn(x, x));
    u1 = __fadd_rn(u1, __fmul_rn(y, y));
  }
  *r0 = u0;
  *r1 = u1;
}

__device__ __forceinline__ void cos_dot2(const float* __restrict__ a, const float* __restrict__ b0,
                                         const float* __restrict__ b1, int n, int l, unsigned mask,
                                         float* r0, float* r1) {
  float s0 = 0.0f, s1 = 0.0f, t0 = 0.0f, t1 = 0.0f;
  const int chunks = n / 32;
  for (int c = 0; c < chunks; c++) {
    const float* pa = a + c * 32 + l;
    const float* p0 = b0 + c * 32 + l;
    const float* p1 = b1 + c * 32 + l;
    const float a0 = pa[0], a1 = pa[16];
    const float x0 = p0[0], x1 = p0[16], y0 = p1[0], y1 = p1[16];
    s0 = __fmaf_rn(a0, x0, s0);
    s1 = __fmaf_rn(a1, x1, s1);
    t0 = __fmaf_rn(a0, y0, t0);
    t1 = __fmaf_rn(a1, y1, t1);
  }
  int i = chunks * 32;
  for (; i + 16 <= n; i += 16) {
    const float av = a[i + l];
    s0 = __fmaf_rn(av, b0[i + l], s0);
    t0 = __fmaf_rn(av, b1[i + l], t0);
  }
  float u0 = hsum16(__fadd_rn(s0, s1), mask);
  float u1 = hsum16(__fadd_rn(t0, t1), mask);
  for (; i < n; i++) {
    u0 = __fadd_rn(u0, __fmul_rn(a[i], b0[i]));
    u1 = __fadd_rn(u1, __fmul_rn(a[i], b1[i]));
  }
  *r0 = u0;
  *r1 = u1;
}

// Rank keys of two rows (see rank_key).
__device__ __forceinline__ void rank_key2(int metric, const float* a, const float* b0, const float* b1,
                                          int n, float na, float nb0, float nb1, int l, unsigned mask,
                                          float* k0, float* k1) {
  switch (metric) {
    case kL2:
    case kMaha: l2_2(a, b0, b1, n, l, mask, k0, k1); return;
    case kDot: dot2(a, b0, b1, n, l, mask, k0, k1); return;
    case kCos: {
      float d0, d1;
      cos_dot2(a, b0, b1, n, l, mask, &d0, &d1);
      *k0 = cos_finish(d0, na, nb0);
      *k1 = cos_finish(d1, na, nb1);
      return;
    }
  }
  *k0 = 0.0f;
  *k1 = 0.0f;
}

// Rank key for the metrics re-ranked by lanes (others are scanned exactly).
__device__ __forceinline__ float rank_key(int metric, const float* a, const float* b, int n, float na,
                                          float nb, int l, unsigned mask = 0xffffffffu) {
  switch (metric) {
    case kL2:
    case kMaha: return l2(a, b, n, l, mask);
    case kDot: return dot(a, b, n, l, mask);
    case kCos: return cos_finish(cos_dot(a, b, n, l, mask), na, nb);
  }
  return 0.0f;
}

}  // namespace lanes
}  // namespace vrs_exact
