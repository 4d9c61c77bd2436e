// vrs_gen.cuh -- seeded synthetic inputs, bit-identical on host and device.
//
// Counter-based Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random
// numbers: as easy as 1, 2, 3", SC'11) keyed by a 64-bit seed; the counter
// is (block_lo, block_hi, stream, 0) so any element of any matrix can be
// produced independently (row shards on different GPUs, host or device).
//
// Normal draws use Box-Muller in double precision with this file's own
// log/sin/cos written from their power series using only IEEE +, *, / and
// sqrt, so host and device produce the same bits. Every double operation
// goes through GD_* below: on the device these are the _rn intrinsics (no
// FMA contraction); the host side is compiled with -ffp-contract=off.
#pragma once
#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define VRS_HD __host__ __device__ __forceinline__
#else
#define VRS_HD inline
#endif

#if defined(__CUDA_ARCH__)
#define GD_MUL(a, b) __dmul_rn((a), (b))
#define GD_ADD(a, b) __dadd_rn((a), (b))
#define GD_SUB(a, b) __dsub_rn((a), (b))
#define GD_DIV(a, b) __ddiv_rn((a), (b))
#define GD_SQRT(a) __dsqrt_rn(a)
#else
#include <math.h>
#define GD_MUL(a, b) ((a) * (b))
#define GD_ADD(a, b) ((a) + (b))
#define GD_SUB(a, b) ((a) - (b))
#define GD_DIV(a, b) ((a) / (b))
#define GD_SQRT(a) sqrt(a)
#endif

namespace vrs_gen {

// Stream ids inside one config seed.
enum Stream : uint32_t { kBase = 0, kQuery = 1, kCentre = 2, kComponent = 3, kNoise = 4 };

struct U4 { uint32_t x, y, z, w; };

VRS_HD uint32_t mulhi32(uint32_t a, uint32_t b) {
  return (uint32_t)(((uint64_t)a * (uint64_t)b) >> 32);
}

// Philox4x32 with 10 rounds; constants are the published multipliers and
// Weyl key increments of the Philox4x32 family.
VRS_HD U4 philox4x32_10(U4 c, uint32_t k0, uint32_t k1) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  const uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; r++) {
    uint32_t hi0 = mulhi32(M0, c.x), lo0 = M0 * c.x;
    uint32_t hi1 = mulhi32(M1, c.z), lo1 = M1 * c.z;
    U4 n;
    n.x = hi1 ^ c.y ^ k0;
    n.y = lo1;
    n.z = hi0 ^ c.w ^ k1;
    n.w = lo0;
    c = n;
    k0 += W0;
    k1 += W1;
  }
  return c;
}

VRS_HD U4 block(uint64_t seed, uint32_t stream, uint64_t b) {
  U4 c = {(uint32_t)b, (uint32_t)(b >> 32), stream, 0u};
  return philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
}

VRS_HD uint32_t word(U4 v, int j) { return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w; }

VRS_HD uint64_t dbits(double x) { uint64_t u; memcpy(&u, &x, 8); return u; }
VRS_HD double bitsd(uint64_t u) { double x; memcpy(&x, &u, 8); return x; }

// ln(x) for x in [2^-32, 1]: x = m 2^e with m in [sqrt(1/2), sqrt(2)],
// ln m = 2 atanh(t), t = (m-1)/(m+1), |t| <= 0.1716, series to t^25.
VRS_HD double ln_unit(double x) {
  uint64_t u = dbits(x);
  int e = (int)((u >> 52) & 0x7ff) - 1023;
  double m = bitsd((u & 0x000fffffffffffffull) | 0x3ff0000000000000ull);  // [1, 2)
  if (m > 0x1.6a09e667f3bcdp+0) { m = GD_MUL(m, 0.5); e += 1; }
  double t = GD_DIV(GD_SUB(m, 1.0), GD_ADD(m, 1.0));
  double t2 = GD_MUL(t, t);
  const double c[13] = {0x1.0000000000000p+0, 0x1.5555555555555p-2, 0x1.999999999999ap-3,
                        0x1.2492492492492p-3, 0x1.c71c71c71c71cp-4, 0x1.745d1745d1746p-4,
                        0x1.3b13b13b13b14p-4, 0x1.1111111111111p-4, 0x1.e1e1e1e1e1e1ep-5,
                        0x1.af286bca1af28p-5, 0x1.8618618618618p-5, 0x1.642c8590b2164p-5,
                        0x1.47ae147ae147bp-5};
  double p = c[12];
  for (int i = 11; i >= 0; i--) p = GD_ADD(GD_MUL(p, t2), c[i]);
  return GD_ADD(GD_MUL((double)e, 0x1.62e42fefa39efp-1), GD_MUL(GD_MUL(2.0, t), p));
}

// sin and cos of 2*pi*u for u = w * 2^-32: quadrant from the top two bits,
// phi = f * pi/2 in [0, pi/2), Taylor series to phi^25.
VRS_HD void sincos_turn(uint32_t w, double* s, double* c) {
  int q = (int)(w >> 30);
  double f = (double)(w & 0x3fffffffu) * 0x1p-30;  // exact
  double x = GD_MUL(f, 0x1.921fb54442d18p+0);
  double x2 = GD_MUL(x, x);
  const double sc[13] = {0x1.0000000000000p+0, -0x1.5555555555555p-3, 0x1.1111111111111p-7,
                         -0x1.a01a01a01a01ap-13, 0x1.71de3a556c734p-19, -0x1.ae64567f544e4p-26,
                         0x1.6124613a86d09p-33, -0x1.ae7f3e733b81fp-41, 0x1.952c77030ad4ap-49,
                         -0x1.2f49b46814157p-57, 0x1.71b8ef6dcf572p-66, -0x1.761b41316381ap-75,
                         0x1.3f3ccdd165fa9p-84};
  const double cc[13] = {0x1.0000000000000p+0, -0x1.0000000000000p-1, 0x1.5555555555555p-5,
                         -0x1.6c16c16c16c17p-10, 0x1.a01a01a01a01ap-16, -0x1.27e4fb7789f5cp-22,
                         0x1.1eed8eff8d898p-29, -0x1.93974a8c07c9dp-37, 0x1.ae7f3e733b81fp-45,
                         -0x1.6827863b97d97p-53, 0x1.e542ba4020225p-62, -0x1.0ce396db7f853p-70,
                         0x1.f2cf01972f578p-80};
  double ps = sc[12], pc = cc[12];
  for (int i = 11; i >= 0; i--) {
    ps = GD_ADD(GD_MUL(ps, x2), sc[i]);
    pc = GD_ADD(GD_MUL(pc, x2), cc[i]);
  }
  double sn = GD_MUL(ps, x), cs = pc;
  switch (q) {
    case 0: *s = sn; *c = cs; break;
    case 1: *s = cs; *c = -sn; break;
    case 2: *s = -sn; *c = -cs; break;
    default: *s = -cs; *c = sn; break;
  }
}

// Standard normal (double) for element e of (seed, stream): Philox block
// e/4 gives two Box-Muller pairs; element e&3 takes cos (even) or sin (odd)
// of pair (e&3)/2.
VRS_HD double normal(uint64_t seed, uint32_t stream, uint64_t e) {
  U4 v = block(seed, stream, e >> 2);
  int j = (int)(e & 3);
  uint32_t u1 = word(v, (j >> 1) * 2), u2 = word(v, (j >> 1) * 2 + 1);
  double U1 = GD_MUL(GD_ADD((double)u1, 1.0), 0x1p-32);  // (0, 1]
  double r = GD_SQRT(GD_MUL(-2.0, ln_unit(U1)));
  double s, c;
  sincos_turn(u2, &s, &c);
  return GD_MUL(r, (j & 1) ? s : c);
}

// Uniform float in [0, 1): (u >> 8) * 2^-24.
VRS_HD float uniform01(uint64_t seed, uint32_t stream, uint64_t e) {
  U4 v = block(seed, stream, e >> 2);
  return (float)(word(v, (int)(e & 3)) >> 8) * 0x1p-24f;
}

// Component index in [0, K) by multiply-shift of a 32-bit draw.
VRS_HD uint32_t component(uint64_t seed, uint64_t i, uint32_t K) {
  U4 v = block(seed, kComponent, i >> 2);
  return (uint32_t)(((uint64_t)word(v, (int)(i & 3)) * (uint64_t)K) >> 32);
}

// Distributions of one matrix row (kind values match vrs.h VRS_GEN_*).
enum Kind : int { kNormal = 0, kNormalUnit = 1, kUniform = 2, kUniformSum1 = 3, kMixture = 4 };

// Writes row `row` (global index) of a rows x d matrix into out[0..d).
// centres (mixture only): K x d floats, generated with kCentre / kNormal.
VRS_HD void gen_row(int kind, uint64_t seed, uint32_t stream, int64_t row, int d,
                    float* out, const float* centres, uint32_t K, double sigma) {
  uint64_t e0 = (uint64_t)row * (uint64_t)d;
  if (kind == kNormal || kind == kNormalUnit) {
    for (int j = 0; j < d; j++) out[j] = (float)normal(seed, stream, e0 + j);
    if (kind == kNormalUnit) {
      double ss = 0.0;
      for (int j = 0; j < d; j++) ss = GD_ADD(ss, GD_MUL((double)out[j], (double)out[j]));
      double nrm = GD_SQRT(ss);
      if (nrm > 0.0)
        for (int j = 0; j < d; j++) out[j] = (float)GD_DIV((double)out[j], nrm);
    }
  } else if (kind == kUniform || kind == kUniformSum1) {
    for (int j = 0; j < d; j++) out[j] = uniform01(seed, stream, e0 + j);
    if (kind == kUniformSum1) {
      double s = 0.0;
      for (int j = 0; j < d; j++) s = GD_ADD(s, (double)out[j]);
      if (s > 0.0)
        for (int j = 0; j < d; j++) out[j] = (float)GD_DIV((double)out[j], s);
    }
  } else {  // kMixture
    uint32_t c = component(seed, (uint64_t)row, K);
    const float* ctr = centres + (uint64_t)c * (uint64_t)d;
    for (int j = 0; j < d; j++)
      out[j] = (float)GD_ADD((double)ctr[j], GD_MUL(sigma, normal(seed, kNoise, e0 + j)));
  }
}

}  // namespace vrs_gen
