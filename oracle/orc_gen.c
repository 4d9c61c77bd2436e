/*
 * orc_gen.c -- TEST INFRASTRUCTURE ONLY: the seeded synthetic inputs of the
 * benchmark configs, generated on the host without libvrs.
 *
 * The reference arm of bench.py times the restated reference CPU path and
 * must not load the product library, yet it has to consume the same input
 * bits as the GPU path. This file restates the product's generator
 * (Philox4x32-10 keyed by a 64-bit seed, counter = (block_lo, block_hi,
 * stream, 0); Box-Muller in double with log/sin/cos from power series using
 * only IEEE +, *, /, sqrt) in plain C. Philox4x32-10 is the published
 * counter-based generator of Salmon, Moraes, Dror and Shaw ("Parallel
 * random numbers: as easy as 1, 2, 3", SC'11). tests/test_gen_oracle.py
 * checks every distribution bit for bit against vrs_gen_rows_host.
 *
 * Built with -ffp-contract=off (oracle/Makefile), so no a*b+c is fused and
 * every double operation rounds exactly as the product's host and device
 * builds do.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <string.h>

enum { G_NORMAL = 0, G_NORMAL_UNIT = 1, G_UNIFORM = 2, G_UNIFORM_SUM1 = 3, G_MIXTURE = 4 };
enum { S_COMPONENT = 3, S_NOISE = 4 };

typedef struct { uint32_t x, y, z, w; } u4_t;

static uint32_t mulhi32(uint32_t a, uint32_t b) { return (uint32_t)(((uint64_t)a * (uint64_t)b) >> 32); }

static u4_t philox(u4_t c, uint32_t k0, uint32_t k1) {
    for (int r = 0; r < 10; r++) {
        uint32_t hi0 = mulhi32(0xD2511F53u, c.x), lo0 = 0xD2511F53u * c.x;
        uint32_t hi1 = mulhi32(0xCD9E8D57u, c.z), lo1 = 0xCD9E8D57u * c.z;
        u4_t n = { hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0 };
        c = n;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return c;
}

static u4_t gblock(uint64_t seed, uint32_t stream, uint64_t b) {
    u4_t c = { (uint32_t)b, (uint32_t)(b >> 32), stream, 0u };
    return philox(c, (uint32_t)seed, (uint32_t)(seed >> 32));
}

static uint32_t gword(u4_t v, int j) { return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w; }

/* ln(x), x in [2^-32, 1]: x = m 2^e, m in [sqrt(1/2), sqrt(2)], ln m =
 * 2 atanh(t) with t = (m-1)/(m+1), odd series to t^25 (Horner in t^2). */
static double ln_unit(double x) {
    uint64_t u;
    memcpy(&u, &x, 8);
    int e = (int)((u >> 52) & 0x7ff) - 1023;
    uint64_t mb = (u & 0x000fffffffffffffull) | 0x3ff0000000000000ull;
    double m;
    memcpy(&m, &mb, 8);
    if (m > 0x1.6a09e667f3bcdp+0) { m = m * 0.5; e += 1; }
    double t = (m - 1.0) / (m + 1.0);
    double t2 = t * t;
    /* 1 / (2i + 1), i = 0..12, correctly rounded. */
    static const double c[13] = {0x1.0000000000000p+0, 0x1.5555555555555p-2, 0x1.999999999999ap-3,
                                 0x1.2492492492492p-3, 0x1.c71c71c71c71cp-4, 0x1.745d1745d1746p-4,
                                 0x1.3b13b13b13b14p-4, 0x1.1111111111111p-4, 0x1.e1e1e1e1e1e1ep-5,
                                 0x1.af286bca1af28p-5, 0x1.8618618618618p-5, 0x1.642c8590b2164p-5,
                                 0x1.47ae147ae147bp-5};
    double p = c[12];
    for (int i = 11; i >= 0; i--) p = p * t2 + c[i];
    return (double)e * 0x1.62e42fefa39efp-1 + (2.0 * t) * p;
}

/* sin and cos of 2 pi w / 2^32: quadrant from the top two bits, phi =
 * f pi/2 in [0, pi/2), Taylor series to phi^25 (coefficients +-1/n!). */
static void sincos_turn(uint32_t w, double* s, double* c) {
    int q = (int)(w >> 30);
    double f = (double)(w & 0x3fffffffu) * 0x1p-30;
    double x = f * 0x1.921fb54442d18p+0;
    double x2 = x * x;
    static const double sc[13] = {0x1.0000000000000p+0, -0x1.5555555555555p-3, 0x1.1111111111111p-7,
                                  -0x1.a01a01a01a01ap-13, 0x1.71de3a556c734p-19, -0x1.ae64567f544e4p-26,
                                  0x1.6124613a86d09p-33, -0x1.ae7f3e733b81fp-41, 0x1.952c77030ad4ap-49,
                                  -0x1.2f49b46814157p-57, 0x1.71b8ef6dcf572p-66, -0x1.761b41316381ap-75,
                                  0x1.3f3ccdd165fa9p-84};
    static const double cc[13] = {0x1.0000000000000p+0, -0x1.0000000000000p-1, 0x1.5555555555555p-5,
                                  -0x1.6c16c16c16c17p-10, 0x1.a01a01a01a01ap-16, -0x1.27e4fb7789f5cp-22,
                                  0x1.1eed8eff8d898p-29, -0x1.93974a8c07c9dp-37, 0x1.ae7f3e733b81fp-45,
                                  -0x1.6827863b97d97p-53, 0x1.e542ba4020225p-62, -0x1.0ce396db7f853p-70,
                                  0x1.f2cf01972f578p-80};
    double ps = sc[12], pc = cc[12];
    for (int i = 11; i >= 0; i--) {
        ps = ps * x2 + sc[i];
        pc = pc * x2 + cc[i];
    }
    double sn = ps * x, cs = pc;
    switch (q) {
    case 0: *s = sn; *c = cs; break;
    case 1: *s = cs; *c = -sn; break;
    case 2: *s = -sn; *c = -cs; break;
    default: *s = -cs; *c = sn; break;
    }
}

/* N(0,1) element e of (seed, stream): block e/4 holds two Box-Muller pairs;
 * even elements take the cosine, odd ones the sine of pair (e&3)/2. */
static double gnormal(uint64_t seed, uint32_t stream, uint64_t e) {
    u4_t v = gblock(seed, stream, e >> 2);
    int j = (int)(e & 3);
    uint32_t u1 = gword(v, (j >> 1) * 2), u2 = gword(v, (j >> 1) * 2 + 1);
    double U1 = ((double)u1 + 1.0) * 0x1p-32;
    double r = sqrt(-2.0 * ln_unit(U1));
    double s, c;
    sincos_turn(u2, &s, &c);
    return r * ((j & 1) ? s : c);
}

static float guniform(uint64_t seed, uint32_t stream, uint64_t e) {
    u4_t v = gblock(seed, stream, e >> 2);
    return (float)(gword(v, (int)(e & 3)) >> 8) * 0x1p-24f;
}

static uint32_t gcomponent(uint64_t seed, uint64_t i, uint32_t K) {
    u4_t v = gblock(seed, S_COMPONENT, i >> 2);
    return (uint32_t)(((uint64_t)gword(v, (int)(i & 3)) * (uint64_t)K) >> 32);
}

static void gen_row(int kind, uint64_t seed, uint32_t stream, int64_t row, int d, float* out,
                    const float* centres, uint32_t K, double sigma) {
    uint64_t e0 = (uint64_t)row * (uint64_t)d;
    if (kind == G_NORMAL || kind == G_NORMAL_UNIT) {
        for (int j = 0; j < d; j++) out[j] = (float)gnormal(seed, stream, e0 + j);
        if (kind == G_NORMAL_UNIT) {
            double ss = 0.0;
            for (int j = 0; j < d; j++) ss = ss + (double)out[j] * (double)out[j];
            double nrm = sqrt(ss);
            if (nrm > 0.0)
                for (int j = 0; j < d; j++) out[j] = (float)((double)out[j] / nrm);
        }
    } else if (kind == G_UNIFORM || kind == G_UNIFORM_SUM1) {
        for (int j = 0; j < d; j++) out[j] = guniform(seed, stream, e0 + j);
        if (kind == G_UNIFORM_SUM1) {
            double s = 0.0;
            for (int j = 0; j < d; j++) s = s + (double)out[j];
            if (s > 0.0)
                for (int j = 0; j < d; j++) out[j] = (float)((double)out[j] / s);
        }
    } else {
        uint32_t c = gcomponent(seed, (uint64_t)row, K);
        const float* ctr = centres + (uint64_t)c * (uint64_t)d;
        for (int j = 0; j < d; j++) out[j] = (float)((double)ctr[j] + sigma * gnormal(seed, S_NOISE, e0 + j));
    }
}

typedef struct {
    int kind; uint64_t seed; uint32_t stream; int64_t row0, r0, r1; int d; float* out;
    const float* centres; uint32_t K; double sigma;
} gen_job_t;

static void* gen_worker(void* arg) {
    gen_job_t* j = arg;
    for (int64_t r = j->r0; r < j->r1; r++)
        gen_row(j->kind, j->seed, j->stream, j->row0 + r, j->d, j->out + r * j->d, j->centres, j->K, j->sigma);
    return NULL;
}

/* Rows [row0, row0 + rows) of the conceptual matrix, packed (d floats
 * apart), split over nthreads host threads. Returns 0, or -1 on bad
 * arguments. kind: 0 N(0,1); 1 N(0,1) rows L2-normalised (f64); 2 U[0,1);
 * 3 U[0,1) rows rescaled to sum 1 (f64); 4 mixture: centre (K x d) chosen
 * per row + sigma * N(0,1). */
int orc_gen_rows(int kind, uint64_t seed, uint32_t stream, int64_t row0, int64_t rows, int d, float* out,
                 const float* centres, uint32_t K, double sigma, int nthreads) {
    if (kind < 0 || kind > 4 || d <= 0 || rows < 0 || (kind == G_MIXTURE && (!centres || K == 0))) return -1;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if (rows < 64 * (int64_t)nthreads) nthreads = 1;
    pthread_t th[256];
    gen_job_t jobs[256];
    int64_t per = (rows + nthreads - 1) / nthreads;
    int started = 0;
    for (int t = 0; t < nthreads; t++) {
        int64_t r0 = t * per, r1 = r0 + per < rows ? r0 + per : rows;
        if (r0 >= r1) break;
        jobs[t] = (gen_job_t){ kind, seed, stream, row0, r0, r1, d, out, centres, K, sigma };
        if (nthreads == 1) {
            gen_worker(&jobs[t]);
            continue;
        }
        pthread_create(&th[t], NULL, gen_worker, &jobs[t]);
        started++;
    }
    for (int t = 0; t < started; t++) pthread_join(th[t], NULL);
    return 0;
}
