/*
 * exl3_oracle.c -- CPU restatement of the EXL3 decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see exl3_oracle.h).  Compiled with
 * -ffp-contract=off so that float expressions keep the reference's operation
 * order exactly (exo_reconstruct is bit-compared against the reference's own
 * dequant_cpu built from source).
 */
#include "exl3_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ---------------------------------------------------------------- halves */

float exo_half_to_float(uint16_t h) {
    const uint32_t sign = (h >> 15) & 1u;
    const uint32_t exp = (h >> 10) & 0x1fu;
    const uint32_t mant = h & 0x3ffu;
    float v;
    if (exp == 0) {
        v = ldexpf((float) mant, -24);
    } else if (exp == 31) {
        v = mant ? NAN : INFINITY;
    } else {
        v = ldexpf((float) (mant | 0x400u), (int) exp - 25);
    }
    return sign ? -v : v;
}

uint16_t exo_half_from_double(double v) {
    if (isnan(v)) return 0x7e00u;
    const uint16_t sign = signbit(v) ? 0x8000u : 0u;
    const double a = fabs(v);
    if (a >= 65520.0) return (uint16_t) (sign | 0x7c00u);
    if (a < 6.103515625e-05) {                 /* below 2^-14: subnormal grid 2^-24 */
        const double q = nearbyint(a * 16777216.0);
        return (uint16_t) (sign | (uint16_t) q);   /* q == 1024 is the smallest normal */
    }
    int e;
    frexp(a, &e);                              /* a = m * 2^e, m in [0.5, 1) */
    double q = nearbyint(ldexp(a, 11 - e));    /* 11 significant bits: [1024, 2048] */
    int E = e - 1;
    if (q >= 2048.0) { q = 1024.0; E += 1; }
    if (E > 15) return (uint16_t) (sign | 0x7c00u);
    return (uint16_t) (sign | (uint16_t) ((E + 15) << 10) | (uint16_t) ((int) q - 1024));
}

/* The reference helper's conversion, kept only to pin the oracle against the
 * reference build: mantissa bits beyond fp16 are dropped, not rounded
 * (orders/F1-ref/exl3_dequant.cuh:41-55). */
uint16_t exo_half_from_float_trunc(float value) {
    uint32_t raw;
    memcpy(&raw, &value, sizeof(raw));
    const uint32_t sign = (raw >> 16) & 0x8000u;
    const int exp = (int) ((raw >> 23) & 0xffu) - 127;
    const uint32_t mant = raw & 0x7fffffu;
    if (exp > 15) return (uint16_t) (sign | 0x7c00u);
    if (exp < -14) {
        if (exp < -24) return (uint16_t) sign;
        const uint32_t m = (mant | 0x800000u) >> (-exp - 1);
        return (uint16_t) (sign | (m >> 13));
    }
    return (uint16_t) (sign | ((uint32_t) (exp + 15) << 10) | (mant >> 13));
}

uint16_t exo_bf16_from_double(double v) {
    if (isnan(v)) return 0x7fc0u;
    float f = (float) v;                       /* correct for the values used here */
    uint32_t raw;
    memcpy(&raw, &f, sizeof(raw));
    const uint32_t lsb = (raw >> 16) & 1u;
    raw += 0x7fffu + lsb;
    return (uint16_t) (raw >> 16);
}

static double bf16_to_double(uint16_t b) {
    uint32_t raw = (uint32_t) b << 16;
    float f;
    memcpy(&f, &raw, sizeof(f));
    return (double) f;
}

/* Load element i of an activation row as an fp16 value (the kernels convert
 * bf16 / fp32 activations to fp16 on load, lna_moe_ticket.cu:122-131). */
static uint16_t load_as_half(const void* x, int dtype, int64_t i) {
    if (dtype == EXO_F16) return ((const uint16_t*) x)[i];
    if (dtype == EXO_BF16) return exo_half_from_double(bf16_to_double(((const uint16_t*) x)[i]));
    return exo_half_from_double((double) ((const float*) x)[i]);
}

/* ------------------------------------------------------- trellis windows */

/* Weight t of a tile is the 16-bit window that ENDS at stream bit
 * (t + 257) * K - 1, modulo the 256 K-bit circular stream of the tile.  The
 * stream is read most-significant-bit first from uint32 words built from
 * little-endian uint16 pairs (exl3_dequant.cuh:110-128, exl3_dq.cuh:15-31). */
uint32_t exo_window(const uint16_t* tile, int K, int t) {
    const int nbits = 256 * K;
    const int start = ((t + 257) * K - 16) % nbits;
    uint32_t w = 0;
    for (int b = 0; b < 16; ++b) {
        const int p = (start + b) % nbits;
        const int wi = p >> 5;
        const uint32_t word = (uint32_t) tile[2 * wi] | ((uint32_t) tile[2 * wi + 1] << 16);
        w = (w << 1) | ((word >> (31 - (p & 31))) & 1u);
    }
    return w;
}

/* --------------------------------------------------------------- codebooks */

static uint32_t lop3_6a(uint32_t a, uint32_t b, uint32_t c) {
    /* LUT 0x6A over (a,b,c) is (a & b) ^ c. */
    return (a & b) ^ c;
}

uint16_t exo_codebook(uint32_t window, int cb, int trunc) {
    uint32_t x = window & 0xffffu;
    if (cb == 0 || cb == 1) {
        if (cb == 0) x = x * 89226354u + 64248484u;   /* 3INST */
        else         x = x * 0xCBAC1FEDu;              /* MCG   */
        x = lop3_6a(x, 0x8fff8fffu, 0x3b603b60u);
        const float lo = exo_half_to_float((uint16_t) (x & 0xffffu));
        const float hi = exo_half_to_float((uint16_t) (x >> 16));
        /* Both halves are forced into [2^-3, 2): the float sum is exact, so a
         * single nearest-even rounding equals the device's __hadd. */
        const double sum = (double) lo + (double) hi;
        return trunc ? exo_half_from_float_trunc((float) sum) : exo_half_from_double(sum);
    }
    /* MUL1: byte sum of the product as an fp16 integer, then one fma. */
    x *= 0x83DCD12Du;
    const uint32_t s = 0x6400u + (x & 0xffu) + ((x >> 8) & 0xffu) + ((x >> 16) & 0xffu) + (x >> 24);
    const double v = (double) exo_half_to_float((uint16_t) s) * (double) exo_half_to_float(0x1eeeu)
                   + (double) exo_half_to_float(0xc931u);
    return trunc ? exo_half_from_float_trunc((float) v) : exo_half_from_double(v);
}

/* The codebook value before any fp16 rounding: lo + hi exactly for 3INST /
 * MCG (the form the fast GEMV path feeds to the tensor core), the fp16
 * result for MUL1 (which has a single value). */
double exo_codebook_exact(uint32_t window, int cb) {
    if (cb == 2) return (double) exo_half_to_float(exo_codebook(window, 2, 0));
    uint32_t x = window & 0xffffu;
    if (cb == 0) x = x * 89226354u + 64248484u;
    else         x = x * 0xCBAC1FEDu;
    x = lop3_6a(x, 0x8fff8fffu, 0x3b603b60u);
    return (double) exo_half_to_float((uint16_t) (x & 0xffffu)) + (double) exo_half_to_float((uint16_t) (x >> 16));
}

/* ----------------------------------------------------------- tile layout */

/* Lane l decodes weights t = 8l .. 8l+7 of a tile; weight t lands at
 *   k = 2(l%4) + (j&1) + 8((j>>1)&1),  n = l/4 + 8(j>>2),   j = t%8
 * which is the host restatement of the fragment swizzle in
 * recipe-lna/lna2/bindings.cpp:52-76 (own/peer lanes l and l+4). */
static void tile_position(int t, int* k, int* n) {
    const int l = t >> 3, j = t & 7;
    *k = 2 * (l & 3) + (j & 1) + 8 * ((j >> 1) & 1);
    *n = (l >> 2) + 8 * (j >> 2);
}

void exo_decode(const int16_t* trellis, int64_t kt, int64_t nt, int K, int cb,
                int trunc, uint16_t* wprime) {
    const int64_t cols = nt * 16;
    for (int64_t a = 0; a < kt; ++a) {
        for (int64_t b = 0; b < nt; ++b) {
            const uint16_t* tile = (const uint16_t*) (trellis + (a * nt + b) * 16 * K);
            for (int t = 0; t < 256; ++t) {
                int k, n;
                tile_position(t, &k, &n);
                wprime[(a * 16 + k) * cols + b * 16 + n] = exo_codebook(exo_window(tile, K, t), cb, trunc);
            }
        }
    }
}

/* W' as doubles: the fp16-rounded weights (exact = 0) or lo + hi (exact = 1).
 * Every weight is computed on its own, so the tile rows are shared out over
 * host threads (EXO_THREADS, default: the online cores, at most 64); the
 * result does not depend on the thread count. */
struct decode_job {
    const int16_t* trellis;
    int64_t kt, nt;
    int K, cb, exact, stride, first;
    double* w;
};

static void* decode_rows(void* arg) {
    const struct decode_job* j = (const struct decode_job*) arg;
    const int64_t cols = j->nt * 16;
    for (int64_t a = j->first; a < j->kt; a += j->stride)
        for (int64_t b = 0; b < j->nt; ++b) {
            const uint16_t* tile = (const uint16_t*) (j->trellis + (a * j->nt + b) * 16 * j->K);
            for (int t = 0; t < 256; ++t) {
                int k, n;
                tile_position(t, &k, &n);
                const uint32_t win = exo_window(tile, j->K, t);
                j->w[(a * 16 + k) * cols + b * 16 + n] =
                    j->exact ? exo_codebook_exact(win, j->cb) : (double) exo_half_to_float(exo_codebook(win, j->cb, 0));
            }
        }
    return NULL;
}

static int oracle_threads(int64_t rows) {
    long n = 0;
    const char* env = getenv("EXO_THREADS");
    if (env && *env) n = strtol(env, NULL, 10);
    if (n <= 0) n = sysconf(_SC_NPROCESSORS_ONLN);
    if (n < 1) n = 1;
    if (n > 64) n = 64;
    if (n > rows) n = (long) rows;
    return (int) n;
}

static double* decode_values(const int16_t* trellis, int64_t kt, int64_t nt, int K, int cb, int exact) {
    double* w = (double*) malloc(sizeof(double) * (size_t) (kt * 16 * nt * 16));
    const int nthr = oracle_threads(kt);
    struct decode_job jobs[64];
    pthread_t tids[64];
    int started[64] = {0};
    for (int i = 0; i < nthr; ++i) {
        jobs[i] = (struct decode_job) {trellis, kt, nt, K, cb, exact, nthr, i, w};
        if (i > 0) started[i] = pthread_create(&tids[i], NULL, decode_rows, &jobs[i]) == 0;
    }
    decode_rows(&jobs[0]);
    for (int i = 1; i < nthr; ++i) {
        if (started[i]) pthread_join(tids[i], NULL);
        else decode_rows(&jobs[i]);   /* no thread: do its rows here */
    }
    return w;
}

/* ---------------------------------------------------------------- hadamard */

static void fwht_float(float* v, int n) {
    for (int stride = 1; stride < n; stride <<= 1)
        for (int base = 0; base < n; base += stride << 1)
            for (int i = 0; i < stride; ++i) {
                const float a = v[base + i], b = v[base + stride + i];
                v[base + i] = a + b;
                v[base + stride + i] = a - b;
            }
}

static void fwht_double(double* v, int n) {
    for (int stride = 1; stride < n; stride <<= 1)
        for (int base = 0; base < n; base += stride << 1)
            for (int i = 0; i < stride; ++i) {
                const double a = v[base + i], b = v[base + stride + i];
                v[base + i] = a + b;
                v[base + stride + i] = a - b;
            }
}

static const float kNormF = 0.08838834764831845f;
static const double kNormD = 0.088388347648318440550; /* 1/sqrt(128) */

void exo_reconstruct(const uint16_t* wprime, const uint16_t* suh, const uint16_t* svh,
                     int64_t k, int64_t n, uint16_t* w) {
    float* m = (float*) malloc(sizeof(float) * (size_t) (k * n));
    float line[128];
    for (int64_t i = 0; i < k * n; ++i) m[i] = exo_half_to_float(wprime[i]);
    for (int64_t r0 = 0; r0 < k; r0 += 128)
        for (int64_t c0 = 0; c0 < n; c0 += 128) {
            for (int r = 0; r < 128; ++r) {
                for (int c = 0; c < 128; ++c) line[c] = m[(r0 + r) * n + c0 + c];
                fwht_float(line, 128);
                for (int c = 0; c < 128; ++c) m[(r0 + r) * n + c0 + c] = line[c] * kNormF;
            }
            for (int c = 0; c < 128; ++c) {
                for (int r = 0; r < 128; ++r) line[r] = m[(r0 + r) * n + c0 + c];
                fwht_float(line, 128);
                for (int r = 0; r < 128; ++r) {
                    const float value = line[r] * kNormF * exo_half_to_float(suh[r0 + r])
                                        * exo_half_to_float(svh[c0 + c]);
                    w[(r0 + r) * n + c0 + c] = exo_half_from_double((double) value);
                }
            }
        }
    free(m);
}

/* ---------------------------------------------------------------- GEMV form */

void exo_input_transform(const void* x, int x_dtype, int64_t R, int64_t k,
                         const uint16_t* suh, uint16_t* xh) {
    double line[128];
    for (int64_t r = 0; r < R; ++r)
        for (int64_t b = 0; b < k; b += 128) {
            for (int i = 0; i < 128; ++i) {
                const uint16_t v = load_as_half(x, x_dtype, r * k + b + i);
                /* fp16 product, as the kernels' __hmul2 (lna_moe_ticket.cu:133-135) */
                line[i] = exo_half_to_float(exo_half_from_double(
                    (double) exo_half_to_float(v) * (double) exo_half_to_float(suh[b + i])));
            }
            fwht_double(line, 128);
            for (int i = 0; i < 128; ++i) xh[r * k + b + i] = exo_half_from_double(line[i] * kNormD);
        }
}

/* y[R, n] = out_transform( xh[R, k] . W'[k, n] ), all in double. */
static void gemv_core(const uint16_t* xh, int64_t R, const double* wprime,
                      const uint16_t* svh, int64_t k, int64_t n, double* y) {
    for (int64_t r = 0; r < R; ++r) {
        double* yr = y + r * n;
        for (int64_t c = 0; c < n; ++c) yr[c] = 0.0;
        for (int64_t i = 0; i < k; ++i) {
            const double a = (double) exo_half_to_float(xh[r * k + i]);
            if (a == 0.0) continue;
            const double* wrow = wprime + i * n;
            for (int64_t c = 0; c < n; ++c) yr[c] += a * wrow[c];
        }
        for (int64_t b = 0; b < n; b += 128) {
            fwht_double(yr + b, 128);
            for (int i = 0; i < 128; ++i)
                yr[b + i] = yr[b + i] * kNormD * (double) exo_half_to_float(svh[b + i]);
        }
    }
}

void exo_gemv_ex(const void* x, int x_dtype, int64_t R, const int16_t* trellis,
                 const uint16_t* suh, const uint16_t* svh, int64_t k, int64_t n,
                 int K, int cb, int exact, double* y) {
    double* wp = decode_values(trellis, k / 16, n / 16, K, cb, exact);
    uint16_t* xh = (uint16_t*) malloc(sizeof(uint16_t) * (size_t) (R * k));
    exo_input_transform(x, x_dtype, R, k, suh, xh);
    gemv_core(xh, R, wp, svh, k, n, y);
    free(xh);
    free(wp);
}

void exo_gemv(const void* x, int x_dtype, int64_t R, const int16_t* trellis,
              const uint16_t* suh, const uint16_t* svh, int64_t k, int64_t n,
              int K, int cb, double* y) {
    exo_gemv_ex(x, x_dtype, R, trellis, suh, svh, k, n, K, cb, 0, y);
}

/* --------------------------------------------------------------------- MoE */

int64_t exo_moe_ex(const void* x, int x_dtype, int64_t T, int64_t H, int64_t I,
                   const int16_t* const* gt, const uint16_t* const* gsu, const uint16_t* const* gsv,
                   const int16_t* const* ut, const uint16_t* const* usu, const uint16_t* const* usv,
                   const int16_t* const* dt, const uint16_t* const* dsu, const uint16_t* const* dsv,
                   const int32_t* Ktab, int cb, int64_t E,
                   const int32_t* ids, const float* weights, int64_t topk,
                   double limit, int exact, double* out) {
    /* dc[r][slot] keeps each row's expert output per slot; duplicated
     * (expert,row) slots reuse the same computed pair. */
    double* dc = (double*) calloc((size_t) (T * topk * H), sizeof(double));
    int64_t pairs = 0;
    const int64_t L = H > I ? H : I;
    uint16_t* xh = (uint16_t*) malloc(sizeof(uint16_t) * (size_t) L);
    uint16_t* act = (uint16_t*) malloc(sizeof(uint16_t) * (size_t) I);
    double* g = (double*) malloc(sizeof(double) * (size_t) I);
    double* u = (double*) malloc(sizeof(double) * (size_t) I);
    double* d = (double*) malloc(sizeof(double) * (size_t) H);

    for (int64_t e = 0; e < E; ++e) {
        int used = 0;
        for (int64_t s = 0; s < T * topk; ++s) used |= ids[s] == e;
        if (!used) continue;
        const int K = Ktab[e];
        double* wg = decode_values(gt[e], H / 16, I / 16, K, cb, exact);
        double* wu = decode_values(ut[e], H / 16, I / 16, K, cb, exact);
        double* wd = decode_values(dt[e], I / 16, H / 16, K, cb, exact);
        for (int64_t r = 0; r < T; ++r) {
            int64_t first = -1;
            for (int64_t s = 0; s < topk; ++s)
                if (ids[r * topk + s] == e) { first = s; break; }
            if (first < 0) continue;
            ++pairs;
            const void* xrow = x_dtype == EXO_F32 ? (const void*) ((const float*) x + r * H)
                                                  : (const void*) ((const uint16_t*) x + r * H);
            exo_input_transform(xrow, x_dtype, 1, H, gsu[e], xh);
            gemv_core(xh, 1, wg, gsv[e], H, I, g);
            exo_input_transform(xrow, x_dtype, 1, H, usu[e], xh);
            gemv_core(xh, 1, wu, usv[e], H, I, u);
            for (int64_t i = 0; i < I; ++i) {
                double gv = g[i], uv = u[i];
                if (gv > limit) gv = limit;                 /* clamp BEFORE SiLU */
                if (uv < -limit) uv = -limit;
                if (uv > limit) uv = limit;
                act[i] = exo_half_from_double(gv / (1.0 + exp(-gv)) * uv);
            }
            exo_input_transform(act, EXO_F16, 1, I, dsu[e], xh);
            gemv_core(xh, 1, wd, dsv[e], I, H, d);
            for (int64_t s = 0; s < topk; ++s)
                if (ids[r * topk + s] == e) memcpy(dc + (r * topk + s) * H, d, sizeof(double) * (size_t) H);
        }
        free(wd); free(wu); free(wg);
    }
    for (int64_t r = 0; r < T; ++r) {
        double* o = out + r * H;
        for (int64_t c = 0; c < H; ++c) o[c] = 0.0;
        for (int64_t s = 0; s < topk; ++s) {
            const int32_t id = ids[r * topk + s];
            if (id < 0 || id >= E) continue;
            const double wv = (double) weights[r * topk + s];
            const double* src = dc + (r * topk + s) * H;
            for (int64_t c = 0; c < H; ++c) o[c] += wv * src[c];
        }
    }
    free(d); free(u); free(g); free(act); free(xh); free(dc);
    return pairs;
}

int64_t exo_moe(const void* x, int x_dtype, int64_t T, int64_t H, int64_t I,
                const int16_t* const* gt, const uint16_t* const* gsu, const uint16_t* const* gsv,
                const int16_t* const* ut, const uint16_t* const* usu, const uint16_t* const* usv,
                const int16_t* const* dt, const uint16_t* const* dsu, const uint16_t* const* dsv,
                const int32_t* Ktab, int cb, int64_t E,
                const int32_t* ids, const float* weights, int64_t topk,
                double limit, double* out) {
    return exo_moe_ex(x, x_dtype, T, H, I, gt, gsu, gsv, ut, usu, usv, dt, dsu, dsv, Ktab, cb, E,
                      ids, weights, topk, limit, 0, out);
}
