/*
 * beacon_oracle.c -- CPU oracle for the beacon transformer hot path.
 * TEST INFRASTRUCTURE ONLY (the checker, never the product); see beacon_oracle.h
 * for what each function restates and the parity status.
 */
#include "beacon_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------- */
/* deterministic inputs                                                      */
/* ------------------------------------------------------------------------- */

uint64_t bo_splitmix64(uint64_t seed, uint64_t i) {
    uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

static inline double top24(uint64_t r) { return (double)(r >> 40); }

void bo_fill_uniform(float* out, size_t n, float lo, float hi, uint64_t seed, uint64_t offset) {
    const double span = (double)hi - (double)lo;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) {
        double u = top24(bo_splitmix64(seed, offset + (uint64_t)i)) / 16777216.0;
        out[i] = (float)((double)lo + span * u);
    }
}

void bo_fill_normal(float* out, size_t n, float mean, float std, uint64_t seed, uint64_t offset) {
    const double two_pi = 6.283185307179586476925286766559;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) {
        uint64_t g = offset + (uint64_t)i;   /* global element index */
        uint64_t p = g >> 1;                 /* Box-Muller pair      */
        double u1 = (top24(bo_splitmix64(seed, 2 * p)) + 1.0) / 16777216.0;
        double u2 = top24(bo_splitmix64(seed, 2 * p + 1)) / 16777216.0;
        double r = sqrt(-2.0 * log(u1));
        double z = (g & 1) ? r * sin(two_pi * u2) : r * cos(two_pi * u2);
        out[i] = (float)((double)mean + (double)std * z);
    }
}

/* ------------------------------------------------------------------------- */
/* dtype codecs: crates/beacon-core/src/dtype.rs                             */
/* ------------------------------------------------------------------------- */

static inline uint32_t f2u(float x) { uint32_t u; memcpy(&u, &x, 4); return u; }
static inline float u2f(uint32_t u) { float x; memcpy(&x, &u, 4); return x; }

/* dtype.rs:58-66: NaN keeps its top half with the quiet bit set; everything else
 * rounds to nearest even by adding 0x7fff + lsb and truncating. */
uint16_t bo_bf16_from_f32(float x) {
    uint32_t bits = f2u(x);
    if ((bits & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((bits >> 16) | 0x0040u);
    uint32_t bias = 0x7fffu + ((bits >> 16) & 1u);
    return (uint16_t)((bits + bias) >> 16);
}

float bo_bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

/* dtype.rs:197-209: ties are detected with an f32::EPSILON window and go to
 * the even neighbour; everything else rounds half away from zero (Rust round). */
static float round_half_even_ref(float x) {
    float r = roundf(x);
    if (fabsf(x - floorf(x) - 0.5f) < FLT_EPSILON) {
        float down = floorf(x);
        return (((int64_t)down) % 2 == 0) ? down : down + 1.0f;
    }
    return r;
}

/* dtype.rs:138-161 */
float bo_fp8e4m3_to_f32(uint8_t b) {
    float sign = (b & 0x80) ? -1.0f : 1.0f;
    int exp = (b >> 3) & 0x0f;
    int mant = b & 0x07;
    if (exp == 0x0f && mant == 0x07) return NAN;
    if (exp == 0) return sign * (float)mant * ldexpf(1.0f, 1 - 7 - 3);
    float frac = 1.0f + (float)mant / 8.0f;
    return sign * frac * ldexpf(1.0f, exp - 7);
}

/* dtype.rs:163-195 */
uint8_t bo_fp8e4m3_from_f32(float x) {
    if (isnan(x)) return 0xff;
    uint8_t sign_bit = signbit(x) ? 0x80 : 0x00;
    float ax = fabsf(x);
    if (ax == 0.0f) return sign_bit;
    if (ax >= 448.0f) return (uint8_t)(sign_bit | 0x7e);
    float min_normal = ldexpf(1.0f, 1 - 7);
    if (ax < min_normal) {
        float scale = ldexpf(1.0f, 1 - 7 - 3);
        float q = ax / scale;
        float m = round_half_even_ref(q);
        if (m > 7.0f) m = 7.0f;
        return (uint8_t)(sign_bit | (uint8_t)m);
    }
    int exp = (int)floorf(log2f(ax));
    if (exp < 1 - 7) exp = 1 - 7;
    float frac = ax / ldexpf(1.0f, exp) - 1.0f;
    int mant = (int)round_half_even_ref(frac * 8.0f);
    int biased = exp + 7;
    if (mant == 8) { mant = 0; biased += 1; }
    if (biased >= 0x0f && mant >= 0x07) return (uint8_t)(sign_bit | 0x7e);
    return (uint8_t)(sign_bit | (uint8_t)(biased << 3) | (uint8_t)mant);
}

void bo_f32_to_bf16(uint16_t* dst, const float* src, size_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) dst[i] = bo_bf16_from_f32(src[i]);
}

void bo_bf16_to_f32_n(float* dst, const uint16_t* src, size_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) dst[i] = bo_bf16_to_f32(src[i]);
}

void bo_round_bf16_inplace(float* x, size_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) x[i] = bo_bf16_to_f32(bo_bf16_from_f32(x[i]));
}

void bo_f32_to_fp8e4m3(uint8_t* dst, const float* src, size_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) dst[i] = bo_fp8e4m3_from_f32(src[i]);
}

void bo_fp8e4m3_to_f32_n(float* dst, const uint8_t* src, size_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) dst[i] = bo_fp8e4m3_to_f32(src[i]);
}

/* ------------------------------------------------------------------------- */
/* GEMM family                                                               */
/* ------------------------------------------------------------------------- */

/* C[M,N] = A[M,K] . B[K,N] with double accumulation (row-major). */
static void gemm_nn(float* C, const float* A, const float* Bm, int64_t M, int64_t K, int64_t N) {
#pragma omp parallel
    {
        double* acc = (double*)malloc(sizeof(double) * (size_t)(N > 0 ? N : 1));
#pragma omp for schedule(static)
        for (int64_t i = 0; i < M; ++i) {
            for (int64_t j = 0; j < N; ++j) acc[j] = 0.0;
            for (int64_t k = 0; k < K; ++k) {
                const double a = A[i * K + k];
                const float* brow = Bm + k * N;
                for (int64_t j = 0; j < N; ++j) acc[j] += a * (double)brow[j];
            }
            for (int64_t j = 0; j < N; ++j) C[i * N + j] = (float)acc[j];
        }
        free(acc);
    }
}

/* C[M,N] = A[M,K] . B[N,K]^T */
static void gemm_nt(float* C, const float* A, const float* Bm, int64_t M, int64_t K, int64_t N) {
#pragma omp parallel for schedule(static) collapse(2)
    for (int64_t i = 0; i < M; ++i)
        for (int64_t j = 0; j < N; ++j) {
            double acc = 0.0;
            const float* a = A + i * K;
            const float* b = Bm + j * K;
            for (int64_t k = 0; k < K; ++k) acc += (double)a[k] * (double)b[k];
            C[i * N + j] = (float)acc;
        }
}

/* C[K,N] = A[M,K]^T . B[M,N] */
static void gemm_tn(float* C, const float* A, const float* Bm, int64_t M, int64_t K, int64_t N) {
#pragma omp parallel
    {
        double* acc = (double*)malloc(sizeof(double) * (size_t)(N > 0 ? N : 1));
#pragma omp for schedule(static)
        for (int64_t r = 0; r < K; ++r) {
            for (int64_t j = 0; j < N; ++j) acc[j] = 0.0;
            for (int64_t i = 0; i < M; ++i) {
                const double a = A[i * K + r];
                const float* brow = Bm + i * N;
                for (int64_t j = 0; j < N; ++j) acc[j] += a * (double)brow[j];
            }
            for (int64_t j = 0; j < N; ++j) C[r * N + j] = (float)acc[j];
        }
        free(acc);
    }
}

void bo_matmul_fwd(float* out, const float* lhs, const float* rhs, int64_t M, int64_t K, int64_t N) {
    gemm_nn(out, lhs, rhs, M, K, N);
}

void bo_matmul_bwd(float* dlhs, float* drhs, const float* dout, const float* lhs, const float* rhs,
                   int64_t M, int64_t K, int64_t N) {
    if (dlhs) gemm_nt(dlhs, dout, rhs, M, N, K);  /* [M,N] . [K,N]^T */
    if (drhs) gemm_tn(drhs, lhs, dout, M, K, N);  /* [M,K]^T . [M,N] */
}

void bo_linear_fwd(float* out, const float* x, const float* w, const float* bias,
                   int64_t M, int64_t K, int64_t N) {
    gemm_nn(out, x, w, M, K, N);
    if (bias) {
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < M; ++i)
            for (int64_t j = 0; j < N; ++j) out[i * N + j] = (float)((double)out[i * N + j] + (double)bias[j]);
    }
}

void bo_linear_bwd(float* dx, float* dw, float* db, const float* dy, const float* x, const float* w,
                   int64_t M, int64_t K, int64_t N) {
    bo_matmul_bwd(dx, dw, dy, x, w, M, K, N);
    if (db) {
#pragma omp parallel for schedule(static)
        for (int64_t j = 0; j < N; ++j) {
            double s = 0.0;
            for (int64_t i = 0; i < M; ++i) s += (double)dy[i * N + j];
            db[j] = (float)s;
        }
    }
}

/* ------------------------------------------------------------------------- */
/* attention                                                                 */
/* ------------------------------------------------------------------------- */

static void attn_fwd_head(float* out, float* lse, const float* q, const float* k, const float* v,
                          int64_t S, int64_t D, int causal, double scale, double* s) {
    for (int64_t i = 0; i < S; ++i) {
        const float* qi = q + i * D;
        const int64_t jend = causal ? i + 1 : S;
        double m = -INFINITY;
        for (int64_t j = 0; j < jend; ++j) {
            const float* kj = k + j * D;
            double acc = 0.0;
            for (int64_t d = 0; d < D; ++d) acc += (double)qi[d] * (double)kj[d];
            s[j] = acc * scale;
            if (s[j] > m) m = s[j];
        }
        double l = 0.0;
        for (int64_t j = 0; j < jend; ++j) { s[j] = exp(s[j] - m); l += s[j]; }
        double* o = s + S;  /* D doubles of scratch after the score row */
        for (int64_t d = 0; d < D; ++d) o[d] = 0.0;
        for (int64_t j = 0; j < jend; ++j) {
            const float* vj = v + j * D;
            const double p = s[j];
            for (int64_t d = 0; d < D; ++d) o[d] += p * (double)vj[d];
        }
        for (int64_t d = 0; d < D; ++d) out[i * D + d] = (float)(o[d] / l);
        lse[i] = (float)(m + log(l));
    }
}

static inline double attn_scale(float scale, int64_t D) {
    return scale > 0.0f ? (double)scale : 1.0 / sqrt((double)D);
}

void bo_attention_fwd_heads(float* out, float* lse, const float* q, const float* k, const float* v,
                            int64_t B, int64_t Hq, int64_t Hkv, int64_t S, int64_t D, int causal,
                            float scale, const int64_t* heads, int64_t nheads) {
    (void)B;
    const double sc = attn_scale(scale, D);
    const int64_t group = Hq / Hkv;
#pragma omp parallel
    {
        double* s = (double*)malloc(sizeof(double) * (size_t)(S + D));
#pragma omp for schedule(dynamic, 1)
        for (int64_t t = 0; t < nheads; ++t) {
            const int64_t bh = heads[t];
            const int64_t b = bh / Hq, h = bh % Hq;
            const int64_t kvh = b * Hkv + h / group;
            attn_fwd_head(out + bh * S * D, lse + bh * S, q + bh * S * D, k + kvh * S * D,
                          v + kvh * S * D, S, D, causal, sc, s);
        }
        free(s);
    }
}

void bo_attention_fwd(float* out, float* lse, const float* q, const float* k, const float* v,
                      int64_t B, int64_t Hq, int64_t Hkv, int64_t S, int64_t D, int causal, float scale) {
    int64_t n = B * Hq;
    int64_t* heads = (int64_t*)malloc(sizeof(int64_t) * (size_t)(n > 0 ? n : 1));
    for (int64_t i = 0; i < n; ++i) heads[i] = i;
    bo_attention_fwd_heads(out, lse, q, k, v, B, Hq, Hkv, S, D, causal, scale, heads, n);
    free(heads);
}

/* Backward of one query head into double accumulators dk/dv of its KV head.
 * P = exp(scale q.k - lse), dV += P^T dO, dP = dO V^T, Dterm = rowsum(P * dP),
 * dS = P (dP - Dterm), dQ = scale dS K, dK += scale dS^T Q. */
static void attn_bwd_head(float* dq, double* dk, double* dv, const float* dout, const float* q,
                          const float* k, const float* v, const float* lse, int64_t S, int64_t D,
                          int causal, double scale, double* p, double* dp) {
    for (int64_t i = 0; i < S; ++i) {
        const float* qi = q + i * D;
        const float* doi = dout + i * D;
        const int64_t jend = causal ? i + 1 : S;
        double dterm = 0.0;
        for (int64_t j = 0; j < jend; ++j) {
            const float* kj = k + j * D;
            const float* vj = v + j * D;
            double acc = 0.0, accp = 0.0;
            for (int64_t d = 0; d < D; ++d) {
                acc += (double)qi[d] * (double)kj[d];
                accp += (double)doi[d] * (double)vj[d];
            }
            p[j] = exp(acc * scale - (double)lse[i]);
            dp[j] = accp;
            dterm += p[j] * dp[j];
        }
        double* dqi = p + S;  /* D doubles of scratch */
        for (int64_t d = 0; d < D; ++d) dqi[d] = 0.0;
        for (int64_t j = 0; j < jend; ++j) {
            const double ds = p[j] * (dp[j] - dterm);
            const float* kj = k + j * D;
            double* dkj = dk + j * D;
            double* dvj = dv + j * D;
            for (int64_t d = 0; d < D; ++d) {
                dqi[d] += ds * (double)kj[d];
                dkj[d] += scale * ds * (double)qi[d];
                dvj[d] += p[j] * (double)doi[d];
            }
        }
        for (int64_t d = 0; d < D; ++d) dq[i * D + d] = (float)(scale * dqi[d]);
    }
}

void bo_attention_bwd(float* dq, float* dk, float* dv, const float* dout,
                      const float* q, const float* k, const float* v, const float* lse,
                      int64_t B, int64_t Hq, int64_t Hkv, int64_t S, int64_t D, int causal, float scale) {
    const double sc = attn_scale(scale, D);
    const int64_t group = Hq / Hkv;
    /* one task per KV head: its query heads run serially so dk/dv need no locks */
#pragma omp parallel
    {
        double* p = (double*)malloc(sizeof(double) * (size_t)(S + D));
        double* dp = (double*)malloc(sizeof(double) * (size_t)S);
        double* dkacc = (double*)malloc(sizeof(double) * (size_t)(S * D));
        double* dvacc = (double*)malloc(sizeof(double) * (size_t)(S * D));
#pragma omp for schedule(dynamic, 1)
        for (int64_t kvh = 0; kvh < B * Hkv; ++kvh) {
            const int64_t b = kvh / Hkv, hk = kvh % Hkv;
            memset(dkacc, 0, sizeof(double) * (size_t)(S * D));
            memset(dvacc, 0, sizeof(double) * (size_t)(S * D));
            for (int64_t g = 0; g < group; ++g) {
                const int64_t bh = b * Hq + hk * group + g;
                attn_bwd_head(dq + bh * S * D, dkacc, dvacc, dout + bh * S * D, q + bh * S * D,
                              k + kvh * S * D, v + kvh * S * D, lse + bh * S, S, D, causal, sc, p, dp);
            }
            for (int64_t e = 0; e < S * D; ++e) {
                dk[kvh * S * D + e] = (float)dkacc[e];
                dv[kvh * S * D + e] = (float)dvacc[e];
            }
        }
        free(p); free(dp); free(dkacc); free(dvacc);
    }
}

void bo_attention_fwd_rows(float* out, float* lse, const float* q, const float* k, const float* v,
                           int64_t S, int64_t D, int causal, float scale, const int64_t* rows, int64_t nrows) {
    const double sc = attn_scale(scale, D);
#pragma omp parallel
    {
        double* s = (double*)malloc(sizeof(double) * (size_t)(S + D));
#pragma omp for schedule(dynamic, 1)
        for (int64_t t = 0; t < nrows; ++t) {
            const int64_t i = rows[t];
            const int64_t jend = causal ? i + 1 : S;
            const float* qi = q + i * D;
            double m = -INFINITY;
            for (int64_t j = 0; j < jend; ++j) {
                const float* kj = k + j * D;
                double acc = 0.0;
                for (int64_t d = 0; d < D; ++d) acc += (double)qi[d] * (double)kj[d];
                s[j] = acc * sc;
                if (s[j] > m) m = s[j];
            }
            double l = 0.0;
            for (int64_t j = 0; j < jend; ++j) { s[j] = exp(s[j] - m); l += s[j]; }
            double* o = s + S;
            for (int64_t d = 0; d < D; ++d) o[d] = 0.0;
            for (int64_t j = 0; j < jend; ++j)
                for (int64_t d = 0; d < D; ++d) o[d] += s[j] * (double)v[j * D + d];
            for (int64_t d = 0; d < D; ++d) out[t * D + d] = (float)(o[d] / l);
            lse[t] = (float)(m + log(l));
        }
        free(s);
    }
}

void bo_attention_bwd_head(float* dq, float* dk, float* dv, const float* dout, const float* q,
                           const float* k, const float* v, const float* lse, int64_t S, int64_t D, int causal,
                           float scale) {
    const double sc = attn_scale(scale, D);
    double* dks = (double*)calloc((size_t)(S * D), sizeof(double));
    double* dvs = (double*)calloc((size_t)(S * D), sizeof(double));
#pragma omp parallel
    {
        double* p = (double*)malloc(sizeof(double) * (size_t)(S + D));
        double* dp = (double*)malloc(sizeof(double) * (size_t)S);
        double* dka = (double*)calloc((size_t)(S * D), sizeof(double));
        double* dva = (double*)calloc((size_t)(S * D), sizeof(double));
        /* one query row at a time: attn_bwd_head's arithmetic for rows [i, i+1) */
#pragma omp for schedule(dynamic, 16)
        for (int64_t i = 0; i < S; ++i) {
            const float* qi = q + i * D;
            const float* doi = dout + i * D;
            const int64_t jend = causal ? i + 1 : S;
            double dterm = 0.0;
            for (int64_t j = 0; j < jend; ++j) {
                double acc = 0.0, accp = 0.0;
                for (int64_t d = 0; d < D; ++d) {
                    acc += (double)qi[d] * (double)k[j * D + d];
                    accp += (double)doi[d] * (double)v[j * D + d];
                }
                p[j] = exp(acc * sc - (double)lse[i]);
                dp[j] = accp;
                dterm += p[j] * dp[j];
            }
            double* dqi = p + S;
            for (int64_t d = 0; d < D; ++d) dqi[d] = 0.0;
            for (int64_t j = 0; j < jend; ++j) {
                const double ds = p[j] * (dp[j] - dterm);
                for (int64_t d = 0; d < D; ++d) {
                    dqi[d] += ds * (double)k[j * D + d];
                    dka[j * D + d] += sc * ds * (double)qi[d];
                    dva[j * D + d] += p[j] * (double)doi[d];
                }
            }
            for (int64_t d = 0; d < D; ++d) dq[i * D + d] = (float)(sc * dqi[d]);
        }
#pragma omp critical
        {
            for (int64_t e = 0; e < S * D; ++e) {
                dks[e] += dka[e];
                dvs[e] += dva[e];
            }
        }
        free(p); free(dp); free(dka); free(dva);
    }
    for (int64_t e = 0; e < S * D; ++e) {
        dk[e] = (float)dks[e];
        dv[e] = (float)dvs[e];
    }
    free(dks); free(dvs);
}

/* ------------------------------------------------------------------------- */
/* RMSNorm                                                                   */
/* ------------------------------------------------------------------------- */

void bo_rmsnorm_fwd(float* y, float* rms, const float* x, const float* g, int64_t T, int64_t dim, float eps) {
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < T; ++t) {
        const float* xt = x + t * dim;
        double ss = 0.0;
        for (int64_t d = 0; d < dim; ++d) ss += (double)xt[d] * (double)xt[d];
        const double r = sqrt(ss / (double)dim + (double)eps);
        rms[t] = (float)r;
        for (int64_t d = 0; d < dim; ++d) y[t * dim + d] = (float)((double)xt[d] * (double)g[d] / r);
    }
}

void bo_rmsnorm_bwd(float* dx, float* dg, const float* dy, const float* x, const float* rms,
                    const float* g, int64_t T, int64_t dim) {
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < T; ++t) {
        const float* xt = x + t * dim;
        const float* dyt = dy + t * dim;
        const double r = (double)rms[t];
        double dot = 0.0;
        for (int64_t d = 0; d < dim; ++d) dot += (double)g[d] * (double)dyt[d] * (double)xt[d];
        const double c = dot / ((double)dim * r * r * r);
        for (int64_t d = 0; d < dim; ++d)
            dx[t * dim + d] = (float)((double)g[d] * (double)dyt[d] / r - (double)xt[d] * c);
    }
    if (dg) {
#pragma omp parallel for schedule(static)
        for (int64_t d = 0; d < dim; ++d) {
            double s = 0.0;
            for (int64_t t = 0; t < T; ++t) s += (double)dy[t * dim + d] * (double)x[t * dim + d] / (double)rms[t];
            dg[d] = (float)s;
        }
    }
}

/* ------------------------------------------------------------------------- */
/* LayerNorm                                                                 */
/* ------------------------------------------------------------------------- */

void bo_layernorm_fwd(float* y, float* mean, float* invstd, const float* x, const float* g, const float* b,
                      int64_t T, int64_t dim, float eps) {
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < T; ++t) {
        const float* xt = x + t * dim;
        double s = 0.0;
        for (int64_t d = 0; d < dim; ++d) s += (double)xt[d];
        const double mu = s / (double)dim;
        double ss = 0.0;
        for (int64_t d = 0; d < dim; ++d) ss += ((double)xt[d] - mu) * ((double)xt[d] - mu);
        const double is = 1.0 / sqrt(ss / (double)dim + (double)eps);
        mean[t] = (float)mu;
        invstd[t] = (float)is;
        for (int64_t d = 0; d < dim; ++d)
            y[t * dim + d] = (float)(((double)xt[d] - mu) * is * (double)g[d] + (double)b[d]);
    }
}

void bo_layernorm_bwd(float* dx, float* dg, float* db, const float* dy, const float* x, const float* mean,
                      const float* invstd, const float* g, int64_t T, int64_t dim) {
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < T; ++t) {
        const float* xt = x + t * dim;
        const float* dyt = dy + t * dim;
        const double mu = (double)mean[t], is = (double)invstd[t];
        double sg = 0.0, sgx = 0.0;
        for (int64_t d = 0; d < dim; ++d) {
            const double gd = (double)g[d] * (double)dyt[d];
            sg += gd;
            sgx += gd * ((double)xt[d] - mu) * is;
        }
        const double mg = sg / (double)dim, mgx = sgx / (double)dim;
        for (int64_t d = 0; d < dim; ++d) {
            const double xh = ((double)xt[d] - mu) * is;
            dx[t * dim + d] = (float)(is * ((double)g[d] * (double)dyt[d] - mg - xh * mgx));
        }
    }
    if (dg || db) {
#pragma omp parallel for schedule(static)
        for (int64_t d = 0; d < dim; ++d) {
            double sw = 0.0, sb = 0.0;
            for (int64_t t = 0; t < T; ++t) {
                const double e = (double)dy[t * dim + d];
                sw += e * ((double)x[t * dim + d] - (double)mean[t]) * (double)invstd[t];
                sb += e;
            }
            if (dg) dg[d] = (float)sw;
            if (db) db[d] = (float)sb;
        }
    }
}

/* ------------------------------------------------------------------------- */
/* SwiGLU MLP                                                                */
/* ------------------------------------------------------------------------- */

static inline double silu(double z) { return z / (1.0 + exp(-z)); }

void bo_swiglu_fwd(float* out, const float* x, const float* wg, const float* wu, const float* wd,
                   int64_t T, int64_t dm, int64_t F) {
    float* gate = (float*)malloc(sizeof(float) * (size_t)(T * F));
    float* up = (float*)malloc(sizeof(float) * (size_t)(T * F));
    gemm_nn(gate, x, wg, T, dm, F);
    gemm_nn(up, x, wu, T, dm, F);
#pragma omp parallel for schedule(static)
    for (int64_t e = 0; e < T * F; ++e) gate[e] = (float)(silu((double)gate[e]) * (double)up[e]);
    gemm_nn(out, gate, wd, T, F, dm);
    free(gate);
    free(up);
}

void bo_swiglu_bwd(float* dx, float* dwg, float* dwu, float* dwd, const float* dy, const float* x,
                   const float* wg, const float* wu, const float* wd, int64_t T, int64_t dm, int64_t F) {
    const size_t tf = (size_t)(T * F);
    float* gate = (float*)malloc(sizeof(float) * tf);
    float* up = (float*)malloc(sizeof(float) * tf);
    float* h = (float*)malloc(sizeof(float) * tf);
    float* dh = (float*)malloc(sizeof(float) * tf);
    gemm_nn(gate, x, wg, T, dm, F);
    gemm_nn(up, x, wu, T, dm, F);
#pragma omp parallel for schedule(static)
    for (int64_t e = 0; e < T * F; ++e) h[e] = (float)(silu((double)gate[e]) * (double)up[e]);
    gemm_tn(dwd, h, dy, T, F, dm);      /* dWd = h^T dy     */
    gemm_nt(dh, dy, wd, T, dm, F);      /* dh  = dy Wd^T    */
#pragma omp parallel for schedule(static)
    for (int64_t e = 0; e < T * F; ++e) {
        const double z = gate[e];
        const double sg = 1.0 / (1.0 + exp(-z));
        const double dhe = dh[e];
        const double dup = dhe * z * sg;                       /* d(up)   */
        const double dgate = dhe * (double)up[e] * sg * (1.0 + z * (1.0 - sg));  /* d(gate) */
        gate[e] = (float)dgate;
        up[e] = (float)dup;
    }
    gemm_tn(dwg, x, gate, T, dm, F);    /* dWg = x^T dgate */
    gemm_tn(dwu, x, up, T, dm, F);      /* dWu = x^T dup   */
    /* dx = dgate Wg^T + dup Wu^T */
    float* tmp = (float*)malloc(sizeof(float) * (size_t)(T * dm));
    gemm_nt(dx, gate, wg, T, F, dm);
    gemm_nt(tmp, up, wu, T, F, dm);
#pragma omp parallel for schedule(static)
    for (int64_t e = 0; e < T * dm; ++e) dx[e] = (float)((double)dx[e] + (double)tmp[e]);
    free(tmp); free(gate); free(up); free(h); free(dh);
}

/* ------------------------------------------------------------------------- */
/* residual add                                                              */
/* ------------------------------------------------------------------------- */

void bo_residual_add_fwd(float* out, const float* a, const float* b, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) out[i] = a[i] + b[i];
}

void bo_residual_add_bwd(float* da, float* db, const float* dout, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) { da[i] = dout[i]; db[i] = dout[i]; }
}

int bo_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void bo_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
