/*
 * vela oracle -- CPU restatement of the reference's exact-integer UNet step.
 * TEST INFRASTRUCTURE ONLY (the checker and the timed CPU baseline); see
 * vela_oracle.h.  Reference citations are file:line in emanwrxsti/vela.
 */
#include "vela_oracle.h"
#include <stdlib.h>
#include <string.h>
#include <stdio.h>
#include <limits.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define I64(x) ((int64_t)(x))

static int g_threads = 0;
void or_set_threads(int n) { g_threads = n; }
int or_get_threads(void) {
#ifdef _OPENMP
    return g_threads > 0 ? g_threads : omp_get_max_threads();
#else
    return 1;
#endif
}
#define NT or_get_threads()

/* ======================================================================
 * primitives -- src/intops.cuh:9-66
 * ==================================================================== */
int64_t or_sat32(int64_t v) { return v < INT32_MIN ? INT32_MIN : (v > INT32_MAX ? INT32_MAX : v); }

/* src/intops.cuh:11-17: rounding (half up) right shift for s >= 0, clamped
 * saturating left shift for s < 0; the result saturates to int32. */
int64_t or_rshr(int64_t v, int64_t s) {
    if (s >= 0) {
        int p = s > 62 ? 62 : (int)s;
        return or_sat32((v + ((I64(1) << p) >> 1)) >> p);
    }
    int neg = -s > 31 ? 31 : (int)(-s);
    int64_t lim = I64(1) << (62 - neg);
    int64_t r = v < -lim ? -lim : (v > lim ? lim : v);
    return or_sat32(r * (I64(1) << neg));
}
/* src/intops.cuh:18 */
int64_t or_floor_div(int64_t a, int64_t b) {
    int64_t q = a / b;
    if ((a % b != 0) && ((a < 0) != (b < 0))) --q;
    return q;
}
/* src/intops.cuh:38: number of k in [15, 32) with m >= 2^k */
int or_row_exp(int64_t m) {
    int e = 0;
    for (int k = 15; k < 32; ++k) e += (m >= (I64(1) << k));
    return e;
}
/* src/intops.cuh:39 */
int64_t or_quant16(int64_t v, int e) {
    int64_t q = or_rshr(v, e);
    return q < -32767 ? -32767 : (q > 32767 ? 32767 : q);
}
/* src/intops.cuh:43-50: 2049-entry Q16 table over [-16, 16), 10-bit linear interpolation */
int32_t or_lut16(int64_t x, const int32_t* L) {
    int64_t z = x + (I64(16) << 16);
    if (z < 0) return 0;
    if (z >= (I64(32) << 16)) return 65536;
    int i = (int)(z >> 10), f = (int)(z & 1023);
    int a = L[i], b = L[i + 1];
    return a + (((b - a) * f) >> 10);
}
/* src/intops.cuh:51-56 computes floor(sqrt(v)) (fp64 seed + integer fix-up);
 * restated as the exact digit-by-digit integer square root. */
int64_t or_isqrt(int64_t v) {
    if (v <= 0) return 0;
    uint64_t op = (uint64_t)v, res = 0, one = UINT64_C(1) << 62;
    while (one > op) one >>= 2;
    while (one) {
        if (op >= res + one) { op -= res + one; res = (res >> 1) + one; }
        else res >>= 1;
        one >>= 2;
    }
    return (int64_t)res;
}
/* src/attn.cu:65-83 evaluates rshr(S, sh) of the exact 16-bit dot product;
 * pinned by src/test_attn_score.cu:28-30 to sat32 of that value. */
int32_t or_score(int64_t S, int sh) { return (int32_t)or_rshr(S, sh); }
void or_score_batch(const int64_t* S, const int32_t* sh, int32_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = or_score(S[i], sh[i]);
}

static inline uint32_t uabs32(int32_t v) { return v < 0 ? (uint32_t)(-(int64_t)v) : (uint32_t)v; }
static inline int32_t clamp16(int64_t q) { return (int32_t)(q < -32767 ? -32767 : (q > 32767 ? 32767 : q)); }
/* 16-bit split, src/intops.cuh:65-66: q = 256*hi + lo + 128 */
static inline void split16(int64_t q, int8_t* hi, int8_t* lo) { *hi = (int8_t)(q >> 8); *lo = (int8_t)((q & 255) - 128); }
/* product that wraps like the device's 64-bit multiply */
static inline int64_t mulw(int64_t a, int64_t b) { return (int64_t)((uint64_t)a * (uint64_t)b); }
/* GEMM epilogue, src/gemm_hl.cu:40-43 / src/kernels.cu:36-39 */
static inline int32_t epi1(int64_t acc, const int32_t* c, int er) {
    return (int32_t)or_sat32(or_rshr(mulw(acc, c[0]), (int64_t)c[1] - er) + c[2]);
}
/* SiLU/GELU style LUT activation: sat32(rshr(x * lut(x), 16)), src/kernels.cu:537 */
static inline int32_t lutact(int64_t x, const int32_t* L) { return (int32_t)or_sat32(or_rshr(x * or_lut16(x, L), 16)); }

/* ======================================================================
 * row quantisation -- src/kernels.cu:42-57
 * ==================================================================== */
void or_quant_rows(const int32_t* X, int M, int K, int ldx, int8_t* hi, int8_t* lo, int32_t* e, int Kp, int Mpad) {
    #pragma omp parallel for num_threads(NT)
    for (int r = 0; r < Mpad; ++r) {
        int8_t* h = hi + (size_t)r * Kp; int8_t* l = lo + (size_t)r * Kp;
        if (r >= M) { for (int k = 0; k < Kp; ++k) { h[k] = 0; l[k] = -128; } continue; }
        const int32_t* x = X + (size_t)r * ldx;
        uint32_t m = 0;
        for (int k = 0; k < K; ++k) { uint32_t a = uabs32(x[k]); if (a > m) m = a; }
        int ee = or_row_exp(m);
        e[r] = ee;
        for (int k = 0; k < Kp; ++k) split16(k < K ? or_quant16(x[k], ee) : 0, &h[k], &l[k]);
    }
}
void or_rowexp_u32(const uint32_t* rowmax, int M, int32_t* e) { for (int r = 0; r < M; ++r) e[r] = or_row_exp(rowmax[r]); }

/* ======================================================================
 * hi/lo GEMM + epilogues -- src/gemm_hl.cu:65-310 (semantics of
 * k_gemm_hl / k_gemm_hl2: Y = epi(256*Ahi.W + Alo.W + 128*wsum))
 * ==================================================================== */
void or_gemm_hl(const int8_t* Ahi, const int8_t* Alo, int lda, int Mreal,
                const int8_t* W, int ldw, int Nreal, int Kp,
                const int32_t* cst, const int32_t* e, const or_epi_t* E) {
    const int epi = E->epi;
    #pragma omp parallel for num_threads(NT) schedule(dynamic, 4)
    for (int r = 0; r < Mreal; ++r) {
        const int8_t* ah = Ahi + (size_t)r * lda; const int8_t* al = Alo + (size_t)r * lda;
        const int er = e[r];
        int32_t* yrow = (int32_t*)malloc(sizeof(int32_t) * (size_t)Nreal);
        for (int n = 0; n < Nreal; ++n) {
            const int8_t* w = W + (size_t)n * ldw;
            int64_t ch = 0, cl = 0;
            for (int k = 0; k < Kp; ++k) { ch += ah[k] * w[k]; cl += al[k] * w[k]; }
            const int32_t* c = cst + 4 * n;
            int64_t acc = 256 * ch + cl + 128 * I64(c[3]);
            yrow[n] = epi1(acc, c, er);
        }
        uint32_t mx = 0;
        if (epi == OR_EPI_PLAIN || epi == OR_EPI_GELU) {
            for (int n = 0; n < Nreal; ++n) {
                int64_t y = yrow[n];
                if (epi == OR_EPI_GELU) y = lutact(y, E->Lphi);
                if (E->residual) y = or_sat32(y + E->residual[(size_t)r * E->ldy + n]);
                E->Y[(size_t)r * E->ldy + n] = (int32_t)y;
                uint32_t a = uabs32((int32_t)y); if (a > mx) mx = a;
            }
        } else if (epi == OR_EPI_SPLIT3) {
            for (int n = 0; n < Nreal; ++n) {
                int part = n >= 2 * E->Cs ? 2 : (n >= E->Cs ? 1 : 0);
                int32_t* dst = part == 0 ? E->Y : (part == 1 ? E->Y1 : E->Y2);
                dst[(size_t)r * E->Cs + (n - part * E->Cs)] = yrow[n];
            }
        } else if (epi == OR_EPI_GEGLU) {   /* interleaved columns: 2c = a_c, 2c+1 = g_c (src/gemm_hl.cu:291-296) */
            for (int n = 0; n + 1 < Nreal; n += 2) {
                int64_t ge = lutact(yrow[n + 1], E->Lphi);
                int32_t v = (int32_t)or_sat32(or_rshr(I64(yrow[n]) * ge, 16));
                E->Y[(size_t)r * E->ldy + (n >> 1)] = v;
                uint32_t a = uabs32(v); if (a > mx) mx = a;
            }
        } else if (epi == OR_EPI_QKV) {     /* src/gemm_hl.cu:179-241 */
            const int C = E->C, b = r / E->T, t = r - b * E->T;
            for (int n0 = 0; n0 < Nreal; n0 += 64) {
                const int part = n0 / C, head = (n0 - part * C) >> 6;
                if (part == 2) {
                    for (int d = 0; d < 64; ++d) E->Y2[(size_t)r * C + head * 64 + d] = yrow[n0 + d];
                    continue;
                }
                uint32_t m = 0;
                for (int d = 0; d < 64; ++d) { uint32_t a = uabs32(yrow[n0 + d]); if (a > m) m = a; }
                const int ee = or_row_exp(m);
                const int Tp = part == 0 ? E->TpQ : E->TpK;
                const size_t gt = (size_t)(b * E->heads + head) * Tp + t;
                int8_t* hi = part == 0 ? E->qhi : E->khi; int8_t* lo = part == 0 ? E->qlo : E->klo;
                int64_t hs = 0, ls = 0, ts = 0;
                for (int d = 0; d < 64; ++d) {
                    int64_t q = or_quant16(yrow[n0 + d], ee);
                    int8_t h, l; split16(q, &h, &l);
                    hi[gt * 64 + d] = h; lo[gt * 64 + d] = l; hs += h; ls += l; ts += q;
                }
                (part == 0 ? E->qe : E->ke)[gt] = ee;
                (part == 0 ? E->qhs : E->khs)[gt] = hs;
                (part == 0 ? E->qls : E->kls)[gt] = ls;
                (part == 0 ? E->qts : E->kts)[gt] = ts;
            }
        }
        if (E->rowmax && (epi == OR_EPI_PLAIN || epi == OR_EPI_GELU || epi == OR_EPI_GEGLU) && mx > E->rowmax[r]) E->rowmax[r] = mx;
        free(yrow);
    }
}

/* ======================================================================
 * conv helpers -- src/kernels.cu:106-170, src/gemm_hl.cu:335-341
 * ==================================================================== */
void or_pixmax(const int32_t* X, int rows, int C, uint32_t* pm) {
    #pragma omp parallel for num_threads(NT)
    for (int r = 0; r < rows; ++r) {
        uint32_t m = 0; const int32_t* x = X + (size_t)r * C;
        for (int c = 0; c < C; ++c) { uint32_t a = uabs32(x[c]); if (a > m) m = a; }
        pm[r] = m;
    }
}
static uint32_t window_max(const uint32_t* pm, int b, int H, int W, int oy, int ox, int stride) {
    uint32_t m = 0;
    for (int ky = 0; ky < 3; ++ky) for (int kx = 0; kx < 3; ++kx) {
        int iy = oy * stride - 1 + ky, ix = ox * stride - 1 + kx;
        if (iy >= 0 && iy < H && ix >= 0 && ix < W) { uint32_t v = pm[((size_t)b * H + iy) * W + ix]; if (v > m) m = v; }
    }
    return m;
}
void or_conv_e(const uint32_t* pm, int B, int H, int W, int stride, int32_t* e) {
    const int Ho = (H - 1) / stride + 1, Wo = (W - 1) / stride + 1;
    for (int r = 0; r < B * Ho * Wo; ++r) {
        int b = r / (Ho * Wo), p = r % (Ho * Wo), oy = p / Wo, ox = p % Wo;
        e[r] = or_row_exp(window_max(pm, b, H, W, oy, ox, stride));
    }
}
void or_im2col3(const int32_t* X, const uint32_t* pm, int B, int H, int W, int C, int stride,
                int8_t* hi, int8_t* lo, int32_t* e, int Kp, int Mpad) {
    const int Ho = (H - 1) / stride + 1, Wo = (W - 1) / stride + 1, rows = B * Ho * Wo, K = 9 * C;
    #pragma omp parallel for num_threads(NT)
    for (int r = 0; r < Mpad; ++r) {
        int8_t* h = hi + (size_t)r * Kp; int8_t* l = lo + (size_t)r * Kp;
        if (r >= rows) { for (int k = 0; k < Kp; ++k) { h[k] = 0; l[k] = -128; } continue; }
        int b = r / (Ho * Wo), p = r % (Ho * Wo), oy = p / Wo, ox = p % Wo;
        int ee = or_row_exp(window_max(pm, b, H, W, oy, ox, stride));
        e[r] = ee;
        for (int tap = 0; tap < 9; ++tap) {
            int iy = oy * stride - 1 + tap / 3, ix = ox * stride - 1 + tap % 3;
            int in = iy >= 0 && iy < H && ix >= 0 && ix < W;
            const int32_t* xp = in ? X + (((size_t)b * H + iy) * W + ix) * C : NULL;
            for (int c = 0; c < C; ++c) split16(in ? or_quant16(xp[c], ee) : 0, &h[tap * C + c], &l[tap * C + c]);
        }
        for (int k = K; k < Kp; ++k) { h[k] = 0; l[k] = -128; }
    }
}

/* ======================================================================
 * GroupNorm / LayerNorm -- src/kernels.cu:173-212 (stats), :285-305 and
 * :420-487 (apply), :223-284 and :350-419 (LayerNorm)
 * ==================================================================== */
/* normalisation constants shared by GN and LN: src/kernels.cu:185-191,204-211 */
static void norm_finish(int64_t sum, int64_t mn, int64_t mx, int64_t n, int64_t* mean, int* e) {
    *mean = or_floor_div(sum + n / 2, n);
    int64_t m = (mx - *mean) > (*mean - mn) ? (mx - *mean) : (*mean - mn);
    int ee = or_row_exp(m) - 5;
    *e = ee < 0 ? 0 : ee;
}
static int64_t norm_sd(int64_t ss, int64_t n, int e, int64_t den) {
    int64_t var = or_floor_div(ss, n);
    int sh = 32 - 2 * e; int64_t one = sh >= 0 ? (I64(1) << sh) : 0;
    int64_t eps = or_floor_div(one + den / 2, den);
    return or_isqrt((var + eps) << 16);
}
/* y = floor((d * 2^(24-e) * 2 + sd) / (2 sd)); out = sat32(rshr(y*g, 16) + beta) */
static inline int64_t norm_apply(int64_t d, int e, int64_t sd, int64_t g, int64_t beta) {
    int64_t yy = or_floor_div(d * (I64(1) << (24 - e)) * 2 + sd, 2 * sd);
    return or_sat32(or_rshr(yy * g, 16) + beta);
}
void or_gn_stats(const int32_t* X, int B, int T, int C, int groups, int64_t den, or_gnstat_t* gs) {
    const int cg = C / groups; const int64_t n = I64(T) * cg;
    #pragma omp parallel for collapse(2) num_threads(NT)
    for (int b = 0; b < B; ++b) for (int g = 0; g < groups; ++g) {
        or_gnstat_t s; memset(&s, 0, sizeof(s));
        int64_t sum = 0; int32_t mn = INT32_MAX, mx = INT32_MIN;
        for (int t = 0; t < T; ++t) {
            const int32_t* x = X + ((size_t)b * T + t) * C + g * cg;
            for (int j = 0; j < cg; ++j) { int32_t v = x[j]; sum += v; if (v < mn) mn = v; if (v > mx) mx = v; }
        }
        int64_t mean; int e; norm_finish(sum, mn, mx, n, &mean, &e);
        int64_t ss = 0;
        for (int t = 0; t < T; ++t) {
            const int32_t* x = X + ((size_t)b * T + t) * C + g * cg;
            for (int j = 0; j < cg; ++j) { int64_t dd = or_rshr(I64(x[j]) - mean, e); ss += dd * dd; }
        }
        s.sum = sum; s.mn = mn; s.mx = mx; s.mean = mean; s.e = e; s.ss = ss; s.sd = norm_sd(ss, n, e, den);
        gs[b * groups + g] = s;
    }
}
/* quantised row output, src/kernels.cu:250-259 / 317-331 */
static void quant_row_out(const int32_t* v, int C, int8_t* h, int8_t* l, int32_t* e, int Kp) {
    uint32_t m = 0;
    for (int c = 0; c < C; ++c) { uint32_t a = uabs32(v[c]); if (a > m) m = a; }
    int ee = or_row_exp(m);
    *e = ee;
    for (int c = 0; c < Kp; ++c) split16(c < C ? or_quant16(v[c], ee) : 0, &h[c], &l[c]);
}
void or_gn_apply_row(const int32_t* X, int B, int T, int C, int groups, const or_gnstat_t* gs,
                     const int32_t* g, const int32_t* beta, const int32_t* Lsig,
                     int32_t* Y, uint32_t* pm, int8_t* hi, int8_t* lo, int32_t* e, int Kp) {
    const int cg = C / groups; const size_t M = (size_t)B * T;
    #pragma omp parallel for num_threads(NT)
    for (size_t row = 0; row < M; ++row) {
        const int b = (int)(row / T);
        const int32_t* x = X + row * C;
        int32_t* v = (int32_t*)malloc(sizeof(int32_t) * C);
        uint32_t m = 0;
        for (int c = 0; c < C; ++c) {
            const or_gnstat_t* st = &gs[b * groups + c / cg];
            int64_t y = norm_apply(I64(x[c]) - st->mean, st->e, st->sd, g[c], beta[c]);
            if (Lsig) y = lutact(y, Lsig);
            v[c] = (int32_t)y; uint32_t a = uabs32(v[c]); if (a > m) m = a;
        }
        if (hi) quant_row_out(v, C, hi + row * Kp, lo + row * Kp, e + row, Kp);
        else { memcpy(Y + row * C, v, sizeof(int32_t) * C); pm[row] = m; }
        free(v);
    }
}
static void lnorm_row(const int32_t* x, int C, const int32_t* g, const int32_t* beta, int64_t den, int32_t* v) {
    int64_t sum = 0; int32_t mn = INT32_MAX, mx = INT32_MIN;
    for (int c = 0; c < C; ++c) { sum += x[c]; if (x[c] < mn) mn = x[c]; if (x[c] > mx) mx = x[c]; }
    int64_t mean; int e; norm_finish(sum, mn, mx, C, &mean, &e);
    int64_t ss = 0;
    for (int c = 0; c < C; ++c) { int64_t dd = or_rshr(I64(x[c]) - mean, e); ss += dd * dd; }
    int64_t sd = norm_sd(ss, C, e, den);
    for (int c = 0; c < C; ++c) v[c] = (int32_t)norm_apply(I64(x[c]) - mean, e, sd, g[c], beta[c]);
}
void or_lnorm_q(const int32_t* X, int M, int C, const int32_t* g, const int32_t* beta, int64_t den,
                int8_t* hi, int8_t* lo, int32_t* e, int Kp) {
    #pragma omp parallel for num_threads(NT)
    for (int r = 0; r < M; ++r) {
        int32_t* v = (int32_t*)malloc(sizeof(int32_t) * C);
        lnorm_row(X + (size_t)r * C, C, g, beta, den, v);
        quant_row_out(v, C, hi + (size_t)r * Kp, lo + (size_t)r * Kp, e + r, Kp);
        free(v);
    }
}
void or_lnorm(const int32_t* X, int M, int C, const int32_t* g, const int32_t* beta, int64_t den, int32_t* Y) {
    #pragma omp parallel for num_threads(NT)
    for (int r = 0; r < M; ++r) lnorm_row(X + (size_t)r * C, C, g, beta, den, Y + (size_t)r * C);
}

/* ======================================================================
 * elementwise -- src/kernels.cu:537-561, 563-607
 * ==================================================================== */
void or_act(int32_t* X, size_t n, const int32_t* L) { for (size_t i = 0; i < n; ++i) X[i] = lutact(X[i], L); }
void or_geglu(int32_t* A, const int32_t* G, size_t n, const int32_t* L) {
    for (size_t i = 0; i < n; ++i) A[i] = (int32_t)or_sat32(or_rshr(I64(A[i]) * lutact(G[i], L), 16));
}
void or_add(int32_t* X, const int32_t* Y, size_t n) { for (size_t i = 0; i < n; ++i) X[i] = (int32_t)or_sat32(I64(X[i]) + Y[i]); }
void or_concat(const int32_t* A, int Ca, const int32_t* Bm, int Cb, int rows, int32_t* out) {
    const int Co = Ca + Cb;
    for (int r = 0; r < rows; ++r) {
        memcpy(out + (size_t)r * Co, A + (size_t)r * Ca, sizeof(int32_t) * Ca);
        memcpy(out + (size_t)r * Co + Ca, Bm + (size_t)r * Cb, sizeof(int32_t) * Cb);
    }
}
void or_upsample2(const int32_t* X, int B, int H, int W, int C, int32_t* out) {
    for (int b = 0; b < B; ++b) for (int y = 0; y < 2 * H; ++y) for (int x = 0; x < 2 * W; ++x)
        memcpy(out + (((size_t)b * 2 * H + y) * 2 * W + x) * C, X + (((size_t)b * H + (y >> 1)) * W + (x >> 1)) * C, sizeof(int32_t) * C);
}
/* ChaCha20 block function (RFC 7539 section 2.3), as used by src/kernels.cu:567-579 */
static inline uint32_t rotl32(uint32_t v, int n) { return (v << n) | (v >> (32 - n)); }
#define OR_QR(a, b, c, d) a += b; d ^= a; d = rotl32(d, 16); c += d; b ^= c; b = rotl32(b, 12); a += b; d ^= a; d = rotl32(d, 8); c += d; b ^= c; b = rotl32(b, 7);
void or_chacha20_block(const uint8_t key[32], uint32_t counter, uint32_t out[16]) {
    uint32_t in[16], st[16];
    in[0] = 0x61707865u; in[1] = 0x3320646eu; in[2] = 0x79622d32u; in[3] = 0x6b206574u;
    for (int i = 0; i < 8; ++i) in[4 + i] = (uint32_t)key[4 * i] | ((uint32_t)key[4 * i + 1] << 8) | ((uint32_t)key[4 * i + 2] << 16) | ((uint32_t)key[4 * i + 3] << 24);
    in[12] = counter; in[13] = 0; in[14] = 0; in[15] = 0;
    for (int i = 0; i < 16; ++i) st[i] = in[i];
    for (int r = 0; r < 10; ++r) {
        OR_QR(st[0], st[4], st[8], st[12]) OR_QR(st[1], st[5], st[9], st[13]) OR_QR(st[2], st[6], st[10], st[14]) OR_QR(st[3], st[7], st[11], st[15])
        OR_QR(st[0], st[5], st[10], st[15]) OR_QR(st[1], st[6], st[11], st[12]) OR_QR(st[2], st[7], st[8], st[13]) OR_QR(st[3], st[4], st[9], st[14])
    }
    for (int i = 0; i < 16; ++i) out[i] = st[i] + in[i];
}
/* src/kernels.cu:567-591: 512 keystream blocks per sample -> 16384 u16 (LE halves)
 * -> n = gauss[u] channel-major [4][4096]; x[p*4+c] = rshr(n*cin, 30) (NHWC) */
void or_noise(const uint8_t* seeds, int B, const int32_t* gauss, int64_t cin, int32_t* n, int32_t* x) {
    for (int b = 0; b < B; ++b) {
        int32_t* nb = n + (size_t)b * 16384; int32_t* xb = x + (size_t)b * 16384;
        for (int blk = 0; blk < 512; ++blk) {
            uint32_t w[16]; or_chacha20_block(seeds + 32 * b, (uint32_t)blk, w);
            for (int i = 0; i < 16; ++i) {
                uint32_t u[2] = { w[i] & 0xffffu, w[i] >> 16 };
                for (int j = 0; j < 2; ++j) {
                    int idx = blk * 32 + 2 * i + j;
                    int64_t g = gauss[u[j]];
                    nb[idx] = (int32_t)g;
                    xb[(idx & 4095) * 4 + (idx >> 12)] = (int32_t)or_rshr(g * cin, 30);
                }
            }
        }
    }
}
/* src/kernels.cu:592-599 */
void or_finalize(const int32_t* n, const int32_t* eps, int B, int64_t sig, uint8_t* out) {
    for (size_t i = 0; i < (size_t)B * 16384; ++i) {
        int b = (int)(i / 16384), idx = (int)(i % 16384), c = idx >> 12, p = idx & 4095;
        int64_t x0 = or_rshr((I64(n[i]) - eps[(size_t)b * 16384 + p * 4 + c]) * sig, 16);
        int64_t q = clamp16(or_rshr(x0, 8));
        uint16_t u = (uint16_t)(int16_t)q;
        out[2 * i] = (uint8_t)(u & 0xff); out[2 * i + 1] = (uint8_t)(u >> 8);
    }
}
/* src/kernels.cu:600-607 */
void or_text_embed(const int32_t* ids, int T, int rowsPad, const int8_t* tw, const int32_t* tm,
                   const int32_t* ts, const int32_t* pos, int D, int32_t* X) {
    for (int t = 0; t < rowsPad; ++t) for (int d = 0; d < D; ++d) {
        if (t >= T) { X[(size_t)t * D + d] = 0; continue; }
        int id = ids[t];
        int64_t v = or_rshr(I64(tw[(size_t)id * D + d]) * tm[id], I64(ts[id]) - 16);
        X[(size_t)t * D + d] = (int32_t)or_sat32(v + pos[(size_t)t * D + d]);
    }
}

/* ======================================================================
 * attention operands -- src/kernels.cu:611-669
 * ==================================================================== */
void or_quant_heads(const int32_t* X, int B, int T, int C, int heads, int Tp,
                    int8_t* hi, int8_t* lo, int32_t* e, int64_t* hs, int64_t* ls, int64_t* tsum) {
    const int G = B * heads;
    #pragma omp parallel for num_threads(NT)
    for (int w = 0; w < G * Tp; ++w) {
        int g = w / Tp, t = w % Tp, b = g / heads, h = g % heads;
        size_t o = (size_t)w * 64;
        if (t >= T) {
            for (int d = 0; d < 64; ++d) { hi[o + d] = 0; lo[o + d] = -128; }
            e[w] = 0; hs[w] = 0; ls[w] = -128 * 64; tsum[w] = 0;
            continue;
        }
        const int32_t* x = X + ((size_t)b * T + t) * C + h * 64;
        uint32_t m = 0;
        for (int d = 0; d < 64; ++d) { uint32_t a = uabs32(x[d]); if (a > m) m = a; }
        int ee = or_row_exp(m);
        int64_t sh = 0, sl = 0, st = 0;
        for (int d = 0; d < 64; ++d) {
            int64_t q = or_quant16(x[d], ee); int8_t a, c; split16(q, &a, &c);
            hi[o + d] = a; lo[o + d] = c; sh += a; sl += c; st += q;
        }
        e[w] = ee; hs[w] = sh; ls[w] = sl; tsum[w] = st;
    }
}
void or_quant_v(const int32_t* X, int B, int Tk, int C, int heads, int Tkp,
                int8_t* vt_hi, int8_t* vt_lo, int32_t* ev, int64_t* vsum) {
    const int G = B * heads;
    #pragma omp parallel for num_threads(NT)
    for (int gd = 0; gd < G * 64; ++gd) {
        int g = gd / 64, d = gd % 64, b = g / heads, h = g % heads;
        const int32_t* x = X + (size_t)b * Tk * C + h * 64 + d;
        uint32_t m = 0;
        for (int t = 0; t < Tk; ++t) { uint32_t a = uabs32(x[(size_t)t * C]); if (a > m) m = a; }
        int e = or_row_exp(m);
        int64_t s = 0;
        for (int t = 0; t < Tkp; ++t) {
            int64_t q = t < Tk ? or_quant16(x[(size_t)t * C], e) : 0;
            if (t < Tk) s += q;
            int8_t a, c; split16(q, &a, &c);
            vt_hi[(size_t)gd * Tkp + t] = a; vt_lo[(size_t)gd * Tkp + t] = c;
        }
        ev[gd] = e; vsum[gd] = s;
    }
}

/* ======================================================================
 * exact attention -- the plain-loop statement of src/kernels.cu:671-722,
 * the same arithmetic the fused kernels compute (src/attn.cu:1-6,113-320):
 *   S = Q.K (16-bit values), s = rshr(S, 19-eq-ek), mx = max s,
 *   E = exp LUT(mx - s) (0 when mx - s >= 2^20), r = floor(2^62 / sum E),
 *   P = min(32767, (E r + 2^46) >> 47), out = rshr(sum P.V, 15 - ev)
 * ==================================================================== */
static inline int32_t lut_exp(int64_t z, const int32_t* L) {
    if (z >= (I64(16) << 16)) return 0;
    int64_t i = z >> 10, f = z & 1023;
    return (int32_t)(L[i] + (((I64(L[i + 1]) - L[i]) * f) >> 10));
}
/* attention core on 16-bit values: Q [G][Tqp][64], K [G][Tkp][64], V [G][Tkp][64] */
static void attn_core(const int16_t* Qv, const int32_t* eq, int Tqp, const int16_t* Kv, const int32_t* ek,
                      const int16_t* Vv, const int32_t* ev, int B, int heads, int Tq, int Tk, int Tkp,
                      int causal, const int32_t* Lexp, int C, int32_t* out, uint32_t* rowmax) {
    const int G = B * heads;
    #pragma omp parallel for collapse(2) num_threads(NT) schedule(dynamic, 8)
    for (int g = 0; g < G; ++g) for (int q = 0; q < Tq; ++q) {
        const int b = g / heads, h = g % heads;
        int32_t* s = (int32_t*)malloc(sizeof(int32_t) * Tkp);
        int64_t* P = (int64_t*)malloc(sizeof(int64_t) * Tkp);
        const int16_t* qv = Qv + ((size_t)g * Tqp + q) * 64;
        const int eqq = eq[(size_t)g * Tqp + q];
        int32_t mx = INT32_MIN;
        int nk = Tk; if (causal && q + 1 < nk) nk = q + 1;
        for (int k = 0; k < nk; ++k) {
            const int16_t* kv = Kv + ((size_t)g * Tkp + k) * 64;
            int64_t S = 0;
            for (int d = 0; d < 64; ++d) S += (int32_t)qv[d] * (int32_t)kv[d];
            s[k] = or_score(S, 19 - eqq - ek[(size_t)g * Tkp + k]);
            if (s[k] > mx) mx = s[k];
        }
        int64_t sum = 0;
        for (int k = 0; k < nk; ++k) { P[k] = lut_exp(I64(mx) - s[k], Lexp); sum += P[k]; }
        int64_t r = sum > 0 ? or_floor_div(I64(1) << 62, sum) : 0;
        for (int k = 0; k < nk; ++k) {
            int64_t E = P[k], p = 0;
            if (E > 0) { p = (E * r + (I64(1) << 46)) >> 47; if (p > 32767) p = 32767; }
            P[k] = p;
        }
        uint32_t am = 0;
        for (int d = 0; d < 64; ++d) {
            int64_t O = 0;
            for (int k = 0; k < nk; ++k) O += P[k] * Vv[((size_t)g * Tkp + k) * 64 + d];
            int32_t o = (int32_t)or_rshr(O, 15 - ev[g * 64 + d]);
            out[((size_t)b * Tq + q) * C + h * 64 + d] = o;
            uint32_t a = uabs32(o); if (a > am) am = a;
        }
        if (rowmax) {
            #pragma omp critical
            { if (am > rowmax[(size_t)b * Tq + q]) rowmax[(size_t)b * Tq + q] = am; }
        }
        free(s); free(P);
    }
}
void or_attention(const int8_t* qhi, const int8_t* qlo, const int32_t* eq, int Tqp,
                  const int8_t* khi, const int8_t* klo, const int32_t* ek,
                  const int8_t* vthi, const int8_t* vtlo, const int32_t* ev,
                  int B, int heads, int Tq, int Tk, int Tkp, int causal, const int32_t* Lexp,
                  int C, int32_t* out, uint32_t* rowmax) {
    const int G = B * heads;
    int16_t* Qv = (int16_t*)malloc(sizeof(int16_t) * (size_t)G * Tqp * 64);
    int16_t* Kv = (int16_t*)malloc(sizeof(int16_t) * (size_t)G * Tkp * 64);
    int16_t* Vv = (int16_t*)malloc(sizeof(int16_t) * (size_t)G * Tkp * 64);
    for (size_t i = 0; i < (size_t)G * Tqp * 64; ++i) Qv[i] = (int16_t)(256 * qhi[i] + qlo[i] + 128);
    for (size_t i = 0; i < (size_t)G * Tkp * 64; ++i) Kv[i] = (int16_t)(256 * khi[i] + klo[i] + 128);
    for (int g = 0; g < G; ++g) for (int d = 0; d < 64; ++d) for (int t = 0; t < Tkp; ++t) {
        size_t src = ((size_t)g * 64 + d) * Tkp + t;
        Vv[((size_t)g * Tkp + t) * 64 + d] = (int16_t)(256 * vthi[src] + vtlo[src] + 128);
    }
    attn_core(Qv, eq, Tqp, Kv, ek, Vv, ev, B, heads, Tq, Tk, Tkp, causal, Lexp, C, out, rowmax);
    free(Qv); free(Kv); free(Vv);
}

/* ======================================================================
 * POISD model file (src/poisd.cpp:11-35) and the UNet step
 * (src/engine.cu:11-101 weight preparation, :389-490 composition,
 *  :491-574 prompt, :599-609 one step)
 * ==================================================================== */
typedef struct { char* name; int dtype; int nd; uint32_t dims[4]; size_t count; const uint8_t* data; } or_entry_t;
typedef struct { int N, K; int16_t* w; int32_t* cst; int conv3; } or_lin_t;          /* cst: {m, s, b, wsum} per row */
typedef struct { int C; int32_t* g; int32_t* beta; int64_t den; } or_norm_t;
typedef struct { int Tk, Tkp, heads; int16_t* K; int32_t* ek; int16_t* V; int32_t* ev; } or_kv_t;   /* one copy (B = 1) */
struct or_model {
    uint8_t* file; size_t size;
    or_entry_t* ent; int nent;
    int32_t *lut_sig, *lut_phi, *lut_exp, *lut_gauss;
    int64_t c_sig, c_cin;
    int32_t ctx[77 * 1024]; int have_ctx;
    or_kv_t cross[16]; char cross_name[16][96];
    /* cache of prepared linears / norms, looked up by name */
    char (*lin_name)[128]; or_lin_t* lins; int nlin, caplin;
    char (*norm_name)[128]; or_norm_t* norms; int nnorm, capnorm;
};

static const or_entry_t* find_entry(const or_model_t* m, const char* name) {
    for (int i = 0; i < m->nent; ++i) if (strcmp(m->ent[i].name, name) == 0) return &m->ent[i];
    return NULL;
}
static const int32_t* i32p(const or_model_t* m, const char* name) {
    const or_entry_t* e = find_entry(m, name);
    if (!e || e->dtype != 2) { fprintf(stderr, "oracle: missing int32 tensor %s\n", name); abort(); }
    return (const int32_t*)e->data;
}
static int endswith(const char* s, const char* suf) { size_t a = strlen(s), b = strlen(suf); return a >= b && strcmp(s + a - b, suf) == 0; }

/* weight preparation restating src/engine.cu:11-46 (the oracle keeps the
 * file's K order, c*9 + tap for 3x3 convolutions, and widens to int16) */
static const or_lin_t* get_lin(or_model_t* m, const char* base) {
    for (int i = 0; i < m->nlin; ++i) if (strcmp(m->lin_name[i], base) == 0) return &m->lins[i];
    char nm[160]; snprintf(nm, sizeof nm, "%s.w", base);
    const or_entry_t* we = find_entry(m, nm);
    if (!we || we->dtype != 0 || we->nd != 2) { fprintf(stderr, "oracle: no linear %s\n", base); abort(); }
    or_lin_t L; L.N = (int)we->dims[0]; L.K = (int)we->dims[1];
    L.conv3 = endswith(base, ".conv1") || endswith(base, ".conv2") || endswith(base, "conv_in") || endswith(base, "conv_out") ||
              endswith(base, "downsamplers.0.conv") || endswith(base, "upsamplers.0.conv");
    L.w = (int16_t*)malloc(sizeof(int16_t) * (size_t)L.N * L.K);
    L.cst = (int32_t*)malloc(sizeof(int32_t) * 4 * (size_t)L.N);
    snprintf(nm, sizeof nm, "%s.m", base); const int32_t* mv = i32p(m, nm);
    snprintf(nm, sizeof nm, "%s.s", base); const int32_t* sv = i32p(m, nm);
    snprintf(nm, sizeof nm, "%s.b", base); const int32_t* bv = i32p(m, nm);
    const int8_t* w8 = (const int8_t*)we->data;
    for (int n = 0; n < L.N; ++n) {
        int64_t ws = 0;
        for (int k = 0; k < L.K; ++k) { L.w[(size_t)n * L.K + k] = w8[(size_t)n * L.K + k]; ws += w8[(size_t)n * L.K + k]; }
        L.cst[4 * n] = mv[n]; L.cst[4 * n + 1] = sv[n]; L.cst[4 * n + 2] = bv[n]; L.cst[4 * n + 3] = (int32_t)ws;
    }
    if (m->nlin == m->caplin) {
        m->caplin = m->caplin ? 2 * m->caplin : 256;
        m->lins = (or_lin_t*)realloc(m->lins, sizeof(or_lin_t) * m->caplin);
        m->lin_name = (char (*)[128])realloc(m->lin_name, 128 * (size_t)m->caplin);
    }
    snprintf(m->lin_name[m->nlin], 128, "%s", base);
    m->lins[m->nlin] = L;
    return &m->lins[m->nlin++];
}
static const or_norm_t* get_norm(or_model_t* m, const char* base) {
    for (int i = 0; i < m->nnorm; ++i) if (strcmp(m->norm_name[i], base) == 0) return &m->norms[i];
    char nm[160]; or_norm_t N;
    snprintf(nm, sizeof nm, "%s.g", base); const or_entry_t* ge = find_entry(m, nm);
    if (!ge) { fprintf(stderr, "oracle: no norm %s\n", base); abort(); }
    N.C = (int)ge->count; N.g = (int32_t*)ge->data;
    snprintf(nm, sizeof nm, "%s.beta", base); N.beta = (int32_t*)i32p(m, nm);
    snprintf(nm, sizeof nm, "%s.eps", base); N.den = i32p(m, nm)[0];
    if (m->nnorm == m->capnorm) {
        m->capnorm = m->capnorm ? 2 * m->capnorm : 256;
        m->norms = (or_norm_t*)realloc(m->norms, sizeof(or_norm_t) * m->capnorm);
        m->norm_name = (char (*)[128])realloc(m->norm_name, 128 * (size_t)m->capnorm);
    }
    snprintf(m->norm_name[m->nnorm], 128, "%s", base);
    m->norms[m->nnorm] = N;
    return &m->norms[m->nnorm++];
}

static uint32_t rd32(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24); }
or_model_t* or_model_load(const char* path, char* err, int errlen) {
    FILE* f = fopen(path, "rb");
    if (!f) { snprintf(err, errlen, "cannot open %s", path); return NULL; }
    fseek(f, 0, SEEK_END); size_t size = (size_t)ftell(f); fseek(f, 0, SEEK_SET);
    uint8_t* buf = (uint8_t*)malloc(size ? size : 1);
    if (fread(buf, 1, size, f) != size) { fclose(f); free(buf); snprintf(err, errlen, "read error"); return NULL; }
    fclose(f);
    static const uint8_t MAGIC[8] = { 'P', 'O', 'I', 'S', 'D', 'v', '1', 0 };
    if (size < 12 || memcmp(buf, MAGIC, 8) != 0) { free(buf); snprintf(err, errlen, "bad magic"); return NULL; }
    or_model_t* m = (or_model_t*)calloc(1, sizeof(or_model_t));
    m->file = buf; m->size = size;
    size_t pos = 8; uint32_t count = rd32(buf + pos); pos += 4;
    m->ent = (or_entry_t*)calloc(count, sizeof(or_entry_t)); m->nent = (int)count;
    static const size_t SZ[4] = { 1, 2, 4, 1 };
    for (uint32_t i = 0; i < count; ++i) {
        if (pos + 2 > size) goto trunc;
        uint16_t nl = (uint16_t)(buf[pos] | (buf[pos + 1] << 8)); pos += 2;
        if (pos + nl + 2 > size) goto trunc;
        or_entry_t* e = &m->ent[i];
        e->name = (char*)malloc(nl + 1); memcpy(e->name, buf + pos, nl); e->name[nl] = 0; pos += nl;
        e->dtype = buf[pos]; e->nd = buf[pos + 1]; pos += 2;
        if (e->dtype > 3 || e->nd > 4) { snprintf(err, errlen, "bad dtype/ndims in %s", e->name); or_model_free(m); return NULL; }
        e->count = 1;
        for (int d = 0; d < e->nd; ++d) { if (pos + 4 > size) goto trunc; e->dims[d] = rd32(buf + pos); e->count *= e->dims[d]; pos += 4; }
        if (pos + e->count * SZ[e->dtype] > size) goto trunc;
        e->data = buf + pos; pos += e->count * SZ[e->dtype];
    }
    if (pos != size) { snprintf(err, errlen, "trailing data"); or_model_free(m); return NULL; }
    m->lut_sig = (int32_t*)i32p(m, "lut.sigmoid"); m->lut_phi = (int32_t*)i32p(m, "lut.phi");
    m->lut_exp = (int32_t*)i32p(m, "lut.exp"); m->lut_gauss = (int32_t*)i32p(m, "lut.gauss");
    m->c_sig = i32p(m, "c.sig")[0]; m->c_cin = i32p(m, "c.cin")[0];
    return m;
trunc:
    snprintf(err, errlen, "truncated model file");
    or_model_free(m);
    return NULL;
}
void or_model_free(or_model_t* m) {
    if (!m) return;
    for (int i = 0; i < m->nlin; ++i) { free(m->lins[i].w); free(m->lins[i].cst); }
    free(m->lins); free(m->lin_name); free(m->norms); free(m->norm_name);
    for (int i = 0; i < 16; ++i) { free(m->cross[i].K); free(m->cross[i].ek); free(m->cross[i].V); free(m->cross[i].ev); }
    for (int i = 0; i < m->nent; ++i) free(m->ent[i].name);
    free(m->ent); free(m->file); free(m);
}
const int32_t* or_context(const or_model_t* m) { return m->have_ctx ? m->ctx : NULL; }

/* ---------------- activation tensors and the composed ops ----------------- */
typedef struct { int32_t* d; int B, T, C; } ten_t;
static ten_t talloc(int B, int T, int C) { ten_t t; t.B = B; t.T = T; t.C = C; t.d = (int32_t*)calloc((size_t)B * T * C, sizeof(int32_t)); return t; }
static void tfree(ten_t* t) { free(t->d); t->d = NULL; }
/* a quantised GEMM operand: 16-bit values q [rows][K] + e [rows] (the hi/lo planes of src/engine.h:46 as values) */
typedef struct { int16_t* q; int32_t* e; int rows, K; } qin_t;
static qin_t qalloc(int rows, int K) { qin_t q; q.rows = rows; q.K = K; q.q = (int16_t*)malloc(sizeof(int16_t) * (size_t)rows * K); q.e = (int32_t*)malloc(sizeof(int32_t) * rows); return q; }
static void qfree(qin_t* q) { free(q->q); free(q->e); }

/* row quantisation with e = row_exp(max |x|) (k_quant_rows, and the SRC_X32 loader given an exact rowmax) */
static qin_t quant_rows_v(const int32_t* X, int rows, int K) {
    qin_t q = qalloc(rows, K);
    #pragma omp parallel for num_threads(NT)
    for (int r = 0; r < rows; ++r) {
        const int32_t* x = X + (size_t)r * K; uint32_t m = 0;
        for (int k = 0; k < K; ++k) { uint32_t a = uabs32(x[k]); if (a > m) m = a; }
        int e = or_row_exp(m); q.e[r] = e;
        for (int k = 0; k < K; ++k) q.q[(size_t)r * K + k] = (int16_t)or_quant16(x[k], e);
    }
    return q;
}
/* exact sum q.w: int32 partial sums over blocks of 256 (|q w| < 2^22) widened to int64 */
static inline int64_t dot16(const int16_t* a, const int16_t* w, int K) {
    int64_t acc = 0;
    for (int k0 = 0; k0 < K; k0 += 256) {
        int k1 = k0 + 256 < K ? k0 + 256 : K; int32_t s = 0;
        for (int k = k0; k < k1; ++k) s += (int32_t)a[k] * (int32_t)w[k];
        acc += s;
    }
    return acc;
}
/* GEMM of a quantised operand with the exact epilogue; acc = sum_k q_k w_k equals
 * 256*Chi + Clo + 128*wsum of src/gemm_hl.cu:40-43 for consistent planes */
static void gemm_q(const qin_t* A, const or_lin_t* L, int32_t* acc_out /* [rows][N] epi(acc) */) {
    if (A->K != L->K) { fprintf(stderr, "oracle: K mismatch %d vs %d\n", A->K, L->K); abort(); }
    #pragma omp parallel for num_threads(NT) schedule(dynamic, 4)
    for (int r = 0; r < A->rows; ++r) {
        const int16_t* a = A->q + (size_t)r * A->K;
        for (int n = 0; n < L->N; ++n)
            acc_out[(size_t)r * L->N + n] = epi1(dot16(a, L->w + (size_t)n * L->K, L->K), L->cst + 4 * n, A->e[r]);
    }
}
/* Engine::linQ / lin / linX with EPI_PLAIN (+ residual, + rowmax) */
static ten_t lin_plain(const qin_t* A, int B, int T, const or_lin_t* L, const int32_t* residual) {
    ten_t y = talloc(B, T, L->N);
    gemm_q(A, L, y.d);
    if (residual) or_add(y.d, residual, (size_t)B * T * L->N);
    return y;
}
static ten_t lin_x(const ten_t* x, const or_lin_t* L, const int32_t* residual) {
    qin_t q = quant_rows_v(x->d, x->B * x->T, x->C);
    ten_t y = lin_plain(&q, x->B, x->T, L, residual);
    qfree(&q);
    return y;
}
/* implicit 3x3 conv: Engine::conv3 (src/engine.cu:254-280), SRC_CONV32 semantics (src/gemm_hl.cu:104-114):
 * e[row] = row_exp(max of pm over the 3x3 window); file K order c*9 + tap */
static ten_t conv3(const ten_t* x, int H, int W, const or_lin_t* L, int stride, const int32_t* residual, const uint32_t* pmIn) {
    const int C = x->C, Ho = (H - 1) / stride + 1, Wo = (W - 1) / stride + 1, rows = x->B * Ho * Wo;
    if (!L->conv3 || C * 9 != L->K) { fprintf(stderr, "oracle: conv shape\n"); abort(); }
    uint32_t* pm = (uint32_t*)pmIn;
    if (!pm) { pm = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)x->B * H * W); or_pixmax(x->d, x->B * H * W, C, pm); }
    qin_t q = qalloc(rows, L->K);
    #pragma omp parallel for num_threads(NT)
    for (int r = 0; r < rows; ++r) {
        int b = r / (Ho * Wo), p = r % (Ho * Wo), oy = p / Wo, ox = p % Wo;
        int e = or_row_exp(window_max(pm, b, H, W, oy, ox, stride)); q.e[r] = e;
        int16_t* dst = q.q + (size_t)r * L->K;
        for (int tap = 0; tap < 9; ++tap) {
            int iy = oy * stride - 1 + tap / 3, ix = ox * stride - 1 + tap % 3;
            int in = iy >= 0 && iy < H && ix >= 0 && ix < W;
            const int32_t* xp = in ? x->d + (((size_t)b * H + iy) * W + ix) * C : NULL;
            for (int c = 0; c < C; ++c) dst[c * 9 + tap] = (int16_t)(in ? or_quant16(xp[c], e) : 0);
        }
    }
    if (!pmIn) free(pm);
    ten_t y = lin_plain(&q, x->B, Ho * Wo, L, residual);
    qfree(&q);
    return y;
}
/* Engine::groupnormSilu (src/engine.cu:242-253): GN stats + apply + SiLU -> int32 + pixel max */
static ten_t gn_silu(or_model_t* m, const ten_t* x, const char* nname, uint32_t** pm) {
    const or_norm_t* N = get_norm(m, nname);
    or_gnstat_t gs[8 * 32 * 4];
    or_gnstat_t* g = x->B * 32 <= (int)(sizeof gs / sizeof gs[0]) ? gs : (or_gnstat_t*)malloc(sizeof(or_gnstat_t) * x->B * 32);
    or_gn_stats(x->d, x->B, x->T, x->C, 32, N->den, g);
    ten_t y = talloc(x->B, x->T, x->C);
    *pm = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)x->B * x->T);
    or_gn_apply_row(x->d, x->B, x->T, x->C, 32, g, N->g, N->beta, m->lut_sig, y.d, *pm, NULL, NULL, NULL, 0);
    if (g != gs) free(g);
    return y;
}
/* quantised row output of a normalised row (src/kernels.cu:250-259) as 16-bit values */
static void qrow_values(const int32_t* v, int C, int16_t* q, int32_t* e) {
    uint32_t m = 0;
    for (int c = 0; c < C; ++c) { uint32_t a = uabs32(v[c]); if (a > m) m = a; }
    int ee = or_row_exp(m); *e = ee;
    for (int c = 0; c < C; ++c) q[c] = (int16_t)or_quant16(v[c], ee);
}
/* Engine::groupnormQ (src/engine.cu:231-241): GN (no activation) -> quantised operand */
static qin_t gn_q(or_model_t* m, const ten_t* x, const char* nname) {
    const or_norm_t* N = get_norm(m, nname);
    or_gnstat_t* g = (or_gnstat_t*)malloc(sizeof(or_gnstat_t) * x->B * 32);
    or_gn_stats(x->d, x->B, x->T, x->C, 32, N->den, g);
    ten_t y = talloc(x->B, x->T, x->C);
    uint32_t* pm = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)x->B * x->T);
    or_gn_apply_row(x->d, x->B, x->T, x->C, 32, g, N->g, N->beta, NULL, y.d, pm, NULL, NULL, NULL, 0);
    qin_t q = qalloc(x->B * x->T, x->C);
    #pragma omp parallel for num_threads(NT)
    for (int r = 0; r < q.rows; ++r) qrow_values(y.d + (size_t)r * x->C, x->C, q.q + (size_t)r * x->C, &q.e[r]);
    free(g); free(pm); tfree(&y);
    return q;
}
/* Engine::layernormQ (src/engine.cu:225-230) */
static qin_t ln_q(or_model_t* m, const ten_t* x, const char* nname) {
    const or_norm_t* N = get_norm(m, nname);
    qin_t q = qalloc(x->B * x->T, x->C);
    #pragma omp parallel for num_threads(NT)
    for (int r = 0; r < q.rows; ++r) {
        int32_t* v = (int32_t*)malloc(sizeof(int32_t) * x->C);
        lnorm_row(x->d + (size_t)r * x->C, x->C, N->g, N->beta, N->den, v);
        qrow_values(v, x->C, q.q + (size_t)r * x->C, &q.e[r]);
        free(v);
    }
    return q;
}
/* per-(sample, head, token) quantisation of a [B,T,C] tensor into [G][Tp][64] values (k_quant_heads / EPI_QKV) */
static void head_quant(const int32_t* X, int B, int T, int C, int heads, int Tp, int16_t* Qv, int32_t* e) {
    const int G = B * heads;
    #pragma omp parallel for num_threads(NT)
    for (int w = 0; w < G * Tp; ++w) {
        int g = w / Tp, t = w % Tp, b = g / heads, h = g % heads;
        if (t >= T) { memset(Qv + (size_t)w * 64, 0, 64 * sizeof(int16_t)); e[w] = 0; continue; }
        qrow_values(X + ((size_t)b * T + t) * C + h * 64, 64, Qv + (size_t)w * 64, &e[w]);
    }
}
/* per-(sample, head, dim) column quantisation of V into [G][Tkp][64] values (k_quant_v) */
static void v_quant(const int32_t* X, int B, int Tk, int C, int heads, int Tkp, int16_t* Vv, int32_t* ev) {
    const int G = B * heads;
    #pragma omp parallel for num_threads(NT)
    for (int gd = 0; gd < G * 64; ++gd) {
        int g = gd / 64, d = gd % 64, b = g / heads, h = g % heads;
        const int32_t* x = X + (size_t)b * Tk * C + h * 64 + d;
        uint32_t mm = 0;
        for (int t = 0; t < Tk; ++t) { uint32_t a = uabs32(x[(size_t)t * C]); if (a > mm) mm = a; }
        int e = or_row_exp(mm); ev[gd] = e;
        for (int t = 0; t < Tkp; ++t) Vv[((size_t)g * Tkp + t) * 64 + d] = (int16_t)(t < Tk ? or_quant16(x[(size_t)t * C], e) : 0);
    }
}
/* self attention of a transformer block: merged q|k|v GEMM (EPI_QKV), quantKVH, fused attention
 * (src/engine.cu:318-350); returns the int32 output [B,T,C] */
static ten_t self_attention(or_model_t* m, const qin_t* n, int B, int T, int C, int heads, const char* pfx, int causal, int Treal) {
    char nm[192];
    ten_t q, k, v;
    snprintf(nm, sizeof nm, "%s.to_q", pfx); q = lin_plain(n, B, T, get_lin(m, nm), NULL);
    snprintf(nm, sizeof nm, "%s.to_k", pfx); k = lin_plain(n, B, T, get_lin(m, nm), NULL);
    snprintf(nm, sizeof nm, "%s.to_v", pfx); v = lin_plain(n, B, T, get_lin(m, nm), NULL);
    const int G = B * heads, Tk = Treal, Tkp = (Tk + 63) / 64 * 64, Tq = Treal, Tqp = (Tq + 127) / 128 * 128;
    int16_t* Qv = (int16_t*)malloc(sizeof(int16_t) * (size_t)G * Tqp * 64); int32_t* eq = (int32_t*)malloc(sizeof(int32_t) * (size_t)G * Tqp);
    int16_t* Kv = (int16_t*)malloc(sizeof(int16_t) * (size_t)G * Tkp * 64); int32_t* ek = (int32_t*)malloc(sizeof(int32_t) * (size_t)G * Tkp);
    int16_t* Vv = (int16_t*)malloc(sizeof(int16_t) * (size_t)G * Tkp * 64); int32_t* ev = (int32_t*)malloc(sizeof(int32_t) * (size_t)G * 64);
    /* q, k of the real tokens; with T > Treal (text encoder padding rows) only the first Treal rows of each sample matter */
    int32_t* qr = q.d; int32_t* kr = k.d; int32_t* vr = v.d;
    int32_t *qc = NULL, *kc = NULL, *vc = NULL;
    if (T != Treal) {
        qc = (int32_t*)malloc(sizeof(int32_t) * (size_t)B * Treal * C); kc = (int32_t*)malloc(sizeof(int32_t) * (size_t)B * Treal * C); vc = (int32_t*)malloc(sizeof(int32_t) * (size_t)B * Treal * C);
        for (int b = 0; b < B; ++b) {
            memcpy(qc + (size_t)b * Treal * C, q.d + (size_t)b * T * C, sizeof(int32_t) * (size_t)Treal * C);
            memcpy(kc + (size_t)b * Treal * C, k.d + (size_t)b * T * C, sizeof(int32_t) * (size_t)Treal * C);
            memcpy(vc + (size_t)b * Treal * C, v.d + (size_t)b * T * C, sizeof(int32_t) * (size_t)Treal * C);
        }
        qr = qc; kr = kc; vr = vc;
    }
    head_quant(qr, B, Treal, C, heads, Tqp, Qv, eq);
    head_quant(kr, B, Treal, C, heads, Tkp, Kv, ek);
    v_quant(vr, B, Treal, C, heads, Tkp, Vv, ev);
    ten_t out = talloc(B, Tq, C);
    attn_core(Qv, eq, Tqp, Kv, ek, Vv, ev, B, heads, Tq, Tk, Tkp, causal, m->lut_exp, C, out.d, NULL);
    free(Qv); free(eq); free(Kv); free(ek); free(Vv); free(ev); free(qc); free(kc); free(vc);
    tfree(&q); tfree(&k); tfree(&v);
    return out;
}
static void emit(or_tap_fn tap, void* user, const char* name, const ten_t* t) { if (tap) tap(user, name, t->d, (size_t)t->B * t->T * t->C); }

/* Engine::resnet, src/engine.cu:389-405 */
static ten_t resnet(or_model_t* m, const ten_t* x, int H, int W, const char* p) {
    char nm[192];
    uint32_t *pm1, *pm2;
    snprintf(nm, sizeof nm, "%s.norm1", p); ten_t h = gn_silu(m, x, nm, &pm1);
    snprintf(nm, sizeof nm, "%s.conv1", p); ten_t h1 = conv3(&h, H, W, get_lin(m, nm), 1, NULL, pm1);
    tfree(&h); free(pm1);
    snprintf(nm, sizeof nm, "%s.norm2", p); ten_t h2 = gn_silu(m, &h1, nm, &pm2);
    tfree(&h1);
    snprintf(nm, sizeof nm, "%s.conv_shortcut.w", p);
    ten_t out;
    if (find_entry(m, nm)) {
        snprintf(nm, sizeof nm, "%s.conv_shortcut", p);
        ten_t xs = lin_x(x, get_lin(m, nm), NULL);
        snprintf(nm, sizeof nm, "%s.conv2", p); out = conv3(&h2, H, W, get_lin(m, nm), 1, xs.d, pm2);
        tfree(&xs);
    } else {
        snprintf(nm, sizeof nm, "%s.conv2", p); out = conv3(&h2, H, W, get_lin(m, nm), 1, x->d, pm2);
    }
    tfree(&h2); free(pm2);
    return out;
}
/* Engine::transformer, src/engine.cu:406-454 */
static ten_t transformer(or_model_t* m, const ten_t* x, const char* p, int heads) {
    char nm[192], b[160];
    snprintf(b, sizeof b, "%s.transformer_blocks.0", p);
    const int B = x->B, T = x->T, C = x->C;
    snprintf(nm, sizeof nm, "%s.norm", p); qin_t xq = gn_q(m, x, nm);
    snprintf(nm, sizeof nm, "%s.proj_in", p); ten_t h = lin_plain(&xq, B, T, get_lin(m, nm), NULL);
    qfree(&xq);
    {   /* self attention */
        snprintf(nm, sizeof nm, "%s.norm1", b); qin_t n = ln_q(m, &h, nm);
        snprintf(nm, sizeof nm, "%s.attn1", b); ten_t a = self_attention(m, &n, B, T, C, heads, nm, 0, T);
        qfree(&n);
        snprintf(nm, sizeof nm, "%s.attn1.to_out.0", b); ten_t h2 = lin_x(&a, get_lin(m, nm), h.d);
        tfree(&a); tfree(&h); h = h2;
    }
    {   /* cross attention against the prompt's K/V */
        snprintf(nm, sizeof nm, "%s.norm2", b); qin_t n = ln_q(m, &h, nm);
        snprintf(nm, sizeof nm, "%s.attn2.to_q", b); ten_t q = lin_plain(&n, B, T, get_lin(m, nm), NULL);
        qfree(&n);
        const or_kv_t* kv = NULL;
        for (int i = 0; i < 16; ++i) if (strcmp(m->cross_name[i], b) == 0) kv = &m->cross[i];
        if (!kv) { fprintf(stderr, "oracle: no cross K/V for %s\n", b); abort(); }
        const int G = B * heads, Tqp = (T + 127) / 128 * 128;
        int16_t* Qv = (int16_t*)malloc(sizeof(int16_t) * (size_t)G * Tqp * 64); int32_t* eq = (int32_t*)malloc(sizeof(int32_t) * (size_t)G * Tqp);
        head_quant(q.d, B, T, C, heads, Tqp, Qv, eq);
        /* replicate the single-prompt K/V over the batch (src/engine.cu:558-568) */
        int16_t* Kv = (int16_t*)malloc(sizeof(int16_t) * (size_t)G * kv->Tkp * 64); int32_t* ek = (int32_t*)malloc(sizeof(int32_t) * (size_t)G * kv->Tkp);
        int16_t* Vv = (int16_t*)malloc(sizeof(int16_t) * (size_t)G * kv->Tkp * 64); int32_t* ev = (int32_t*)malloc(sizeof(int32_t) * (size_t)G * 64);
        for (int bb = 0; bb < B; ++bb) {
            memcpy(Kv + (size_t)bb * heads * kv->Tkp * 64, kv->K, sizeof(int16_t) * (size_t)heads * kv->Tkp * 64);
            memcpy(ek + (size_t)bb * heads * kv->Tkp, kv->ek, sizeof(int32_t) * (size_t)heads * kv->Tkp);
            memcpy(Vv + (size_t)bb * heads * kv->Tkp * 64, kv->V, sizeof(int16_t) * (size_t)heads * kv->Tkp * 64);
            memcpy(ev + (size_t)bb * heads * 64, kv->ev, sizeof(int32_t) * (size_t)heads * 64);
        }
        ten_t a = talloc(B, T, C);
        attn_core(Qv, eq, Tqp, Kv, ek, Vv, ev, B, heads, T, kv->Tk, kv->Tkp, 0, m->lut_exp, C, a.d, NULL);
        free(Qv); free(eq); free(Kv); free(ek); free(Vv); free(ev); tfree(&q);
        snprintf(nm, sizeof nm, "%s.attn2.to_out.0", b); ten_t h2 = lin_x(&a, get_lin(m, nm), h.d);
        tfree(&a); tfree(&h); h = h2;
    }
    {   /* GEGLU feed-forward (interleaved a|g GEMM, src/engine.cu:443-450) */
        snprintf(nm, sizeof nm, "%s.norm3", b); qin_t n = ln_q(m, &h, nm);
        snprintf(nm, sizeof nm, "%s.ff.net.0.proj.a", b); ten_t a = lin_plain(&n, B, T, get_lin(m, nm), NULL);
        snprintf(nm, sizeof nm, "%s.ff.net.0.proj.g", b); ten_t g = lin_plain(&n, B, T, get_lin(m, nm), NULL);
        qfree(&n);
        or_geglu(a.d, g.d, (size_t)B * T * a.C, m->lut_phi);
        tfree(&g);
        snprintf(nm, sizeof nm, "%s.ff.net.2", b); ten_t h2 = lin_x(&a, get_lin(m, nm), h.d);
        tfree(&a); tfree(&h); h = h2;
    }
    snprintf(nm, sizeof nm, "%s.proj_out", p); ten_t out = lin_x(&h, get_lin(m, nm), x->d);
    tfree(&h);
    return out;
}

static const int HEADS[4] = { 5, 10, 20, 20 };
static const char* cross_block_name(int idx, char* buf, size_t n, int* heads) {
    if (idx < 6) { snprintf(buf, n, "unet.down_blocks.%d.attentions.%d.transformer_blocks.0", idx / 2, idx % 2); *heads = HEADS[idx / 2]; }
    else if (idx == 6) { snprintf(buf, n, "unet.mid_block.attentions.0.transformer_blocks.0"); *heads = 20; }
    else { int i = 1 + (idx - 7) / 3, j = (idx - 7) % 3; snprintf(buf, n, "unet.up_blocks.%d.attentions.%d.transformer_blocks.0", i, j); *heads = HEADS[3 - i]; }
    return buf;
}

/* Engine::textEncoder + setPrompt (src/engine.cu:491-574).  Only the 77 real
 * rows are computed: every op on this path is row-local and the causal
 * attention masks keys >= 77, so the padding rows 77..95 never reach them. */
int or_set_prompt(or_model_t* m, const int32_t* tokens, int ntok) {
    const int T = 77, D = 1024;
    if (ntok + 2 > T) return -1;
    int32_t ids[77]; int n = 0;
    ids[n++] = 49406; for (int i = 0; i < ntok; ++i) ids[n++] = tokens[i]; ids[n++] = 49407;
    while (n < T) ids[n++] = 0;
    const or_entry_t* tw = find_entry(m, "te.tok.w");
    ten_t x = talloc(1, T, D);
    or_text_embed(ids, T, T, (const int8_t*)tw->data, i32p(m, "te.tok.m"), i32p(m, "te.tok.s"), i32p(m, "te.pos"), D, x.d);
    char nm[192], p[64];
    for (int l = 0; l < 23; ++l) {
        snprintf(p, sizeof p, "te.layers.%d", l);
        snprintf(nm, sizeof nm, "%s.layer_norm1", p); qin_t nq = ln_q(m, &x, nm);
        /* the text encoder's projections are named q_proj/k_proj/v_proj */
        ten_t q, k, v;
        snprintf(nm, sizeof nm, "%s.self_attn.q_proj", p); q = lin_plain(&nq, 1, T, get_lin(m, nm), NULL);
        snprintf(nm, sizeof nm, "%s.self_attn.k_proj", p); k = lin_plain(&nq, 1, T, get_lin(m, nm), NULL);
        snprintf(nm, sizeof nm, "%s.self_attn.v_proj", p); v = lin_plain(&nq, 1, T, get_lin(m, nm), NULL);
        qfree(&nq);
        const int heads = 16, G = heads, Tkp = 128, Tqp = 128;
        int16_t* Qv = (int16_t*)malloc(sizeof(int16_t) * G * Tqp * 64); int32_t* eq = (int32_t*)malloc(sizeof(int32_t) * G * Tqp);
        int16_t* Kv = (int16_t*)malloc(sizeof(int16_t) * G * Tkp * 64); int32_t* ek = (int32_t*)malloc(sizeof(int32_t) * G * Tkp);
        int16_t* Vv = (int16_t*)malloc(sizeof(int16_t) * G * Tkp * 64); int32_t* ev = (int32_t*)malloc(sizeof(int32_t) * G * 64);
        head_quant(q.d, 1, T, D, heads, Tqp, Qv, eq);
        head_quant(k.d, 1, T, D, heads, Tkp, Kv, ek);
        v_quant(v.d, 1, T, D, heads, Tkp, Vv, ev);
        ten_t a = talloc(1, T, D);
        attn_core(Qv, eq, Tqp, Kv, ek, Vv, ev, 1, heads, T, T, Tkp, 1, m->lut_exp, D, a.d, NULL);
        free(Qv); free(eq); free(Kv); free(ek); free(Vv); free(ev); tfree(&q); tfree(&k); tfree(&v);
        snprintf(nm, sizeof nm, "%s.self_attn.out_proj", p); ten_t x2 = lin_x(&a, get_lin(m, nm), x.d);
        tfree(&a); tfree(&x); x = x2;
        snprintf(nm, sizeof nm, "%s.layer_norm2", p); qin_t n2 = ln_q(m, &x, nm);
        snprintf(nm, sizeof nm, "%s.mlp.fc1", p); ten_t f = lin_plain(&n2, 1, T, get_lin(m, nm), NULL);
        qfree(&n2);
        or_act(f.d, (size_t)T * f.C, m->lut_phi);    /* EPI_GELU (src/gemm_hl.cu:279-280) */
        snprintf(nm, sizeof nm, "%s.mlp.fc2", p); x2 = lin_x(&f, get_lin(m, nm), x.d);
        tfree(&f); tfree(&x); x = x2;
    }
    const or_norm_t* fn = get_norm(m, "te.final_layer_norm");
    or_lnorm(x.d, T, D, fn->g, fn->beta, fn->den, m->ctx);
    tfree(&x);
    m->have_ctx = 1;
    /* cross-attention K/V per transformer block, computed once (B = 1) */
    ten_t ctx; ctx.d = m->ctx; ctx.B = 1; ctx.T = T; ctx.C = D;
    for (int i = 0; i < 16; ++i) {
        int heads; char bn[96]; cross_block_name(i, bn, sizeof bn, &heads);
        or_kv_t* kv = &m->cross[i];
        free(kv->K); free(kv->ek); free(kv->V); free(kv->ev);
        snprintf(m->cross_name[i], sizeof m->cross_name[i], "%s", bn);
        snprintf(nm, sizeof nm, "%s.attn2.to_k", bn); ten_t k = lin_x(&ctx, get_lin(m, nm), NULL);
        snprintf(nm, sizeof nm, "%s.attn2.to_v", bn); ten_t v = lin_x(&ctx, get_lin(m, nm), NULL);
        kv->heads = heads; kv->Tk = T; kv->Tkp = 128;
        kv->K = (int16_t*)malloc(sizeof(int16_t) * heads * 128 * 64); kv->ek = (int32_t*)malloc(sizeof(int32_t) * heads * 128);
        kv->V = (int16_t*)malloc(sizeof(int16_t) * heads * 128 * 64); kv->ev = (int32_t*)malloc(sizeof(int32_t) * heads * 64);
        head_quant(k.d, 1, T, k.C, heads, 128, kv->K, kv->ek);
        v_quant(v.d, 1, T, v.C, heads, 128, kv->V, kv->ev);
        tfree(&k); tfree(&v);
    }
    return 0;
}

/* Engine::forwardIO + Engine::unet (src/engine.cu:455-490,599-609) */
int or_unet_step(or_model_t* m, const uint8_t* seeds, int B, uint8_t* x0, int32_t* eps_out, or_tap_fn tap, void* user) {
    if (!m->have_ctx) return -1;
    char nm[192];
    int32_t* noise = (int32_t*)malloc(sizeof(int32_t) * (size_t)B * 16384);
    ten_t x = talloc(B, 4096, 4);
    or_noise(seeds, B, m->lut_gauss, m->c_cin, noise, x.d);
    emit(tap, user, "x", &x);
    int H = 64, W = 64;
    ten_t h = conv3(&x, H, W, get_lin(m, "unet.conv_in"), 1, NULL, NULL);
    tfree(&x);
    emit(tap, user, "conv_in", &h);
    ten_t skips[12]; int ns = 0;
    skips[ns++] = h;
    for (int i = 0; i < 4; ++i) {
        for (int j = 0; j < 2; ++j) {
            snprintf(nm, sizeof nm, "unet.down_blocks.%d.resnets.%d", i, j);
            ten_t r = resnet(m, &h, H, W, nm); emit(tap, user, nm, &r);
            if (i < 3) {
                snprintf(nm, sizeof nm, "unet.down_blocks.%d.attentions.%d", i, j);
                ten_t t = transformer(m, &r, nm, HEADS[i]); emit(tap, user, nm, &t);
                tfree(&r); r = t;
            }
            h = r; skips[ns++] = h;
        }
        if (i < 3) {
            snprintf(nm, sizeof nm, "unet.down_blocks.%d.downsamplers.0.conv", i);
            h = conv3(&h, H, W, get_lin(m, nm), 2, NULL, NULL); emit(tap, user, nm, &h);
            H /= 2; W /= 2; skips[ns++] = h;
        }
    }
    ten_t r = resnet(m, &h, H, W, "unet.mid_block.resnets.0"); emit(tap, user, "unet.mid_block.resnets.0", &r);
    h = r;
    ten_t t = transformer(m, &h, "unet.mid_block.attentions.0", 20); emit(tap, user, "unet.mid_block.attentions.0", &t);
    tfree(&h); h = t;
    r = resnet(m, &h, H, W, "unet.mid_block.resnets.1"); emit(tap, user, "unet.mid_block.resnets.1", &r);
    tfree(&h); h = r;
    for (int i = 0; i < 4; ++i) {
        for (int j = 0; j < 3; ++j) {
            ten_t s = skips[--ns];
            ten_t c = talloc(h.B, h.T, h.C + s.C);
            or_concat(h.d, h.C, s.d, s.C, h.B * h.T, c.d);
            tfree(&h); tfree(&s);
            snprintf(nm, sizeof nm, "unet.up_blocks.%d.resnets.%d", i, j);
            h = resnet(m, &c, H, W, nm); emit(tap, user, nm, &h);
            tfree(&c);
            if (i > 0) {
                snprintf(nm, sizeof nm, "unet.up_blocks.%d.attentions.%d", i, j);
                t = transformer(m, &h, nm, HEADS[3 - i]); emit(tap, user, nm, &t);
                tfree(&h); h = t;
            }
        }
        if (i < 3) {
            ten_t u = talloc(h.B, h.T * 4, h.C);
            or_upsample2(h.d, h.B, H, W, h.C, u.d);
            tfree(&h); H *= 2; W *= 2;
            snprintf(nm, sizeof nm, "unet.up_blocks.%d.upsamplers.0.conv", i);
            h = conv3(&u, H, W, get_lin(m, nm), 1, NULL, NULL); emit(tap, user, nm, &h);
            tfree(&u);
        }
    }
    uint32_t* pmo;
    ten_t nrm = gn_silu(m, &h, "unet.conv_norm_out", &pmo);
    tfree(&h);
    ten_t eps = conv3(&nrm, H, W, get_lin(m, "unet.conv_out"), 1, NULL, pmo);
    tfree(&nrm); free(pmo);
    emit(tap, user, "eps", &eps);
    if (eps_out) memcpy(eps_out, eps.d, sizeof(int32_t) * (size_t)B * 16384);
    or_finalize(noise, eps.d, B, m->c_sig, x0);
    tfree(&eps); free(noise);
    return 0;
}
