/*
 * vela oracle: a CPU restatement, in plain C, of the exact-integer inference
 * path of the reference miner (emanwrxsti/vela, "supr-meow-vela" 0.1.6).
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the CUDA path
 * is compared against, and the timed CPU baseline of bench.py.  Nothing in
 * the product (vela_b200/) links, loads or calls it.
 *
 * Every function states the reference file:line whose arithmetic it follows
 * (paths are relative to the reference project root).  All values are
 * integers; intermediate products are int64 exactly as in the reference.
 *
 * Pinning: the restatement is checked against outputs of the reference's own
 * kernels (compiled from the reference sources into oracle/_ref by
 * oracle/Makefile and run on a B200), committed as fixtures under
 * tests/golden/, and against the reference's CPU known-answer generators
 * (src/test_attn_score.cu, src/test_im2col.cu, src/test_normalization.cpp),
 * which tests/ re-run through this library.
 */
#ifndef VELA_ORACLE_H
#define VELA_ORACLE_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- primitives: src/intops.cuh:9-66 ---------------------------------- */
int64_t or_sat32(int64_t v);
int64_t or_rshr(int64_t v, int64_t s);
int64_t or_floor_div(int64_t a, int64_t b);
int     or_row_exp(int64_t m);
int64_t or_quant16(int64_t v, int e);
int32_t or_lut16(int64_t x, const int32_t* L);
int64_t or_isqrt(int64_t v);
/* exact attention score: sat32(rshr(S, sh)), the value src/attn.cu:65-83 computes */
int32_t or_score(int64_t S, int sh);
/* batch form of or_score for the known-answer test of src/test_attn_score.cu */
void or_score_batch(const int64_t* S, const int32_t* sh, int32_t* out, size_t n);

/* ---- GroupNorm statistics record, layout of struct GnStat (src/kernels.h:9) */
typedef struct { int64_t sum; int32_t mn, mx; int64_t mean; int32_t e; int32_t pad_; int64_t ss; int64_t sd; } or_gnstat_t;

/* ---- row quantisation: src/kernels.cu:42-57 (+ warp form :488-497) ------ */
/* rows [M, Mpad) are written as value 0 = (hi 0, lo -128); e is written for rows < M */
void or_quant_rows(const int32_t* X, int M, int K, int ldx, int8_t* hi, int8_t* lo, int32_t* e, int Kp, int Mpad);

/* ---- hi/lo GEMM with fused epilogues: src/gemm_hl.cu:40-52,175-309 ---- */
enum { OR_EPI_PLAIN = 0, OR_EPI_SPLIT3 = 1, OR_EPI_GEGLU = 2, OR_EPI_GELU = 3, OR_EPI_QKV = 4 };
typedef struct {
    int epi;
    int32_t* Y; int ldy; const int32_t* residual;
    int Cs; int32_t* Y1; int32_t* Y2; const int32_t* Lphi;
    uint32_t* rowmax;                  /* optional: max |y| per row (max-combined into existing values) */
    int heads, T, TpQ, TpK, C;         /* EPI_QKV */
    int8_t *qhi, *qlo, *khi, *klo; int32_t *qe, *ke;
    int64_t *qhs, *qls, *qts, *khs, *kls, *kts;
} or_epi_t;
/* cst[4n..4n+3] = {m, s, b, wsum}; A rows r < Mreal, columns n < Nreal */
void or_gemm_hl(const int8_t* Ahi, const int8_t* Alo, int lda, int Mreal,
                const int8_t* W, int ldw, int Nreal, int Kp,
                const int32_t* cst, const int32_t* e, const or_epi_t* E);
/* e of a SRC_X32 operand: row_exp(rowmax[r]) (src/gemm_hl.cu:102) */
void or_rowexp_u32(const uint32_t* rowmax, int M, int32_t* e);

/* ---- conv helpers: src/kernels.cu:106-170, src/gemm_hl.cu:335-341 ------ */
void or_pixmax(const int32_t* X, int rows, int C, uint32_t* pm);
void or_conv_e(const uint32_t* pm, int B, int H, int W, int stride, int32_t* e);
/* im2col with per-output-row quantisation, K index tap*C + c (tap-major); rows [rows, Mpad) value 0 */
void or_im2col3(const int32_t* X, const uint32_t* pm, int B, int H, int W, int C, int stride,
                int8_t* hi, int8_t* lo, int32_t* e, int Kp, int Mpad);

/* ---- GroupNorm / LayerNorm: src/kernels.cu:172-305,350-487 ------------- */
void or_gn_stats(const int32_t* X, int B, int T, int C, int groups, int64_t den, or_gnstat_t* gs);
/* apply (+ optional SiLU LUT); either int32 Y + pixel max pm, or planes hi/lo + e (when hi != NULL) */
void or_gn_apply_row(const int32_t* X, int B, int T, int C, int groups, const or_gnstat_t* gs,
                     const int32_t* g, const int32_t* beta, const int32_t* Lsig,
                     int32_t* Y, uint32_t* pm, int8_t* hi, int8_t* lo, int32_t* e, int Kp);
void or_lnorm_q(const int32_t* X, int M, int C, const int32_t* g, const int32_t* beta, int64_t den,
                int8_t* hi, int8_t* lo, int32_t* e, int Kp);
void or_lnorm(const int32_t* X, int M, int C, const int32_t* g, const int32_t* beta, int64_t den, int32_t* Y);

/* ---- elementwise: src/kernels.cu:537-561,592-607 ----------------------- */
void or_act(int32_t* X, size_t n, const int32_t* L);
void or_geglu(int32_t* A, const int32_t* G, size_t n, const int32_t* L);
void or_add(int32_t* X, const int32_t* Y, size_t n);
void or_concat(const int32_t* A, int Ca, const int32_t* Bm, int Cb, int rows, int32_t* out);
void or_upsample2(const int32_t* X, int B, int H, int W, int C, int32_t* out);
void or_chacha20_block(const uint8_t key[32], uint32_t counter, uint32_t out[16]);
void or_noise(const uint8_t* seeds, int B, const int32_t* gauss, int64_t cin, int32_t* n, int32_t* x);
void or_finalize(const int32_t* n, const int32_t* eps, int B, int64_t sig, uint8_t* out);
void or_text_embed(const int32_t* ids, int T, int rowsPad, const int8_t* tw, const int32_t* tm,
                   const int32_t* ts, const int32_t* pos, int D, int32_t* X);

/* ---- attention operands and exact attention: src/kernels.cu:611-722 ---- */
void or_quant_heads(const int32_t* X, int B, int T, int C, int heads, int Tp,
                    int8_t* hi, int8_t* lo, int32_t* e, int64_t* hs, int64_t* ls, int64_t* tsum);
void or_quant_v(const int32_t* X, int B, int Tk, int C, int heads, int Tkp,
                int8_t* vt_hi, int8_t* vt_lo, int32_t* ev, int64_t* vsum);
/* out[b, q, h*64+d] for q < Tq; rowmax optional (max-combined) */
void or_attention(const int8_t* qhi, const int8_t* qlo, const int32_t* eq, int Tqp,
                  const int8_t* khi, const int8_t* klo, const int32_t* ek,
                  const int8_t* vthi, const int8_t* vtlo, const int32_t* ev,
                  int B, int heads, int Tq, int Tk, int Tkp, int causal, const int32_t* Lexp,
                  int C, int32_t* out, uint32_t* rowmax);

/* ---- the UNet step on a POISD model file: src/engine.cu:11-101,389-609 - */
typedef struct or_model or_model_t;
or_model_t* or_model_load(const char* path, char* err, int errlen);
void        or_model_free(or_model_t* m);
/* set the prompt (text encoder + cross-attention K/V, src/engine.cu:491-574) */
int  or_set_prompt(or_model_t* m, const int32_t* tokens, int ntok);
/* the 77x1024 context after the text encoder (valid after or_set_prompt) */
const int32_t* or_context(const or_model_t* m);
/* one denoising step for B seeds (32 bytes each) -> x0 (32768 bytes each).
 * Optional taps (may be NULL): eps [B,4096,4] int32, and every activation
 * the UNet produces, in call order, handed to `tap(user, name, data, count)`. */
typedef void (*or_tap_fn)(void* user, const char* name, const int32_t* data, size_t count);
int  or_unet_step(or_model_t* m, const uint8_t* seeds, int B, uint8_t* x0, int32_t* eps_out,
                  or_tap_fn tap, void* user);
/* threads used by the OpenMP loops (0 = library default) */
void or_set_threads(int n);
/* Seeded random-init POISDv1 model (oracle/synth_model.c): the same bytes as the product's
 * vela_synth_model_write for the same seed.  0 on success. */
int or_synth_model_write(const char* path, uint64_t seed);
int  or_get_threads(void);

#ifdef __cplusplus
}
#endif
#endif
