/*
 * vela_b200 -- C ABI of the B200 (sm_100a) integer UNet-step engine.
 *
 * Drop-in for the inference hot path of the Vela PoI v2 miner
 * (emanwrxsti/vela 0.1.6).  Each entry point replaces one function of the
 * reference's operator API (src/kernels.h, src/gemm_hl.h, src/attn.cu) or
 * engine API (src/engine.h); the reference interface it replaces is cited
 * beside it.  Conventions:
 *   - plain pointers and sizes only; device pointers unless stated "host";
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy stream);
 *   - every call returns VELA_OK (0) or a negative VELA_ERR_* status and
 *     never throws; vela_last_error() describes the last failure of the
 *     calling thread (the reference throws std::runtime_error instead,
 *     src/common.h:10-11);
 *   - activations are int32 row-major [rows, C] (NHWC for images); GEMM A
 *     operands are 16-bit values q stored as two int8 planes
 *     hi = q >> 8, lo = (q & 255) - 128 (q = 256 hi + lo + 128) plus a
 *     per-row power-of-two exponent e (src/intops.cuh:39,65-66).
 */
#ifndef VELA_B200_H
#define VELA_B200_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VELA_OK            0
#define VELA_ERR_ARG      -1   /* bad argument or unsupported shape */
#define VELA_ERR_CUDA     -2   /* CUDA runtime/driver error */
#define VELA_ERR_ARENA    -3   /* activation arena exhausted (src/engine.cu:108) */
#define VELA_ERR_TIMEOUT  -4   /* a bounded device-side wait gave up (device error flag set) */
#define VELA_ERR_IO       -5   /* model file missing, truncated or malformed */
#define VELA_ERR_STATE    -6   /* call out of order (no prompt, nothing in flight, ...) */

/* Description of the last failing call on this thread ("" if none). */
const char* vela_last_error(void);
/* Library version string. */
const char* vela_version(void);

/* GroupNorm statistics of one (sample, group); layout of struct GnStat (src/kernels.h:9). */
typedef struct vela_gnstat { int64_t sum; int32_t mn, mx; int64_t mean; int32_t e; int32_t pad_; int64_t ss; int64_t sd; } vela_gnstat;

/* Read (and with clear != 0 reset) the device error words of the current device: non-zero when a
 * bounded wait inside a kernel gave up (VELA_ERR_TIMEOUT class; no reference counterpart). */
unsigned vela_device_error(int clear);

/* ---------------------------------------------------------------------------------
 * W8A16 hi/lo GEMM on the sm_100a tensor cores.
 * ------------------------------------------------------------------------------ */
#define VELA_SRC_I8      0     /* planar int8 hi/lo rows + per-row e */
#define VELA_SRC_X32     1     /* int32 rows quantised on load with e = row_exp(rowmax[row]) */
#define VELA_SRC_CONV32  2     /* NHWC int32 image, implicit 3x3 pad-1 im2col, K = 9C tap-major (C % 32 == 0 or C == 4), e from vela_conv_e */
#define VELA_EPI_PLAIN   0     /* y (+ residual), optional per-row max |y| */
#define VELA_EPI_SPLIT3  1     /* column n -> (Y | Y1 | Y2)[row][n % Cs] */
#define VELA_EPI_GEGLU   2     /* interleaved a|g columns: Y[row][c] = a * GELU(g) / 2^16, optional row max */
#define VELA_EPI_GELU    3     /* y * GELU(y) / 2^16 (+ residual), optional row max */
#define VELA_EPI_QKV     4     /* merged q|k|v: q, k head-quantised (vela_quant_heads layout), v int32 */

/* A operand; struct ASrc of src/gemm_hl.h:13-18 */
typedef struct vela_asrc {
    int src;
    const int8_t* hi; const int8_t* lo; int ld8; const int32_t* e;
    const int32_t* x; int ldx; const uint32_t* rowmax; int K;
    const int32_t* img; int H, W, C, stride, Ho, Wo;
} vela_asrc;
/* Epilogue; struct AEpi of src/gemm_hl.h:19-25, plus an optional split-K workspace
 * (used when the output tiles cannot fill the GPU: 2 * splits * Mp * Np * 4 bytes). */
typedef struct vela_aepi {
    int epi; int32_t* Y; int ldy; const int32_t* residual;
    int Cs; int32_t* Y1; int32_t* Y2; const int32_t* Lphi;
    uint32_t* rowmax;
    int heads, T, TpQ, TpK, C;
    int8_t *qhi, *qlo, *khi, *klo; int32_t *qe, *ke; int64_t *qhs, *qls, *qts, *khs, *kls, *kts;
    void* workspace; size_t workspace_bytes;
} vela_aepi;

/* Y[r, n] = epi(sat32(rshr((256*Ahi[r].W[n] + Alo[r].W[n] + 128*wsum[n]) * m[n], s[n] - e[r]) + b[n])).
 * W int8 [Np, ldw] (K-major), cst int32 [Np][4] = {m, s, b, wsum}.  Mp rows of A are addressable,
 * Mreal rows and Nreal columns are computed.  Replaces k_gemm_hl2 (src/gemm_hl.h:27); all three A
 * sources and all five epilogues; deep K included (the reference's cuBLASLt path, src/engine.cu:153-157). */
int vela_gemm_w8a16(void* stream, const vela_asrc* A, int Mp, int Mreal, const int8_t* W, int ldw, int Np, int Nreal, int Kp,
                    const int32_t* cst, const vela_aepi* E);
/* Failure-path test entry (no reference counterpart; the reference's kernels have no bounded waits): the launch of
 * vela_gemm_w8a16 with its TMA producers idle and every barrier wait limited to wait_limit_cycles SM clock cycles, so
 * the waits run out, the kernel drains (nothing is in flight), frees its TMEM and returns; the timeout then reads
 * as non-zero from vela_device_error.  Outputs are left unwritten. */
int vela_gemm_w8a16_stalled(void* stream, const vela_asrc* A, int Mp, int Mreal, const int8_t* W, int ldw, int Np, int Nreal, int Kp,
                            const int32_t* cst, const vela_aepi* E, long long wait_limit_cycles);
/* Planar form; replaces k_gemm_hl (src/gemm_hl.h:31-33). */
int vela_gemm_hl(void* stream, const int8_t* Ahi, const int8_t* Alo, int lda, int Mp, int Mreal, const int8_t* W, int ldw, int Np, int Nreal, int Kp,
                 const int32_t* cst, const int32_t* e, int32_t* Y, int ldy, const int32_t* residual, int epi, int Cs, int32_t* Y1, int32_t* Y2,
                 const int32_t* Lphi);
/* e[row] = row_exp(max of pm over the 3x3 window); replaces k_conv_e (src/gemm_hl.h:29). */
int vela_conv_e(void* stream, const uint32_t* pm, int B, int H, int W, int stride, int32_t* e);

/* ---------------------------------------------------------------------------------
 * Row / memory-bound operators (src/kernels.h).  int64 arguments (den, cin, sig) and
 * int64 LUTs / parameters keep the reference's types.
 * ------------------------------------------------------------------------------ */
/* Per-row power-of-two quantisation of X[M, K] (row stride ldx) into hi/lo [*, Kp] + e[M]; columns
 * [K, Kp) and rows [M, align32(M)) are written as the value 0.  k_quant_rows (src/kernels.h:14). */
int vela_quant_rows(void* stream, const int32_t* X, int M, int K, int ldx, int8_t* hi, int8_t* lo, int32_t* e, int Kp);
/* vela_quant_rows with the row maxima already known (rowmax[r] = max_c |X[r, c]|, as the producing GEMM epilogues
 * and norms write them): e[r] = the exponent of rowmax[r], rows [M, Mpad) written as the value 0; K % 4 == 0.
 * No reference counterpart (the reference's engine re-reads each row for its maximum). */
int vela_quant_rows_rm(void* stream, const int32_t* X, const uint32_t* rowmax, int M, int K, int ldx, int8_t* hi, int8_t* lo, int32_t* e, int Kp, int Mpad);
/* pm[r] = max_c |X[r, c]|.  k_pixmax (src/kernels.h:19). */
int vela_pixmax(void* stream, const int32_t* X, int rows, int C, uint32_t* pm);
/* 3x3 pad-1 im2col with per-output-pixel quantisation, K index tap*C + c.  k_im2col3 (src/kernels.h:21-22). */
int vela_im2col3(void* stream, const int32_t* X, const uint32_t* pm, int B, int H, int W, int C, int stride, int8_t* hi, int8_t* lo, int32_t* e, int Kp);
/* GroupNorm statistics of X[B, T, C] (32 groups): the complete GnStat records.  k_gn_stats1 + k_gn_stats2 (src/kernels.h:24-29). */
int vela_gn_stats(void* stream, const int32_t* X, int B, int T, int C, int groups, long long den, vela_gnstat* gs);
/* GroupNorm apply (+ optional SiLU LUT): int32 Y + pixel max pm, or (hi != NULL) planes + e.  k_gn_apply_row (src/kernels.h:61-62). */
int vela_gn_apply_row(void* stream, const int32_t* X, int B, int T, int C, int groups, const vela_gnstat* gs, const int32_t* g, const int32_t* beta,
                      const int32_t* Lsig, int32_t* Y, uint32_t* pm, int8_t* hi, int8_t* lo, int32_t* e, int Kp);
/* LayerNorm rows of X[M, C] -> quantised planes + e.  k_lnorm_q (src/kernels.h:59). */
int vela_lnorm_q(void* stream, const int32_t* X, int M, int C, const int32_t* g, const int32_t* beta, long long den, int8_t* hi, int8_t* lo, int32_t* e, int Kp);
/* LayerNorm rows of X[M, C] -> int32.  k_lnorm (src/kernels.h:31). */
int vela_lnorm(void* stream, const int32_t* X, int M, int C, const int64_t* g, const int64_t* beta, long long den, int32_t* Y);
/* x = sat32(rshr(x * lut(x), 16)) in place.  k_act (src/kernels.h:32). */
int vela_act(void* stream, int32_t* X, size_t n, const int32_t* L);
/* a = sat32(rshr(a * gelu(g), 16)).  k_geglu (src/kernels.h:33). */
int vela_geglu(void* stream, int32_t* A, const int32_t* G, size_t n, const int32_t* L);
/* x = sat32(x + y).  k_add (src/kernels.h:34). */
int vela_add(void* stream, int32_t* X, const int32_t* Y, size_t n);
/* out[r] = [A[r] | B[r]] (Ca, Cb multiples of 4).  k_concat (src/kernels.h:35). */
int vela_concat(void* stream, const int32_t* A, int Ca, const int32_t* Bm, int Cb, int rows, int32_t* out);
/* nearest x2 upsample of NHWC X.  k_upsample2 (src/kernels.h:36). */
int vela_upsample2(void* stream, const int32_t* X, int B, int H, int W, int C, int32_t* out);
/* ChaCha20(seed) keystream -> u16 -> gauss LUT -> n [B,4,4096] channel-major, x = rshr(n*cin, 30) NHWC.  k_noise (src/kernels.h:38). */
int vela_noise(void* stream, const uint8_t* seeds, int B, const int64_t* gauss, long long cin, int32_t* n, int32_t* x);
/* x0 = rshr((n - eps)*sig, 16); out = clamp(rshr(x0, 8)) int16 LE [B, 32768 bytes].  k_finalize (src/kernels.h:40). */
int vela_finalize(void* stream, const int32_t* n, const int32_t* eps, int B, long long sig, uint8_t* out);
/* token embedding + position.  k_text_embed (src/kernels.h:42). */
int vela_text_embed(void* stream, const int32_t* ids, int T, int rowsPad, const int8_t* tw, const int64_t* tm, const int64_t* ts, const int64_t* pos, int D, int32_t* X);
/* Q/K head quantisation [G, Tp, 64] + e, hs, ls, tsum; rows t >= T value 0.  k_quant_heads (src/kernels.h:45-46). */
int vela_quant_heads(void* stream, const int32_t* X, int B, int T, int C, int heads, int Tp, int8_t* hi, int8_t* lo, int32_t* e, int64_t* hs, int64_t* ls, int64_t* tsum);
/* rows [T, Tp) of G head-quantised operands set to the value 0.  k_quant_heads_pad (src/kernels.h:57). */
int vela_quant_heads_pad(void* stream, int G, int T, int Tp, int8_t* hi, int8_t* lo, int32_t* e, int64_t* hs, int64_t* ls, int64_t* tsum);
/* V column quantisation, transposed [G, 64, Tkp] + ev, vsum; scratch u32[G*64].  k_quant_v (src/kernels.h:49-50). */
int vela_quant_v(void* stream, const int32_t* X, int B, int Tk, int C, int heads, int Tkp, int8_t* vt_hi, int8_t* vt_lo, int32_t* ev, int64_t* vsum, uint32_t* scratch);
/* vela_quant_v for callers that must not allocate device memory (no counterpart in the reference): the same
 * outputs, with the column-max scratch in a library-owned static device array of VELA_QUANT_V_STATIC_MAX_COLS
 * words (256 KiB per GPU, held until exit) instead of a caller buffer.  Requires B*heads*64 <= that maximum
 * (VELA_ERR_ARG otherwise).  The first call on a device looks up the array's device address; make it before any
 * stream capture.  All calls on a device share the array: calls that overlap on the GPU race, so order them on
 * one stream.  The address stays cached for the life of the process: do not call it on a device after resetting
 * that device (cudaDeviceReset). */
#define VELA_QUANT_V_STATIC_MAX_COLS 65536
int vela_quant_v_static(void* stream, const int32_t* X, int B, int Tk, int C, int heads, int Tkp, int8_t* vt_hi, int8_t* vt_lo, int32_t* ev, int64_t* vsum);

/* ---------------------------------------------------------------------------------
 * Exact integer attention on the tensor cores.
 * ------------------------------------------------------------------------------ */
/* out[b, q, h*64 + d] for q < Tq (+ row max |out| into rowmax, optional) from head-quantised Q
 * [G, Tqp, 64] (+ eq, qhs, qls), K [G, Tkp, 64] (+ ek, ksum = true-value row sums) and V^T
 * [G, 64, Tkp] (+ ev, vsum); G = B * heads; Tqp, Tkp multiples of 64, Tk <= Tkp <= 4096.
 * lexp32 is the exp LUT (>= 1025 int32 entries).  Replaces k_fused_attention (src/kernels.h:72-78);
 * gmx / gr (the reference's between-pass scratch) are accepted and unused: one CTA runs all three
 * exact passes of a query tile, so the row maxima and reciprocals stay in registers. */
int vela_fused_attention(void* stream, const int8_t* qhi, const int8_t* qlo, const int32_t* eq, const int64_t* qhs, const int64_t* qls,
                         const int8_t* khi, const int8_t* klo, const int32_t* ek, const int64_t* ksum,
                         const int8_t* vthi, const int8_t* vtlo, const int32_t* ev, const int64_t* vsum,
                         int B, int heads, int Tq, int Tqp, int Tk, int Tkp, int causal, const int32_t* lexp32, int C,
                         int32_t* gmx, int64_t* gr, int32_t* out, uint32_t* rowmax);

/* Failure-path test entry (no reference counterpart): vela_fused_attention with its TMA producer idle and every
 * wait limited to wait_limit_cycles SM clock cycles; the kernel drains and returns, vela_device_error reads non-zero. */
int vela_fused_attention_stalled(void* stream, const int8_t* qhi, const int8_t* qlo, const int32_t* eq, const int64_t* qhs, const int64_t* qls,
                                 const int8_t* khi, const int8_t* klo, const int32_t* ek, const int64_t* ksum,
                                 const int8_t* vthi, const int8_t* vtlo, const int32_t* ev, const int64_t* vsum,
                                 int B, int heads, int Tq, int Tqp, int Tk, int Tkp, int causal, const int32_t* lexp32, int C,
                                 int32_t* out, uint32_t* rowmax, long long wait_limit_cycles);

/* ---------------------------------------------------------------------------------
 * Engine: one denoising step of the SD-turbo UNet per batch (src/engine.h:16-124).
 * A model holds the prepared weights of one GPU and is shared read-only by its engines; an engine
 * (one per host thread, the reference's "lane") owns a stream, an activation arena and two
 * pipeline slots, each with its own CUDA graph of the whole step and pinned I/O buffers.
 * ------------------------------------------------------------------------------ */
typedef struct vela_model vela_model;
typedef struct vela_engine vela_engine;
typedef struct vela_engine_config {
    int batch;              /* inferences per step (EngineConfig::batch) */
    int graph;              /* 1: replay one CUDA graph per slot (EngineConfig::graph); 0: eager launches */
    size_t arena_bytes;     /* activation arena; 0 = 1 GiB + 512 MiB per inference */
} vela_engine_config;
typedef void (*vela_tap_fn)(void* user, const char* name, const int32_t* data, size_t count);

/* Load a POISD model file onto `device` (DevModel::load, src/engine.cu:11-70). NULL on failure. */
vela_model* vela_model_load(int device, const char* path);
/* The same from a POISD file image already in host memory (DevModel::load(int, const Poisd&), src/engine.h:18 --
 * the reference's host parses the file once and hands the parsed model to every GPU).  The image is read during
 * the call only.  NULL on failure. */
vela_model* vela_model_load_memory(int device, const uint8_t* image, size_t bytes);
void vela_model_free(vela_model* m);
size_t vela_model_bytes(const vela_model* m);
/* Engine(dm, cfg) (src/engine.cu:114-129). NULL on failure. */
vela_engine* vela_engine_create(const vela_model* m, const vela_engine_config* cfg);
void vela_engine_destroy(vela_engine* e);
/* Text encoder + cross-attention K/V of a prompt of BPE token ids (Engine::setPrompt, src/engine.cu:528-574). */
int vela_engine_set_prompt(vela_engine* e, const int32_t* tokens, int n);
/* host: the 77 x 1024 int32 context of the current prompt (the text encoder's output). */
int vela_engine_context(vela_engine* e, int32_t* ctx);
/* host seeds [batch][32] -> host x0 [batch][32768] (int16 LE), synchronous (Engine::run, src/engine.cu:650-677). */
int vela_engine_run(vela_engine* e, const uint8_t* seeds, uint8_t* x0);
/* two batches in flight: submit enqueues (Engine::submit), collect waits for the oldest (Engine::collect). */
int vela_engine_submit(vela_engine* e, const uint8_t* seeds);
int vela_engine_collect(vela_engine* e, uint8_t* x0);
/* one eager step handing every block output (host int32) to `tap` in UNet order (no reference counterpart: parity taps). */
int vela_engine_step_taps(vela_engine* e, const uint8_t* seeds, uint8_t* x0, vela_tap_fn tap, void* user);
/* Device-resident form of one step (no reference counterpart: the reference's forwardIO always copies the seeds
 * from and x0 to pinned host memory, src/engine.cu:599-609).  d_seeds [batch][32] and d_x0 [batch][32768] are
 * device pointers on the engine's device.  The step is enqueued on vela_engine_stream() and the call returns
 * without waiting; the first call captures its CUDA graph. */
int vela_engine_launch_device(vela_engine* e, const uint8_t* d_seeds, uint8_t* d_x0);
/* kernel nodes in the engine's last captured step graph (0 before the first capture; no reference counterpart) */
int vela_engine_graph_kernels(const vela_engine* e);
/* The engine's own device error word (its kernels report a timed-out bounded wait there; a step whose kernels did
 * makes vela_engine_collect / vela_engine_run return VELA_ERR_TIMEOUT).  Synchronises the engine's stream;
 * clear != 0 resets the word.  No reference counterpart (the reference's kernels have no bounded waits). */
unsigned vela_engine_device_error(vela_engine* e, int clear);
/* Self-check of the attention kernel (Engine::testAttention, src/engine.cu:575-597): seeded activations of random
 * bit width 1..bits (0: zeros) for Q [B, Tq, 64 heads] and K, V [B, Tk, 64 heads], quantised by the library, then the
 * tiled kernel against the exact definition written as plain GPU loops; returns the number of differing output
 * words, or -1 on error.  No batches may be in flight. */
long long vela_engine_test_attention(vela_engine* e, int B, int Tq, int Tk, int heads, int causal, int bits);
int vela_engine_in_flight(const vela_engine* e);
int vela_engine_batch(const vela_engine* e);
size_t vela_engine_arena_peak(const vela_engine* e);
void* vela_engine_stream(const vela_engine* e);
double vela_engine_last_ms(const vela_engine* e);   /* device time of the last vela_engine_run, ms */

/* ---------------------------------------------------------------------------------
 * Host share hashing (the reference's mining / verify path; FIPS 180-4 SHA-256 on the host, no CUDA).
 * ------------------------------------------------------------------------------ */
/* sha256d(data) = SHA-256(SHA-256(data)) (meow::sha256d, src/sha256.h:84). */
int vela_sha256d(const uint8_t* data, size_t n, uint8_t* out32);
/* the proof-of-inference output hash of one inference: the tagged hash "POI/out" over seed[32] || x0[32768]
 * (poiOut, src/main.cpp:79; TaggedHasher, src/sha256.h:86-91). */
int vela_poi_out(const uint8_t* seed32, const uint8_t* x0, uint8_t* out32);
/* vela_poi_out over a batch (seeds [batch][32], x0 [batch][32768], out [batch][32]) on up to `threads` host
 * threads (the per-inference loop of src/main.cpp:139 and 262). */
int vela_poi_out_batch(const uint8_t* seeds, const uint8_t* x0, int batch, int threads, uint8_t* out);
/* the share hash: sha256d(header[80] || poi[32]) (src/main.cpp:263-264). */
int vela_share_hash(const uint8_t* header80, const uint8_t* poi32, uint8_t* out32);

/* ---------------------------------------------------------------------------------
 * Tooling (no reference counterpart): seeded random-init model in the POISDv1
 * format the reference loads (src/poisd.cpp:17-35), with every tensor of the
 * SD-2.1 UNet and 23-layer text encoder.  Host path.  ~1.19 GB.
 * ------------------------------------------------------------------------------ */
int vela_synth_model_write(const char* path, uint64_t seed);

#ifdef __cplusplus
}
#endif
#endif
