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
