// Host launchers of every kernel (internal; the C ABI in vela_b200.h wraps them with status codes).
// All throw vela::Error on bad arguments; none synchronises or allocates.
#pragma once
#include "vela_b200.h"
#include "host_util.h"
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace vela {
typedef int64_t i64;
void gemm_w8a16(cudaStream_t st, const vela_asrc& A, int Mp, int Mreal, const int8_t* W, int ldw, int Np, int Nreal, int Kp,
                const int32_t* cst, const vela_aepi& E, const LaunchOpts& o = LaunchOpts());
void conv_e(cudaStream_t st, const uint32_t* pm, int B, int H, int W, int stride, int32_t* e);
void quant_rows(cudaStream_t st, const int32_t* X, int M, int K, int ldx, int8_t* hi, int8_t* lo, int32_t* e, int Kp);
// quant_rows with the row maxima given (row_exp(rowmax[r]) = the row's exponent); rows [M, Mpad) zero-valued
void quant_rows_rm(cudaStream_t st, const int32_t* X, const uint32_t* rowmax, int M, int K, int ldx, int8_t* hi, int8_t* lo, int32_t* e, int Kp, int Mpad);
void pixmax(cudaStream_t st, const int32_t* X, int rows, int C, uint32_t* pm);
void im2col3(cudaStream_t st, const int32_t* X, const uint32_t* pm, int B, int H, int W, int C, int stride, int8_t* hi, int8_t* lo, int32_t* e, int Kp);
void gn_stats(cudaStream_t st, const int32_t* X, int B, int T, int C, i64 den, vela_gnstat* gs);
void gn_apply(cudaStream_t st, const int32_t* X, int B, int T, int C, const vela_gnstat* gs, const int32_t* g, const int32_t* beta,
              const int32_t* Lsig, int32_t* Y, uint32_t* pm, int8_t* hi, int8_t* lo, int32_t* e, int Kp);
void lnorm_q(cudaStream_t st, const int32_t* X, int M, int C, const int32_t* g, const int32_t* beta, i64 den, int8_t* hi, int8_t* lo, int32_t* e, int Kp);
void lnorm(cudaStream_t st, const int32_t* X, int M, int C, const i64* g, const i64* beta, i64 den, int32_t* Y);
void act(cudaStream_t st, int32_t* X, size_t n, const int32_t* L);
void geglu(cudaStream_t st, int32_t* A, const int32_t* G, size_t n, const int32_t* L);
void add(cudaStream_t st, int32_t* X, const int32_t* Y, size_t n);
void concat(cudaStream_t st, const int32_t* A, int Ca, const int32_t* Bm, int Cb, int rows, int32_t* out);
void upsample2(cudaStream_t st, const int32_t* X, int B, int H, int W, int C, int32_t* out);
void noise(cudaStream_t st, const uint8_t* seeds, int B, const i64* gauss64, const int32_t* gauss32, i64 cin, int32_t* n, int32_t* x);
void finalize(cudaStream_t st, const int32_t* n, const int32_t* eps, int B, i64 sig, uint8_t* out);
void text_embed(cudaStream_t st, const int32_t* ids, int T, int rowsPad, const int8_t* tw, const i64* tm, const i64* ts, const i64* pos, int D, int32_t* X);
void quant_heads(cudaStream_t st, const int32_t* X, int B, int T, int C, int heads, int Tp, int8_t* hi, int8_t* lo, int32_t* e, i64* hs, i64* ls, i64* tsum, int tFrom);
void quant_v(cudaStream_t st, const int32_t* X, int B, int Tk, int C, int heads, int Tkp, int8_t* vh, int8_t* vl, int32_t* ev, i64* vsum, uint32_t* colmax);
void fused_attention(cudaStream_t st, const int8_t* qhi, const int8_t* qlo, const int32_t* eq, const i64* qhs, const i64* qls,
                     const int8_t* khi, const int8_t* klo, const int32_t* ek, const i64* ksum,
                     const int8_t* vthi, const int8_t* vtlo, const int32_t* ev, const i64* vsum,
                     int B, int heads, int Tq, int Tqp, int Tk, int Tkp, bool causal, const int32_t* lexp, int C, int32_t* out, uint32_t* rowmax,
                     const LaunchOpts& o = LaunchOpts());
// the exact definition as plain loops on the GPU (one thread per query), for checking fused_attention
void attention_plain(cudaStream_t st, const int8_t* qhi, const int8_t* qlo, const int32_t* eq, int Tqp, const int8_t* khi, const int8_t* klo,
                     const int32_t* ek, const int8_t* vhi, const int8_t* vlo, const int32_t* ev, int B, int heads, int Tq, int Tk, int Tkp,
                     bool causal, const int32_t* lexp, int C, int32_t* out);
}  // namespace vela
