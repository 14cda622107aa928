// Exact integer primitives of the PoI v2 arithmetic, device (and host) side.
//
// Same semantics as the reference's src/intops.cuh:9-66 (the consensus
// spec of the whole path); restated here from the definitions:
//   sat32      clamp to int32
//   rshr(v,s)  round-half-up arithmetic right shift for s >= 0 (shift capped
//              at 62), saturating left shift for s < 0 (|s| capped at 31,
//              operand clamped to +-2^(62-|s|)); result saturated to int32
//   row_exp(m) max(0, bitlen(m) - 15) for 0 <= m < 2^32
//   quant16    clamp(rshr(v, e), +-32767)
//   lut16      2049-entry Q16 table on [-16, 16), 10-bit linear interpolation,
//              0 below the range and 65536 above it
//   planes     q = 256*hi + lo + 128, hi = q >> 8, lo = (q & 255) - 128
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace vela {
typedef int64_t i64;
typedef uint32_t u32;

__host__ __device__ __forceinline__ i64 sat32(i64 v) { return v < INT32_MIN ? INT32_MIN : (v > INT32_MAX ? INT32_MAX : v); }

__host__ __device__ __forceinline__ i64 rshr(i64 v, i64 s) {
    if (s >= 0) {
        const int p = s > 62 ? 62 : int(s);
        return sat32((v + ((i64(1) << p) >> 1)) >> p);
    }
    const int n = -s > 31 ? 31 : int(-s);
    const i64 lim = i64(1) << (62 - n);
    const i64 c = v < -lim ? -lim : (v > lim ? lim : v);
    return sat32(c * (i64(1) << n));
}
// rshr for a shift known to lie in [1, 62]: one add and one shift, then saturate.
__device__ __forceinline__ i64 rshr_pos(i64 v, int s) { return sat32((v + (i64(1) << (s - 1))) >> s); }

__host__ __device__ __forceinline__ i64 floor_div(i64 a, i64 b) {
    i64 q = a / b;
    if ((a % b != 0) && ((a < 0) != (b < 0))) --q;
    return q;
}

__device__ __forceinline__ int row_exp(u32 m) { const int e = 17 - __clz(m); return e > 0 ? e : 0; }
__host__ __forceinline__ int row_exp_host(u32 m) { int e = 0; for (int k = 15; k < 32; ++k) e += (uint64_t(m) >= (uint64_t(1) << k)); return e; }

__device__ __forceinline__ u32 uabs(int v) { return v < 0 ? 0u - u32(v) : u32(v); }

// quant16 of an int32 for e in [0, 17]: floor((v + 2^(e-1)) / 2^e) = (v >> e) + bit (e-1) of v, no overflow.
__device__ __forceinline__ int quant16(int v, int e) {
    const int q = e ? (v >> e) + ((v >> (e - 1)) & 1) : v;
    return min(max(q, -32767), 32767);
}
// saturating int32 addition (sat32 of the exact sum)
__device__ __forceinline__ int add_sat(int a, int b) { int r; asm("add.sat.s32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b)); return r; }
// quant16 with the row's shift split as (s1, r, s2) = (e - 1, 1, 1) for e >= 1 and (0, 0, 0) for e = 0:
// ((v >> s1) + r) >> s2 = floor((v + 2^(e-1)) / 2^e) without overflow, then the +-32767 clamp.
__device__ __forceinline__ int quant16_fast(int v, int s1, int r, int s2) {
    return min(max(((v >> s1) + r) >> s2, -32767), 32767);
}
// Four int32 values quantised with the row's shift split (s1, r, s2) straight into their hi and lo plane bytes:
// the rounded shift in 32-bit, then pairs narrowed with saturation to 16 bits (cvt.pack.sat: the first source
// goes to the upper half), -32768 raised to -32767 on both halves at once (max.s16x2), and the byte selections.
__device__ __forceinline__ void quant_pack4(int v0, int v1, int v2, int v3, int s1, int r, int s2, uint32_t& hw, uint32_t& lw) {
    const int q0 = ((v0 >> s1) + r) >> s2, q1 = ((v1 >> s1) + r) >> s2, q2 = ((v2 >> s1) + r) >> s2, q3 = ((v3 >> s1) + r) >> s2;
    uint32_t w01, w23;
    asm("cvt.pack.sat.s16.s32 %0, %1, %2;" : "=r"(w01) : "r"(q1), "r"(q0));
    asm("cvt.pack.sat.s16.s32 %0, %1, %2;" : "=r"(w23) : "r"(q3), "r"(q2));
    asm("max.s16x2 %0, %0, %1;" : "+r"(w01) : "r"(0x80018001u));
    asm("max.s16x2 %0, %0, %1;" : "+r"(w23) : "r"(0x80018001u));
    hw = __byte_perm(w01, w23, 0x7531);
    lw = __byte_perm(w01, w23, 0x6420) ^ 0x80808080u;
}
// The same for a row exponent e <= 15 (h = 2^e >> 1): every |v| < 2^(15+e) <= 2^30, so v + h cannot overflow and
// floor((v + 2^(e-1)) / 2^e) is one add and one arithmetic shift.
__device__ __forceinline__ void quant_pack4_e15(int v0, int v1, int v2, int v3, int h, int e, uint32_t& hw, uint32_t& lw) {
    const int q0 = (v0 + h) >> e, q1 = (v1 + h) >> e, q2 = (v2 + h) >> e, q3 = (v3 + h) >> e;
    uint32_t w01, w23;
    asm("cvt.pack.sat.s16.s32 %0, %1, %2;" : "=r"(w01) : "r"(q1), "r"(q0));
    asm("cvt.pack.sat.s16.s32 %0, %1, %2;" : "=r"(w23) : "r"(q3), "r"(q2));
    asm("max.s16x2 %0, %0, %1;" : "+r"(w01) : "r"(0x80018001u));
    asm("max.s16x2 %0, %0, %1;" : "+r"(w23) : "r"(0x80018001u));
    hw = __byte_perm(w01, w23, 0x7531);
    lw = __byte_perm(w01, w23, 0x6420) ^ 0x80808080u;
}
// Whether a row whose largest magnitude is m (e = row_exp(m)) needs the +-32767 saturation at all: for e = 0 every
// |v| <= m < 2^15; for e >= 1 the rounded extremes (m + 2^(e-1)) >> e and (-m + 2^(e-1)) >> e stay inside +-32767
// exactly when m + 2^(e-1) < 2^(15+e).  Most rows qualify (only an m in the top 2^(e-1) of its binade does not).
__device__ __forceinline__ bool quant_nosat(u32 m, int e) {
    return e == 0 || uint64_t(m) + (uint64_t(1) << (e - 1)) < (uint64_t(1) << (15 + e));
}
// quant_pack4_e15 for such a row: the rounded values are 16-bit already, so their hi / lo plane bytes are bytes 1
// and 0 of the 32-bit results, gathered by four byte selections (lo bytes then offset by 128).
__device__ __forceinline__ void quant_pack4_e15_nosat(int v0, int v1, int v2, int v3, int h, int e, uint32_t& hw, uint32_t& lw) {
    const int q0 = (v0 + h) >> e, q1 = (v1 + h) >> e, q2 = (v2 + h) >> e, q3 = (v3 + h) >> e;
    const uint32_t a = __byte_perm(q0, q1, 0x4051), b = __byte_perm(q2, q3, 0x4051);   // [q0.b1 q1.b1 q0.b0 q1.b0] ...
    hw = __byte_perm(a, b, 0x5410);
    lw = __byte_perm(a, b, 0x7632) ^ 0x80808080u;
}
// hi bytes / lo bytes of four 16-bit values packed into one word each
__device__ __forceinline__ u32 pack_hi4(int q0, int q1, int q2, int q3) {
    return __byte_perm(__byte_perm(q0, q1, 0x0051), __byte_perm(q2, q3, 0x0051), 0x5410);
}
__device__ __forceinline__ u32 pack_lo4(int q0, int q1, int q2, int q3) {
    return __byte_perm(__byte_perm(q0, q1, 0x0040), __byte_perm(q2, q3, 0x0040), 0x5410) ^ 0x80808080u;
}

__device__ __forceinline__ int lut16(i64 x, const int32_t* __restrict__ L) {
    const i64 z = x + (i64(16) << 16);
    if (z < 0) return 0;
    if (z >= (i64(32) << 16)) return 65536;
    const int i = int(z >> 10), f = int(z & 1023);
    const int a = __ldg(L + i), b = __ldg(L + i + 1);
    return a + (((b - a) * f) >> 10);
}
// x * lut(x) / 2^16, rounded and saturated: SiLU / GELU of a Q16 value
__device__ __forceinline__ int lut_act(int x, const int32_t* __restrict__ L) { return int(rshr_pos(i64(x) * lut16(x, L), 16)); }

// lut16 / lut_act from the table staged in shared memory with sentinels: T[0] = (0, 0) for x below
// the range, T[1 + i] = (L[i], L[i+1] - L[i]) for i < 2048, T[2049] = (65536, 0) above it, so the range tests
// become one clamp of the index ((x >> 10) + 1024 = (x + 2^20) >> 10 without the overflow of the sum).
// Staged only when every L[i] lies in [0, 65536]: then x * lut(x) / 2^16 never exceeds |x| and needs no saturation.
constexpr int LUT_S_ENTRIES = 2050;
__device__ __forceinline__ int lut16_s(int x, const int2* __restrict__ T) {
    const int2 e = T[min(max((x >> 10) + 1024, -1), 2048) + 1];
    return e.x + ((e.y * (x & 1023)) >> 10);
}
__device__ __forceinline__ int lut_act_s(int x, const int2* __restrict__ T) {
    const i64 t = i64(x) * lut16_s(x, T) + 32768;
    return int(__funnelshift_r(uint32_t(t), uint32_t(t >> 32), 16));
}
// the same activation for a table with entries outside [0, 65536]: saturating
__device__ __forceinline__ int lut_act_s_sat(int x, const int2* __restrict__ T) { return int(rshr_pos(i64(x) * lut16_s(x, T), 16)); }
// stage the sentinel table T[LUT_S_ENTRIES] from L[2049] (block-strided); returns this thread's part of the
// "every entry in [0, 65536]" test, to be and-reduced over the block
__device__ __forceinline__ int stage_lut_s(int2* T, const int32_t* __restrict__ L) {
    int in_range = 1;
    for (int i = threadIdx.x; i < LUT_S_ENTRIES; i += blockDim.x) {
        int2 v = make_int2(i == 0 ? 0 : 65536, 0);
        if (i > 0 && i <= 2048) {
            const int x0 = __ldg(L + i - 1), x1 = __ldg(L + i);
            v = make_int2(x0, x1 - x0);
            in_range &= x0 >= 0 && x0 <= 65536 && x1 >= 0 && x1 <= 65536;
        }
        T[i] = v;
    }
    return in_range;
}

// Exact floor(sqrt(v)) for 0 <= v < 2^62: double seed, then integer correction.
__host__ __device__ __forceinline__ i64 isqrt(i64 v) {
    if (v <= 0) return 0;
    i64 s = i64(sqrt(double(v)));
    while (s > 0 && s * s > v) --s;
    while ((s + 1) * (s + 1) <= v) ++s;
    return s;
}

// GEMM epilogue y = sat32(rshr(acc * m, s - e) + b) with acc = 256*chi + clo + 128*wsum
__device__ __forceinline__ int epi_y(int chi, int clo, int m, int sh, int b, int wsum128) {
    const i64 acc = 256 * i64(chi) + clo + wsum128;
    const i64 v = acc * i64(m);
    const i64 r = (sh >= 1 && sh <= 62) ? rshr_pos(v, sh) : rshr(v, sh);
    return int(sat32(r + b));
}
// epi_y for a shift known to lie in [1, 31] and |m| < 2^23: the rounded shift of the 64-bit product is one funnel shift for the
// low word plus a test that the high word is its sign extension (else the value saturates); + b saturating.
// (clo + 128 wsum fits 32 bits: |clo|, |128 wsum| <= 128 * 127 * K < 2^30 for K <= 2^16.)
// The product is formed as two 32x32 -> 64-bit multiply-adds, chi * (256 m) + ((clo + 128 wsum) m + 2^(sh-1)), which
// needs |m| < 2^23 (the caller checks it per tile).
__device__ __forceinline__ int epi_y_fast(int chi, int clo, int m, int sh, int b, int wsum128) {
    const i64 t = i64(chi) * (m << 8) + (i64(clo + wsum128) * m + i64(1u << (sh - 1)));
    const int lo = int(__funnelshift_r(uint32_t(t), uint32_t(t >> 32), sh));
    const int hs = int(t >> 32) >> sh;
    return add_sat(hs == (lo >> 31) ? lo : (t < 0 ? INT32_MIN : INT32_MAX), b);
}
}  // namespace vela
