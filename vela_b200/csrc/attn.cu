// Exact integer attention on the sm_100a tensor cores (tcgen05.mma kind::i8).
//
// Semantics: the reference's fused attention (src/attn.cu:1-6,113-320; the plain-loop
// statement is src/kernels.cu:671-722).  For query row q and key k of one (batch, head):
//     S  = sum_d Q_d K_d over the 16-bit values (Q = 256 qh + ql + 128, K likewise)
//     s  = sat32(rshr(S, 19 - eq - ek)),  mx = max over valid keys of s
//     E  = expLUT(mx - s) (0 when mx - s >= 2^20),  r = floor(2^62 / sum E)
//     P  = min(32767, (E r + 2^46) >> 47),  O_d = sum_k P V_kd,  out = rshr(O_d, 15 - ev_d)
// Exactness needs the final row max and sum before any P is rounded, so every key tile is
// scored three times (max, sum, P.V); the score matrix is never written anywhere.
//
// One CTA = one (batch, head) x 128 query rows, all three passes, so the row max and r stay in
// registers.  Products on the tensor core with signed int8 planes only:
//     S = 65536 HH + 256 X + LL + (32768 qhs + 128 qls) + 128 ksum_k
//       HH = Qh.Kh, X = Qh.Kl + Ql.Kh, LL = Ql.Kl  (three s32 TMEM accumulators, N = 64 keys)
//     O = 65536 A + 256 Y + D + 128 (sum_k P + vsum_d) - 16384 n
//       P = 256 ph + pl + 128 with ph = P >> 8, pl = (P & 255) - 128 written to shared memory by the
//       softmax warps as the A operand; A = Ph.Vh, Y = Ph.Vl + Pl.Vh, D = Pl.Vl (K-major V^T tiles);
//       n = number of keys swept (padded keys carry V = 0 and P = 0).
//     sum_k P comes from the tensor core too: the V^T tiles have 16 constant rows below the 64 dims (N = 80), row 64
//       of the lo plane all ones and the rest zero, so column 64 holds Y = sum ph and D = sum pl, and
//       sum P = 256 Y + D + 128 n.
// Softmax arithmetic per score element (the CUDA-core work that bounds the kernel): the score in 32-bit wrapping
// arithmetic as hh M + (T >> a) (see div_pow2), the exp-table index and fraction taken from mx 2^b - that quotient
// without forming the score itself (see exp_fast_d), the table interpolated with one mad.hi on entries
// (L[i], 2 (L[i+1] - L[i])), and P from two multiply-adds of E with the 64-bit reciprocal's halves, saturated to
// 32767 by the packing instruction; the integer work is split between the ALU and FMA pipes.  A per-stage aux warp
// turns each K tile's ksum into int32 and classifies the 16-key quarters (exponent form, masking) once per CTA, so
// the softmax warps read one word per tile.
// Warp roles: warp 0 TMA (Q once; K tiles + per-key ek/ksum each pass; V^T tiles in pass 2),
// warp 1 TMEM allocation + MMA issue, warp 18 per-stage key data, warps 2..17 softmax (thread = one query row = one TMEM
// lane; the four warps of a lane quarter split each 64-key tile, and the output dims, in quarters).
// TMEM: QK buffers at columns [0,192) and [192,384) (passes 0-1 alternate; pass 2 uses the first),
// P.V accumulators A, Y, D at [192,272), [272,352), [352,432) during pass 2.  All barrier waits are bounded.
#include "intops.cuh"
#include "tc.cuh"
#include "host_util.h"
#include "ops.h"
#include "vela_b200.h"
#include <climits>
#include <cstring>

namespace vela {
namespace {

static __device__ unsigned g_attn_err;

constexpr int KS = 4, VS = 2;                         // K and V ring depths
constexpr int Q_BYTES = 128 * 64;                     // one plane of the 128-query tile
constexpr int KT_BYTES = 64 * 64;                     // one plane of a 64-key tile
constexpr int KSTAGE = 2 * KT_BYTES;                  // K hi + lo
constexpr int PV_N = 80;                              // P.V MMA width: 64 output dims + 16 constant rows (sum P)
constexpr int VT_BYTES = PV_N * 64;                   // one plane of a V^T tile: 64 dims from TMA, then the constant rows
constexpr int VSTAGE = 2 * VT_BYTES;                  // V^T hi + lo
constexpr int P_BYTES = 128 * 64;                     // one plane of P
// shared memory map (offsets from a 1024-aligned base)
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + 2 * Q_BYTES;
constexpr int OFF_V = OFF_K + KS * KSTAGE;
constexpr int OFF_P = OFF_V + VS * VSTAGE;
constexpr int OFF_KAUX = OFF_P + 2 * P_BYTES;          // per K stage: ek int32[64], ksum int64[64] (TMA), then the aux
constexpr int KAUX_TMA = 64 * 4 + 64 * 8;              // warp's kc int32[64] (= 128 ksum) and one info word per 16-key quarter
constexpr int KAUX_KC = KAUX_TMA, KAUX_QI = KAUX_KC + 64 * 4;
constexpr int KAUX_BYTES = KAUX_QI + 4 * 4;
// quarter info word: bits 0-7 the largest key exponent, bits 8-9 the form (0: one exponent; 1: exponents differ;
// 2: some shift of the CTA's rows falls outside [5, 19]), bit 10: every key valid (no causal mask, none past Tk)
constexpr int QI_MODE = 8, QI_FULL = 1 << 10;
// P.V accumulator columns in TMEM
constexpr uint32_t PV_A = 192, PV_Y = PV_A + PV_N, PV_D = PV_Y + PV_N;
constexpr int OFF_LUT = OFF_KAUX + KS * KAUX_BYTES;    // int2[1025] exp table (see exp_fast_d / exp_general); entry 1024 = (0, 0)
constexpr int SW = 16;                                 // softmax warps: four per TMEM lane quarter, 16 keys each
constexpr int AUX_WARP = 2 + SW;                      // per K stage: kc and the quarters' info words, once per CTA
constexpr int THREADS = 32 * (3 + SW);
constexpr int OFF_RED = OFF_LUT + 1032 * 8;            // cross-warp reductions: 4 x 128 x 8 bytes
constexpr int OFF_BAR = OFF_RED + 4 * 128 * 8;
constexpr int NBAR = 1 + 3 * KS + 2 * VS + 2 + 2 + 2 + 1;
constexpr int SMEM = 1024 + OFF_BAR + NBAR * 8 + 16;
constexpr int TMEM_COLS = 512;
static_assert(PV_D + PV_N <= TMEM_COLS && OFF_V % 1024 == 0 && VT_BYTES % 1024 == 0 && KAUX_BYTES % 16 == 0, "layout");

// Constants the softmax multiplies by, passed as kernel arguments so the compiler keeps the multiply forms on the FMA
// pipe instead of turning them into shifts and adds on the ALU pipe: 256, 8.
struct OpK { int c256, c8; };

struct AttnArgs {
    CUtensorMap tmQh, tmQl, tmKh, tmKl, tmVh, tmVl;
    const int32_t* eq; const i64* qhs; const i64* qls;
    const int32_t* ek; const i64* ksum;
    const int32_t* ev; const i64* vsum;
    const int32_t* lexp;
    int32_t* out; uint32_t* rowmax;
    int heads, Tq, Tqp, Tk, Tkp, C, causal;
    unsigned* err;
    long long wait_limit;          // SM clock cycles before a barrier wait gives up
    int stall;                     // failure-path tests: the TMA producer issues nothing
    OpK k;                         // the constants 256 and 8 (see OpK)
};

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// ---- integer building blocks with a chosen pipe.  The softmax's integer work is split between the two integer pipes
// of the SM sub-partition (each issues a warp instruction every other cycle): multiplies, multiply-highs (right shifts
// by a power of two) and multiply-adds run on the FMA pipe, adds / min / max / logic / funnel shifts on the ALU pipe.
// The multipliers that are powers of two come from kernel arguments (OpK), so the compiler keeps the multiply forms.
// Measured on B200: mad.lo, shifts, prmt, min and adds issue at half the warp rate; mad.hi / mul.hi at a quarter, so
// right shifts stay shifts.
__device__ __forceinline__ int mad_lo(int a, int b, int c) { int d; asm("mad.lo.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d; }
__device__ __forceinline__ int mul_lo(int a, int b) { int d; asm("mul.lo.s32 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b)); return d; }
__device__ __forceinline__ int mad_hi(int a, int b, int c) { int d; asm("mad.hi.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d; }
__device__ __forceinline__ uint32_t mad_hi_u(uint32_t a, uint32_t b, uint32_t c) { uint32_t d; asm("mad.hi.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d; }
__device__ __forceinline__ uint32_t mad_lo_u(uint32_t a, uint32_t b, uint32_t c) { uint32_t d; asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d; }
__device__ __forceinline__ int2 lds_v2(uint32_t addr) { int2 v; asm("ld.shared.v2.s32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr)); return v; }

// ---- score arithmetic (fast forms; every shift sh = 19 - eq - ek of the chunk lies in [5, 19])
// s = floor((65536 hh + T) / 2^sh) with T = 256 xx + ll + cq + 128 ksum + 2^(sh-1) (the rounding term included; |T| < 2^31)
// is computed in 32 bits as  s = (hh M + (T >> a)) >> b  with a = min(sh, 16), b = sh - a, M = 2^(16 - a):
//   sh <= 16: 65536 hh = 2^sh (hh M), so the quotient is hh M + floor(T / 2^sh);
//   sh > 16:  floor(floor((65536 hh + T) / 2^16) / 2^b) = (hh + (T >> 16)) >> b.
// |s| < 2^31 (|S| < 2^36, sh >= 5), so hh M + (T >> a) is formed modulo 2^32: an intermediate wrap cancels.
// A chunk whose keys have different exponents takes the smallest shift sh0 = 19 - eq - max ek for the division
// and shifts each key's result right by the remainder d = max ek - ek (nested floors), with each key's own rounding
// term 2^(19 - eq - ek - 1) in T.
struct ShiftSplit { int a, b; int M; };
__device__ __forceinline__ ShiftSplit split_shift(int sh) {
    const int a = min(sh, 16);
    return ShiftSplit{a, sh - a, 1 << (16 - a)};
}
__device__ __forceinline__ int div_pow2(int hh, int T, const ShiftSplit& p) { return mad_lo(hh, p.M, T >> p.a); }

// ---- exp table: E = L[i] + floor((L[i+1] - L[i]) f / 2^10) for z = mx - s, i = min(z, 2^20) >> 10, f = its low 10 bits
// (index 1024 is a sentinel (0, 0): E = 0 from z = 2^20 on).  Fast table (every L[i] in [0, 2^32 / 3], so three E add
// up in 32 bits, and every difference below 2^30 in magnitude): entries (L[i], 2 (L[i+1] - L[i])) and
// E = hi32(2 D * f 2^21) + L[i] in one mad.hi.  General table: entries (L[i], L[i+1]) and the difference in 64 bits,
// exactly as the reference does.
//
// The fast form reads i and f without forming s or z.  With the score s = u >> b (u = hh M + (T >> a), b in [0, 3]) and
// mxb = mx 2^b + 2^b - 1:  d = mxb - u >= 0 for every valid key and d >> b = mx - floor(u / 2^b) = z
// (ceil((u - 2^b + 1) / 2^b) = floor(u / 2^b)), so i = min(d >> (b + 10), 1024) and f 2^21 = (d 2^(21 - b)) & (1023 << 21).
// |u| < 2^21 when b > 0, so mx 2^b cannot wrap; with b = 0 the quotient is the score and d = z modulo 2^32.  An invalid
// key's d is arbitrary, its index still lies in [0, 1024] and its E is masked afterwards.
struct ExpIdx { int shi, mulf; };                          // b + 10 and 2^(21 - b)
__device__ __forceinline__ ExpIdx exp_idx(int b) { return ExpIdx{b + 10, 1 << (21 - b)}; }
__device__ __forceinline__ int exp_fast_d(uint32_t d, const ExpIdx& x, uint32_t lut_addr, const OpK& k) {
    const uint32_t i = min(d >> x.shi, 1024u);
    const int2 e = lds_v2(uint32_t(mad_lo(int(i), k.c8, int(lut_addr))));
    return mad_hi(e.y, int(uint32_t(mul_lo(int(d), x.mulf)) & 0x7FE00000u), e.x);
}
__device__ __forceinline__ uint32_t zclamp(int mx, int s) { return min(uint32_t(mx) - uint32_t(s), 1u << 20); }
__device__ __forceinline__ int exp_general(uint32_t zc, const int2* __restrict__ T) {
    const int2 e = T[zc >> 10];
    return int(i64(e.x) + (((i64(e.y) - e.x) * int(zc & 1023u)) >> 10));
}
// P before the 32767 clamp: (E r + 2^46) >> 47 for 0 <= E <= sum E, r = floor(2^62 / sum E) = rhi 2^32 + rlo: E r <= 2^62,
// so floor((E r + 2^46) / 2^47) = floor((E rhi + hi32(E rlo) + 2^14) / 2^15), every term below 2^32, the result below
// 2^17.  The clamp is the saturation of the packing instruction (pack_sat2).
__device__ __forceinline__ int p_of(uint32_t E, uint32_t rlo, uint32_t rhi) {
    return int(mad_lo_u(E, rhi, mad_hi_u(E, rlo, 16384u)) >> 15);
}
// two non-negative values saturated to 32767 and packed as 16-bit halves (hi, lo)
__device__ __forceinline__ uint32_t pack_sat2(int hi, int lo) {
    uint32_t w;
    asm("cvt.pack.sat.s16.s32 %0, %1, %2;" : "=r"(w) : "r"(hi), "r"(lo));
    return w;
}
// the same for any table: E may be negative; the reference's int64 arithmetic with P = 0 unless E > 0
__device__ __forceinline__ int p_general(int E, uint64_t r) {
    if (E <= 0) return 0;
    const i64 p = (i64(E) * i64(r) + (i64(1) << 46)) >> 47;
    return int(p > 32767 ? 32767 : p);
}

// Per-chunk row data of one thread: shq = 19 - eq, cq = 32768 qhs + 128 qls, r0 = 2^(shq - 1).
struct RowK { int shq, cq, r0; };

// One 16-key quarter tile of one pass for one query row (this thread): scores from the three TMEM accumulators
// (HH at taddr, X at +64, LL at +128; ekp / kcp = the 16 keys' exponents and 128 ksum), then
// PASS 0: row max; PASS 1: sum of E; PASS 2: P (into pw_h / pw_l).  TF: the fast exp table; FULL: every key of the
// chunk is valid (no causal mask, no key past Tk), else invalid keys take E = 0 and do not enter the max.
// mode 0: one key exponent eku for the chunk; 1: exponents differ (eku = their max); 2: a shift outside [5, 19].
template <int PASS, bool TF, bool FULL>
__device__ __forceinline__ void softmax_tile(uint32_t taddr, const int* __restrict__ ekp, const int* __restrict__ kcp, const RowK& rk, int mode, int eku,
                                             int kbase, int q, int Tk, int causal, const int2* __restrict__ L2, uint32_t lut_addr, const OpK& k,
                                             int& mx, uint64_t& sum, uint32_t rlo, uint32_t rhi, uint32_t* pw_h, uint32_t* pw_l,
                                             uint64_t* rel_qk) {
    int s[16];
    bool pre_shift = false;          // PASS 0, mode 0: s holds hh M + (T >> a); the row max takes the >> b once per chunk
    int bsh = 0;
    // passes 1-2 with the fast table: s holds u (mode 0: before the >> b) and the exp index comes from mxb - u
    uint32_t mxb = uint32_t(mx);
    ExpIdx xi = exp_idx(0);
    const ShiftSplit p = split_shift(mode == 2 ? 16 : rk.shq - eku);
    // X and LL first, folded into T (16 registers), then HH: the three accumulators are never all live at once
    int hh[16];
    {
        int xx[16], ll[16];
        tmem_ld16(taddr + 64, xx); tmem_ld16(taddr + 128, ll); tmem_ld16(taddr, hh);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive(rel_qk);
        if (mode == 0) {
            const int cr = rk.cq + (1 << (rk.shq - eku - 1));
            #pragma unroll
            for (int u = 0; u < 16; u += 4) {
                const int4 k4 = *reinterpret_cast<const int4*>(kcp + u);
                s[u] = mad_lo(xx[u], k.c256, ll[u] + k4.x + cr); s[u + 1] = mad_lo(xx[u + 1], k.c256, ll[u + 1] + k4.y + cr);
                s[u + 2] = mad_lo(xx[u + 2], k.c256, ll[u + 2] + k4.z + cr); s[u + 3] = mad_lo(xx[u + 3], k.c256, ll[u + 3] + k4.w + cr);
            }
        } else if (mode == 1) {          // each key's own rounding term 2^(shq - ek - 1) = r0 >> ek
            #pragma unroll
            for (int u = 0; u < 16; u += 4) {
                const int4 e4 = *reinterpret_cast<const int4*>(ekp + u);
                const int4 k4 = *reinterpret_cast<const int4*>(kcp + u);
                s[u] = mad_lo(xx[u], k.c256, ll[u] + k4.x + (rk.cq + (rk.r0 >> e4.x)));
                s[u + 1] = mad_lo(xx[u + 1], k.c256, ll[u + 1] + k4.y + (rk.cq + (rk.r0 >> e4.y)));
                s[u + 2] = mad_lo(xx[u + 2], k.c256, ll[u + 2] + k4.z + (rk.cq + (rk.r0 >> e4.z)));
                s[u + 3] = mad_lo(xx[u + 3], k.c256, ll[u + 3] + k4.w + (rk.cq + (rk.r0 >> e4.w)));
            }
        } else {
            #pragma unroll
            for (int u = 0; u < 16; ++u) s[u] = xx[u] * 256 + ll[u] + rk.cq + kcp[u];
        }
    }
    {
        if (mode == 0) {
            #pragma unroll
            for (int u = 0; u < 16; ++u) s[u] = div_pow2(hh[u], s[u], p);
            if (PASS == 0 && FULL) { pre_shift = true; bsh = p.b; }
            else if (PASS >= 1 && TF) { xi = exp_idx(p.b); mxb = (uint32_t(mx) << p.b) + ((1u << p.b) - 1u); }
            else if (__any_sync(0xffffffffu, p.b != 0)) {
                #pragma unroll
                for (int u = 0; u < 16; ++u) s[u] >>= p.b;
            }
        } else if (mode == 1) {
            const int bb = p.b + eku;                         // key u: >> (b + max ek - ek_u)
            #pragma unroll
            for (int u = 0; u < 16; u += 4) {
                const int4 e4 = *reinterpret_cast<const int4*>(ekp + u);
                s[u] = div_pow2(hh[u], s[u], p) >> (bb - e4.x); s[u + 1] = div_pow2(hh[u + 1], s[u + 1], p) >> (bb - e4.y);
                s[u + 2] = div_pow2(hh[u + 2], s[u + 2], p) >> (bb - e4.z); s[u + 3] = div_pow2(hh[u + 3], s[u + 3], p) >> (bb - e4.w);
            }
        } else {          // a shift outside [5, 19] somewhere in the tile: the 64-bit rshr with saturation
            #pragma unroll
            for (int u = 0; u < 16; ++u) s[u] = int(rshr((i64(hh[u]) << 16) + s[u], rk.shq - ekp[u]));
        }
    }
    uint32_t vmask = 0xFFFFu;   // validity by key position (a valid score may itself saturate to INT_MIN)
    if (!FULL) {
        vmask = 0;
        #pragma unroll
        for (int u = 0; u < 16; ++u) { const int key = kbase + u; vmask |= uint32_t(key < Tk && !(causal && key > q)) << u; }
    }
    if constexpr (PASS == 0) {
        if (pre_shift) {
            int m = s[0];
            #pragma unroll
            for (int u = 1; u < 16; ++u) m = max(m, s[u]);
            mx = max(mx, m >> bsh);
        } else {
            if (!FULL) {
                #pragma unroll
                for (int u = 0; u < 16; ++u) s[u] = (vmask >> u) & 1u ? s[u] : INT_MIN;
            }
            #pragma unroll
            for (int u = 0; u < 16; ++u) mx = max(mx, s[u]);
        }
    } else if constexpr (PASS == 1) {
        if constexpr (TF) {
            // each E <= 2^32 / 3: three add up in 32 bits (one three-input add), then to the 64-bit sum
            uint32_t e[16];
            #pragma unroll
            for (int u = 0; u < 16; ++u) {
                e[u] = uint32_t(exp_fast_d(mxb - uint32_t(s[u]), xi, lut_addr, k));
                if (!FULL) e[u] = (vmask >> u) & 1u ? e[u] : 0u;
            }
            #pragma unroll
            for (int u = 0; u < 15; u += 3) sum += e[u] + e[u + 1] + e[u + 2];
            sum += e[15];
        } else {
            #pragma unroll
            for (int u = 0; u < 16; ++u) {
                const int e = exp_general(zclamp(mx, s[u]), L2);
                if ((vmask >> u) & 1u) sum += uint64_t(i64(e));
            }
        }
    } else {
        #pragma unroll
        for (int u = 0; u < 16; u += 4) {
            int P[4];
            #pragma unroll
            for (int w = 0; w < 4; ++w) {
                if constexpr (TF) P[w] = p_of(uint32_t(exp_fast_d(mxb - uint32_t(s[u + w]), xi, lut_addr, k)), rlo, rhi);
                else P[w] = p_general(exp_general(zclamp(mx, s[u + w]), L2), (uint64_t(rhi) << 32) | rlo);
                if (!FULL) P[w] = (vmask >> (u + w)) & 1u ? P[w] : 0;
            }
            // 0 <= P < 2^17, saturated to 32767 while packed as 16-bit halves; then the hi bytes and (lo bytes - 128)
            const uint32_t w01 = pack_sat2(P[1], P[0]), w23 = pack_sat2(P[3], P[2]);
            pw_h[u / 4] = __byte_perm(w01, w23, 0x7531);
            pw_l[u / 4] = __byte_perm(w01, w23, 0x6420) ^ 0x80808080u;
        }
    }
}

// Per-thread constants of the softmax warps and their running row state.
struct SoftCtx {
    uint64_t *qk_full, *qk_free, *k_empty, *kinfo_full, *p_full, *p_free;
    const uint8_t* kaux;            // stage 0 of the per-stage key data
    const int2* lut;
    uint32_t lut_addr;              // shared-memory address of the exp table
    uint8_t *pst_h, *pst_l;         // this thread's 16 P bytes in the hi / lo P tiles (pass 2)
    uint32_t tq;                    // TMEM address of this thread's lane quarter and key quarter in QK buffer 0
    RowK rk;
    int kq, q, nT;
};
struct SoftState { int mx; uint64_t sum; uint32_t rlo, rhi; bool ok; };

// One pass over every key tile for this thread's row and key quarter.  Every warp runs every iteration, also after
// a timed-out wait (it then skips the work), so the barriers' arrival counts stay consistent.
template <int PASS, bool TF>
__device__ __forceinline__ void softmax_pass(const AttnArgs& a, const SoftCtx& c, SoftState& st) {
    const int lane = threadIdx.x & 31;
    for (int j = 0; j < c.nT; ++j) {
        const unsigned it = unsigned(PASS * c.nT + j), ks = it % KS;
        const unsigned b = PASS < 2 ? (it & 1u) : 0u;
        const unsigned ub = PASS < 2 ? (it >> 1) : it - unsigned(c.nT);     // earlier uses of buffer b
        if (st.ok) st.ok = __all_sync(0xffffffffu, mbar_wait(&c.qk_full[b], ub & 1u, a.err, DEVERR_TIMEOUT_FULL, a.wait_limit) &&
                                                   mbar_wait(&c.kinfo_full[ks], (it / KS) & 1u, a.err, DEVERR_TIMEOUT_FULL, a.wait_limit));
        if (!st.ok) continue;
        tc_fence_after();
        const uint8_t* aux = c.kaux + ks * KAUX_BYTES;
        const int info = reinterpret_cast<const int*>(aux + KAUX_QI)[c.kq];
        const int eku = info & 255, mode = (info >> QI_MODE) & 3;
        const int kbase = j * 64 + c.kq * 16;
        uint32_t pw_h[4], pw_l[4];
        const int* ekp = reinterpret_cast<const int*>(aux) + c.kq * 16;
        const int* kcp = reinterpret_cast<const int*>(aux + KAUX_KC) + c.kq * 16;
        if (info & QI_FULL) softmax_tile<PASS, TF, true>(c.tq + b * 192u, ekp, kcp, c.rk, mode, eku, kbase, c.q, a.Tk, a.causal, c.lut, c.lut_addr, a.k,
                                                         st.mx, st.sum, st.rlo, st.rhi, pw_h, pw_l, &c.qk_free[b]);
        else softmax_tile<PASS, TF, false>(c.tq + b * 192u, ekp, kcp, c.rk, mode, eku, kbase, c.q, a.Tk, a.causal, c.lut, c.lut_addr, a.k,
                                           st.mx, st.sum, st.rlo, st.rhi, pw_h, pw_l, &c.qk_free[b]);
        bool pout = false;
        if (PASS == 2) {
            st.ok = __all_sync(0xffffffffu, mbar_wait(c.p_free, (j & 1) ^ 1, a.err, DEVERR_TIMEOUT_EMPTY, a.wait_limit));
            if (st.ok) {
                *reinterpret_cast<uint4*>(c.pst_h) = make_uint4(pw_h[0], pw_h[1], pw_h[2], pw_h[3]);
                *reinterpret_cast<uint4*>(c.pst_l) = make_uint4(pw_l[0], pw_l[1], pw_l[2], pw_l[3]);
                fence_async_smem();
                pout = true;
            }
        }
        __syncwarp();
        if (lane == 0) {
            if (pout) mbar_arrive(c.p_full);
            mbar_arrive(&c.k_empty[ks]);      // this warp has read the stage's per-key data
        }
    }
}

__global__ void __launch_bounds__(THREADS, 1) attn_kernel(const __grid_constant__ AttnArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align_smem_1024(smem_raw);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
    uint64_t* q_full = bars;
    uint64_t* k_full = bars + 1; uint64_t* k_empty = k_full + KS;
    uint64_t* v_full = k_empty + KS; uint64_t* v_empty = v_full + VS;
    uint64_t* qk_full = v_empty + VS; uint64_t* qk_free = qk_full + 2;
    uint64_t* p_full = qk_free + 2; uint64_t* p_free = p_full + 1;
    uint64_t* pv_done = p_free + 1;
    uint64_t* kinfo_full = pv_done + 1;                   // [KS] the aux warp has written stage ks's kc / exponent ranges
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NBAR);
    int2* lut2 = reinterpret_cast<int2*>(sm + OFF_LUT);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = blockIdx.y, q0 = blockIdx.x * 128;
    const int nT = a.Tkp / 64, nIt = 3 * nT;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < KS; ++s) { mbar_init(&k_full[s], 1); mbar_init(&k_empty[s], 1 + SW); }
        for (int s = 0; s < VS; ++s) { mbar_init(&v_full[s], 1); mbar_init(&v_empty[s], 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(&qk_full[b], 1); mbar_init(&qk_free[b], SW); }
        mbar_init(p_full, SW); mbar_init(p_free, 1); mbar_init(pv_done, 1);
        for (int s = 0; s < KS; ++s) mbar_init(&kinfo_full[s], 1);
        mbar_fence_init();
    }
    if (warp == 1) { tmem_alloc(tmem_slot, TMEM_COLS); tmem_relinquish(); }
    // exp table: (L[i], L[i+1]) staged, and whether it qualifies for the fast form (every L[i] in [0, 2^32 / 3] and every
    // difference below 2^30 in magnitude); then the fast form replaces L[i+1] by 2 (L[i+1] - L[i])
    int tf = 1;
    for (int i = threadIdx.x; i <= 1024; i += blockDim.x) {
        int2 v = make_int2(0, 0);
        if (i < 1024) {
            v = make_int2(__ldg(a.lexp + i), __ldg(a.lexp + i + 1));
            const i64 d = i64(v.y) - v.x;
            tf &= v.x >= 0 && v.y >= 0 && v.x <= 0x55555555 && v.y <= 0x55555555 && d < (i64(1) << 30) && d > -(i64(1) << 30);
        }
        lut2[i] = v;
    }
    // the constant rows 64..79 of every V^T stage: zero, except row 64 of the lo plane, all ones (16-byte chunks)
    for (int i = threadIdx.x; i < VS * 2 * 64; i += blockDim.x) {
        const int s = i >> 7, plane = (i >> 6) & 1, c = i & 63;
        const uint32_t v = (plane == 1 && c < 4) ? 0x01010101u : 0u;
        *reinterpret_cast<uint4*>(sm + OFF_V + s * VSTAGE + plane * VT_BYTES + KT_BYTES + c * 16) = make_uint4(v, v, v, v);
    }
    fence_async_smem();
    const bool tfast = __syncthreads_and(tf) != 0;
    if (tfast)
        for (int i = threadIdx.x; i < 1024; i += blockDim.x) lut2[i].y = 2 * (lut2[i].y - lut2[i].x);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------------------------------------------------------- producer
        if (lane == 0 && !a.stall) {
            mbar_arrive_expect_tx(q_full, 2 * Q_BYTES);
            tma_load_2d(sm + OFF_Q, &a.tmQh, q_full, 0, g * a.Tqp + q0);
            tma_load_2d(sm + OFF_Q + Q_BYTES, &a.tmQl, q_full, 0, g * a.Tqp + q0);
            for (int it = 0; it < nIt; ++it) {
                const int j = it % nT, ks = it % KS;
                if (!mbar_wait(&k_empty[ks], ((it / KS) & 1) ^ 1, a.err, DEVERR_TIMEOUT_EMPTY, a.wait_limit)) break;
                uint8_t* kst = sm + OFF_K + ks * KSTAGE;
                uint8_t* aux = sm + OFF_KAUX + ks * KAUX_BYTES;
                mbar_arrive_expect_tx(&k_full[ks], KSTAGE + KAUX_TMA);
                tma_load_2d(kst, &a.tmKh, &k_full[ks], 0, g * a.Tkp + j * 64);
                tma_load_2d(kst + KT_BYTES, &a.tmKl, &k_full[ks], 0, g * a.Tkp + j * 64);
                bulk_load(aux, a.ek + size_t(g) * a.Tkp + j * 64, 64 * 4, &k_full[ks]);
                bulk_load(aux + 256, a.ksum + size_t(g) * a.Tkp + j * 64, 64 * 8, &k_full[ks]);
                if (it >= 2 * nT) {
                    const int vs = j % VS;
                    if (!mbar_wait(&v_empty[vs], ((j / VS) & 1) ^ 1, a.err, DEVERR_TIMEOUT_EMPTY, a.wait_limit)) break;
                    mbar_arrive_expect_tx(&v_full[vs], 2 * KT_BYTES);
                    uint8_t* vst = sm + OFF_V + vs * VSTAGE;
                    tma_load_2d(vst, &a.tmVh, &v_full[vs], j * 64, g * 64);
                    tma_load_2d(vst + VT_BYTES, &a.tmVl, &v_full[vs], j * 64, g * 64);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_i8(128, 64), idesc_pv = idesc_i8(128, PV_N);
            const uint32_t qh = smem_u32(sm + OFF_Q), ql = qh + Q_BYTES;
            const uint32_t ph = smem_u32(sm + OFF_P), pl = ph + P_BYTES;
            bool ok = mbar_wait(q_full, 0, a.err, DEVERR_TIMEOUT_FULL, a.wait_limit);
            auto issue_pv = [&](int j) -> bool {
                const int vs = j % VS;
                if (!mbar_wait(p_full, j & 1, a.err, DEVERR_TIMEOUT_FULL, a.wait_limit)) return false;
                if (!mbar_wait(&v_full[vs], (j / VS) & 1, a.err, DEVERR_TIMEOUT_FULL, a.wait_limit)) return false;
                tc_fence_after();
                const uint32_t vh = smem_u32(sm + OFF_V + vs * VSTAGE), vl = vh + VT_BYTES;
                #pragma unroll
                for (int kk = 0; kk < 2; ++kk) {
                    const bool acc = (j | kk) != 0;
                    mma_i8(tmem + PV_A, sdesc_sw64(ph + kk * 32), sdesc_sw64(vh + kk * 32), idesc_pv, acc);
                    mma_i8(tmem + PV_Y, sdesc_sw64(ph + kk * 32), sdesc_sw64(vl + kk * 32), idesc_pv, acc);
                    mma_i8(tmem + PV_Y, sdesc_sw64(pl + kk * 32), sdesc_sw64(vh + kk * 32), idesc_pv, true);
                    mma_i8(tmem + PV_D, sdesc_sw64(pl + kk * 32), sdesc_sw64(vl + kk * 32), idesc_pv, acc);
                }
                mma_commit(p_free);
                mma_commit(&v_empty[vs]);
                return true;
            };
            for (int it = 0; it < nIt && ok; ++it) {
                const int pass = it / nT, j = it % nT, ks = it % KS;
                const int b = pass < 2 ? (it & 1) : 0;
                // earlier uses of buffer b: passes 0-1 alternate the buffers, pass 2 keeps buffer 0
                const int ub = it < 2 * nT ? (it >> 1) : it - nT;
                if (pass == 2 && j == 0) {      // the P.V accumulators reuse buffer 1's columns (used nT times)
                    if (!mbar_wait(&qk_free[1], (nT & 1) ^ 1, a.err, DEVERR_TIMEOUT_EMPTY, a.wait_limit)) { ok = false; break; }
                }
                if (!mbar_wait(&k_full[ks], (it / KS) & 1, a.err, DEVERR_TIMEOUT_FULL, a.wait_limit)) { ok = false; break; }
                if (!mbar_wait(&qk_free[b], (ub & 1) ^ 1, a.err, DEVERR_TIMEOUT_EMPTY, a.wait_limit)) { ok = false; break; }
                tc_fence_after();
                const uint32_t kh = smem_u32(sm + OFF_K + ks * KSTAGE), kl = kh + KT_BYTES;
                const uint32_t d = tmem + b * 192;
                #pragma unroll
                for (int kk = 0; kk < 2; ++kk) {
                    mma_i8(d, sdesc_sw64(qh + kk * 32), sdesc_sw64(kh + kk * 32), idesc, kk != 0);
                    mma_i8(d + 64, sdesc_sw64(qh + kk * 32), sdesc_sw64(kl + kk * 32), idesc, kk != 0);
                    mma_i8(d + 64, sdesc_sw64(ql + kk * 32), sdesc_sw64(kh + kk * 32), idesc, true);
                    mma_i8(d + 128, sdesc_sw64(ql + kk * 32), sdesc_sw64(kl + kk * 32), idesc, kk != 0);
                }
                mma_commit(&qk_full[b]);
                mma_commit(&k_empty[ks]);
                if (pass == 2 && j >= 1) ok = issue_pv(j - 1);
            }
            if (ok) ok = issue_pv(nT - 1);
            mma_commit(pv_done);
        }
    } else if (warp == AUX_WARP) {
        // ---------------------------------------------------------------- per-stage key data, once per CTA
        // kc = 128 ksum as int32 (|ksum| <= 64 * 32767) and each 16-key quarter's info word: its largest key exponent,
        // the score form and whether every key is valid.  The fast forms need every shift 19 - eq - ek of the CTA's
        // rows in [5, 19], checked against the CTA's largest row exponent (rows past Tqp do not exist).
        int eqmax = 0;
        for (int r = lane; r < 128; r += 32)
            if (q0 + r < a.Tqp) eqmax = max(eqmax, __ldg(a.eq + size_t(g) * a.Tqp + q0 + r));
        const int shq_min = 19 - __reduce_max_sync(0xffffffffu, eqmax);
        auto info_word = [&](int emin, int emax, int kbase) {
            const int mode = shq_min - emax < 5 ? 2 : (emin == emax ? 0 : 1);
            return emax | (mode << QI_MODE) | (!a.causal && kbase + 16 <= a.Tk ? QI_FULL : 0);
        };
        bool ok = true;
        for (int it = 0; it < nIt && ok; ++it) {
            const int ks = it % KS, j = it % nT;
            ok = __all_sync(0xffffffffu, mbar_wait(&k_full[ks], (it / KS) & 1, a.err, DEVERR_TIMEOUT_FULL, a.wait_limit));
            if (!ok) break;
            uint8_t* aux = sm + OFF_KAUX + ks * KAUX_BYTES;
            const int32_t* ek = reinterpret_cast<const int32_t*>(aux);
            const i64* ksum = reinterpret_cast<const i64*>(aux + 256);
            int32_t* kc = reinterpret_cast<int32_t*>(aux + KAUX_KC);
            int* qi = reinterpret_cast<int*>(aux + KAUX_QI);
            const int e0 = ek[lane], e1 = ek[lane + 32];            // quarters lane >> 4 and 2 + (lane >> 4)
            kc[lane] = int(128 * ksum[lane]); kc[lane + 32] = int(128 * ksum[lane + 32]);
            int mn0 = e0, mx0 = e0, mn1 = e1, mx1 = e1;
            #pragma unroll
            for (int o = 8; o; o >>= 1) {
                mn0 = min(mn0, __shfl_xor_sync(0xffffffffu, mn0, o)); mx0 = max(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
                mn1 = min(mn1, __shfl_xor_sync(0xffffffffu, mn1, o)); mx1 = max(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
            }
            if ((lane & 15) == 0) {
                const int k0 = lane >> 4;
                qi[k0] = info_word(mn0, mx0, j * 64 + k0 * 16);
                qi[2 + k0] = info_word(mn1, mx1, j * 64 + (2 + k0) * 16);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&kinfo_full[ks]);
        }
    } else {
        // ---------------------------------------------------------------- softmax / output warps
        const int qq = warp & 3, kq = (warp - 2) >> 2;             // lane quarter; key quarter (and dim quarter)
        const int rl = qq * 32 + lane, q = q0 + rl;
        const uint32_t tl = uint32_t(qq * 32) << 16;
        const size_t rq = size_t(g) * a.Tqp + q;
        const bool qin = q < a.Tqp;                                 // the last query tile may reach past Tqp (Tqp % 128 == 64)
        const int eqv = qin ? __ldg(a.eq + rq) : 0;
        const int cq = qin ? int(32768 * __ldg(a.qhs + rq) + 128 * __ldg(a.qls + rq)) : 0;
        const int shq = 19 - eqv;                                   // eq <= 17, so shq >= 2
        SoftCtx c;
        c.qk_full = qk_full; c.qk_free = qk_free; c.k_empty = k_empty; c.kinfo_full = kinfo_full; c.p_full = p_full; c.p_free = p_free;
        c.kaux = sm + OFF_KAUX; c.lut = lut2; c.lut_addr = smem_u32(lut2);
        c.pst_h = sm + OFF_P + sw64_off(rl, kq); c.pst_l = c.pst_h + P_BYTES;
        c.tq = tmem + tl + uint32_t(kq * 16);
        c.rk = RowK{shq, cq, 1 << (shq - 1)};                       // r0: rounding term of shift shq; >> ek gives that of shq - ek
        c.kq = kq; c.q = q; c.nT = nT;
        i64* red = reinterpret_cast<i64*>(sm + OFF_RED);          // [4][128]
        SoftState st{INT_MIN, 0, 0, 0, true};
        // combine the four key quarters of each row after pass 0 (max) and pass 1 (sum -> r)
        auto combine = [&](i64 v, i64* o) {
            red[kq * 128 + rl] = v;
            asm volatile("bar.sync 1, %0;" :: "r"(SW * 32) : "memory");
            #pragma unroll
            for (int w = 1; w < 4; ++w) o[w - 1] = red[((kq + w) & 3) * 128 + rl];
            asm volatile("bar.sync 1, %0;" :: "r"(SW * 32) : "memory");
        };
        i64 o[3];
        if (tfast) softmax_pass<0, true>(a, c, st); else softmax_pass<0, false>(a, c, st);
        combine(i64(st.mx), o);
        st.mx = max(max(st.mx, int(o[0])), max(int(o[1]), int(o[2])));
        if (tfast) softmax_pass<1, true>(a, c, st); else softmax_pass<1, false>(a, c, st);
        combine(i64(st.sum), o);
        {
            const uint64_t tot = st.sum + uint64_t(o[0]) + uint64_t(o[1]) + uint64_t(o[2]);
            const uint64_t r = tot ? (uint64_t(1) << 62) / tot : 0;
            st.rlo = uint32_t(r); st.rhi = uint32_t(r >> 32);
        }
        if (tfast) softmax_pass<2, true>(a, c, st); else softmax_pass<2, false>(a, c, st);
        const bool ok = st.ok;
        // ---------------------------------------------------------------- output
        const bool done = ok && __all_sync(0xffffffffu, mbar_wait(pv_done, 0, a.err, DEVERR_TIMEOUT_ACC, a.wait_limit));
        tc_fence_after();
        if (done) {
            const int bidx = g / a.heads, h = g % a.heads;
            const i64 n = a.Tkp;
            // sum_k P = 256 sum ph + sum pl + 128 n from column 64 of the Y and D accumulators
            int ysum, dsum;
            tmem_ld1(tmem + tl + PV_Y + 64, &ysum); tmem_ld1(tmem + tl + PV_D + 64, &dsum);
            u32 am = 0;
            #pragma unroll
            for (int hv = 0; hv < 2; ++hv) {           // two halves of 8 output dims: fewer live registers
                int A[8], Y[8], D[8];
                const uint32_t col = uint32_t(kq * 16 + hv * 8);
                tmem_ld8(tmem + tl + PV_A + col, A); tmem_ld8(tmem + tl + PV_Y + col, Y); tmem_ld8(tmem + tl + PV_D + col, D);
                tmem_ld_wait();
                const i64 ps = 256 * i64(ysum) + dsum + 128 * n;
                if (q < a.Tq) {
                    int o[8];
                    #pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        const int dd = kq * 16 + hv * 8 + u;
                        const i64 O = 65536 * i64(A[u]) + 256 * i64(Y[u]) + D[u] + 128 * (ps + __ldg(a.vsum + g * 64 + dd)) - 16384 * n;
                        o[u] = int(rshr(O, 15 - __ldg(a.ev + g * 64 + dd)));
                        am = max(am, uabs(o[u]));
                    }
                    int32_t* dst = a.out + (size_t(bidx) * a.Tq + q) * a.C + h * 64 + kq * 16 + hv * 8;
                    *reinterpret_cast<int4*>(dst) = make_int4(o[0], o[1], o[2], o[3]);
                    *reinterpret_cast<int4*>(dst + 4) = make_int4(o[4], o[5], o[6], o[7]);
                }
            }
            if (a.rowmax && q < a.Tq && am) atomicMax(a.rowmax + size_t(bidx) * a.Tq + q, am);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) { tc_fence_after(); tmem_dealloc(tmem, TMEM_COLS); }
}
}  // namespace

void fused_attention(cudaStream_t st, const int8_t* qhi, const int8_t* qlo, const int32_t* eq, const i64* qhs, const i64* qls,
                     const int8_t* khi, const int8_t* klo, const int32_t* ek, const i64* ksum,
                     const int8_t* vthi, const int8_t* vtlo, const int32_t* ev, const i64* vsum,
                     int B, int heads, int Tq, int Tqp, int Tk, int Tkp, bool causal, const int32_t* lexp, int C, int32_t* out, uint32_t* rowmax,
                     const LaunchOpts& o) {
    VELA_REQUIRE(qhi && qlo && eq && qhs && qls && khi && klo && ek && ksum && vthi && vtlo && ev && vsum && lexp && out, "attention: null operand");
    VELA_REQUIRE(B > 0 && heads > 0 && C == heads * 64 && Tq > 0 && Tq <= Tqp && Tqp % 64 == 0 && Tk > 0 && Tk <= Tkp && Tkp % 64 == 0 && Tkp <= 4096,
                 "attention: needs C = 64*heads, Tqp % 64 == 0, Tkp % 64 == 0, Tk <= Tkp <= 4096");
    const int G = B * heads;
    AttnArgs a;
    std::memset(static_cast<void*>(&a), 0, sizeof(a));
    a.tmQh = tmap2d(qhi, CU_TENSOR_MAP_DATA_TYPE_UINT8, 64, uint64_t(G) * Tqp, 64, 64, 128, Swz::B64);
    a.tmQl = tmap2d(qlo, CU_TENSOR_MAP_DATA_TYPE_UINT8, 64, uint64_t(G) * Tqp, 64, 64, 128, Swz::B64);
    a.tmKh = tmap2d(khi, CU_TENSOR_MAP_DATA_TYPE_UINT8, 64, uint64_t(G) * Tkp, 64, 64, 64, Swz::B64);
    a.tmKl = tmap2d(klo, CU_TENSOR_MAP_DATA_TYPE_UINT8, 64, uint64_t(G) * Tkp, 64, 64, 64, Swz::B64);
    a.tmVh = tmap2d(vthi, CU_TENSOR_MAP_DATA_TYPE_UINT8, uint64_t(Tkp), uint64_t(G) * 64, uint64_t(Tkp), 64, 64, Swz::B64);
    a.tmVl = tmap2d(vtlo, CU_TENSOR_MAP_DATA_TYPE_UINT8, uint64_t(Tkp), uint64_t(G) * 64, uint64_t(Tkp), 64, 64, Swz::B64);
    a.eq = eq; a.qhs = qhs; a.qls = qls; a.ek = ek; a.ksum = ksum; a.ev = ev; a.vsum = vsum; a.lexp = lexp;
    a.out = out; a.rowmax = rowmax;
    a.heads = heads; a.Tq = Tq; a.Tqp = Tqp; a.Tk = Tk; a.Tkp = Tkp; a.C = C; a.causal = causal ? 1 : 0;
    a.err = o.err ? o.err : device_error_word(&g_attn_err);
    a.wait_limit = o.wait_limit > 0 ? o.wait_limit : WAIT_LIMIT_CYCLES;
    a.stall = o.stall;
    a.k = OpK{256, 8};
    static std::atomic<int> attr_done[64];
    once_per_device(attr_done, [] { VELA_CUDA(cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM)); });
    attn_kernel<<<dim3(ceil_div(Tqp, 128), G), THREADS, SMEM, st>>>(a);
    VELA_CUDA(cudaGetLastError());
}
}  // namespace vela

using namespace vela;
// Replaces k_fused_attention (src/kernels.h:72-78 / src/attn.cu:551-600).  gmx / gr (the reference's
// between-pass scratch) are accepted for signature compatibility and unused: the row max and the
// reciprocal stay in registers.  Lexp is the int64 exp LUT of the reference API (values < 2^31);
// lexp32 is the int32 copy the kernel reads (B200 callers pass it; when null it must be provided).
extern "C" int vela_fused_attention(void* stream, const int8_t* qhi, const int8_t* qlo, const int32_t* eq, const int64_t* qhs, const int64_t* qls,
                                    const int8_t* khi, const int8_t* klo, const int32_t* ek, const int64_t* ksum,
                                    const int8_t* vthi, const int8_t* vtlo, const int32_t* ev, const int64_t* vsum,
                                    int B, int heads, int Tq, int Tqp, int Tk, int Tkp, int causal, const int32_t* lexp32, int C,
                                    int32_t* gmx, int64_t* gr, int32_t* out, uint32_t* rowmax) {
    (void)gmx; (void)gr;
    return guarded("vela_fused_attention", [&] {
        fused_attention(static_cast<cudaStream_t>(stream), qhi, qlo, eq, qhs, qls, khi, klo, ek, ksum, vthi, vtlo, ev, vsum,
                        B, heads, Tq, Tqp, Tk, Tkp, causal != 0, lexp32, C, out, rowmax);
    });
}
// Failure-path test of the bounded waits (no reference counterpart): vela_fused_attention with the TMA producer idle
// and a wait limit of wait_limit_cycles, so every wait of the MMA and softmax warps runs out; the kernel drains, frees
// its TMEM and returns, and vela_device_error reports the timeout.  Nothing is in flight when the waits give up.
extern "C" int vela_fused_attention_stalled(void* stream, const int8_t* qhi, const int8_t* qlo, const int32_t* eq, const int64_t* qhs, const int64_t* qls,
                                            const int8_t* khi, const int8_t* klo, const int32_t* ek, const int64_t* ksum,
                                            const int8_t* vthi, const int8_t* vtlo, const int32_t* ev, const int64_t* vsum,
                                            int B, int heads, int Tq, int Tqp, int Tk, int Tkp, int causal, const int32_t* lexp32, int C,
                                            int32_t* out, uint32_t* rowmax, long long wait_limit_cycles) {
    return guarded("vela_fused_attention_stalled", [&] {
        VELA_REQUIRE(wait_limit_cycles > 0, "non-positive wait limit");
        LaunchOpts o; o.wait_limit = wait_limit_cycles; o.stall = 1;
        fused_attention(static_cast<cudaStream_t>(stream), qhi, qlo, eq, qhs, qls, khi, klo, ek, ksum, vthi, vtlo, ev, vsum,
                        B, heads, Tq, Tqp, Tk, Tkp, causal != 0, lexp32, C, out, rowmax, o);
    });
}

namespace vela {
namespace {
// Exact attention written as plain loops, one thread per (head-batch g, query q): the definition restated
// (src/kernels.cu:671-722) with 64-bit sums and no tiling, used only to check the tiled kernel (Engine::test_attention,
// the reference's --test-attn).  Q, K: head-quantised planes [G, Tp, 64] + e; V^T planes [G, 64, Tkp] + ev.
__global__ void attention_plain_kernel(const int8_t* __restrict__ qhi, const int8_t* __restrict__ qlo, const int32_t* __restrict__ eq, int Tqp,
                                       const int8_t* __restrict__ khi, const int8_t* __restrict__ klo, const int32_t* __restrict__ ek,
                                       const int8_t* __restrict__ vhi, const int8_t* __restrict__ vlo, const int32_t* __restrict__ ev,
                                       int heads, int Tq, int Tk, int Tkp, int causal, const int32_t* __restrict__ L, int C, int32_t* __restrict__ out) {
    const int g = blockIdx.y, q = blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= Tq) return;
    const int nk = causal ? min(Tk, q + 1) : Tk;
    auto qval = [&](int d) { const size_t i = (size_t(g) * Tqp + q) * 64 + d; return 256 * int(qhi[i]) + int(qlo[i]) + 128; };
    auto score = [&](int k) {
        i64 S = 0;
        const size_t kb = (size_t(g) * Tkp + k) * 64;
        for (int d = 0; d < 64; ++d) S += i64(qval(d)) * (256 * int(khi[kb + d]) + int(klo[kb + d]) + 128);
        return int(rshr(S, 19 - eq[size_t(g) * Tqp + q] - ek[size_t(g) * Tkp + k]));
    };
    auto expl = [&](i64 z) -> i64 {
        if (z >= (i64(1) << 20)) return 0;
        const int i = int(z >> 10), f = int(z & 1023);
        return int32_t(L[i] + (((i64(L[i + 1]) - L[i]) * f) >> 10));
    };
    int mx = INT_MIN;
    for (int k = 0; k < nk; ++k) mx = max(mx, score(k));
    i64 sum = 0;
    for (int k = 0; k < nk; ++k) sum += expl(i64(mx) - score(k));
    const i64 r = sum > 0 ? floor_div(i64(1) << 62, sum) : 0;
    i64 O[64];
    for (int d = 0; d < 64; ++d) O[d] = 0;
    for (int k = 0; k < nk; ++k) {
        const i64 E = expl(i64(mx) - score(k));
        if (E <= 0) continue;
        const i64 P = min(i64(32767), (E * r + (i64(1) << 46)) >> 47);
        for (int d = 0; d < 64; ++d) {
            const size_t vi = (size_t(g) * 64 + d) * Tkp + k;
            O[d] += P * (256 * int(vhi[vi]) + int(vlo[vi]) + 128);
        }
    }
    const int b = g / heads, h = g % heads;
    for (int d = 0; d < 64; ++d) out[(size_t(b) * Tq + q) * C + h * 64 + d] = int(rshr(O[d], 15 - ev[g * 64 + d]));
}
}  // namespace

void attention_plain(cudaStream_t st, const int8_t* qhi, const int8_t* qlo, const int32_t* eq, int Tqp, const int8_t* khi, const int8_t* klo,
                     const int32_t* ek, const int8_t* vhi, const int8_t* vlo, const int32_t* ev, int B, int heads, int Tq, int Tk, int Tkp,
                     bool causal, const int32_t* lexp, int C, int32_t* out) {
    VELA_REQUIRE(B > 0 && heads > 0 && Tq > 0 && Tk > 0 && Tk <= Tkp && C == 64 * heads, "attention_plain: bad shape");
    attention_plain_kernel<<<dim3(ceil_div(Tq, 64), B * heads), 64, 0, st>>>(qhi, qlo, eq, Tqp, khi, klo, ek, vhi, vlo, ev, heads, Tq, Tk, Tkp,
                                                                             causal ? 1 : 0, lexp, C, out);
    VELA_CUDA(cudaGetLastError());
}
}  // namespace vela
