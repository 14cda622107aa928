// W8A16 hi/lo GEMM on the sm_100a tensor cores (tcgen05.mma kind::i8).
//
// Computes, for output row r and column n (the semantics of the reference's
// gemm_hl kernel, src/gemm_hl.cu:40-52,175-309):
//     acc = 256 * (Ahi[r] . W[n]) + Alo[r] . W[n] + 128 * wsum[n]      (= sum_k q[r,k] W[n,k])
//     y   = sat32(rshr(acc * m[n], s[n] - e[r]) + b[n])
// followed by one of the fused epilogues (plain / GELU / + residual / row max,
// GEGLU, q|k|v head quantisation, 3-way split), or raw s32 partials for split-K.
//
// Operand staging on chip (shared by every kernel that includes this header): a 128-row tile of A as two
// K-major int8 planes, A-hi and A-lo [128 x 64 bytes per K step], and W [BN x 64], all with the 64-byte
// swizzle; per 32-byte K slice two tcgen05.mma (M=128, N=BN, K=32) accumulate A-hi x W and A-lo x W into two
// s32 TMEM accumulators, so the hi/lo recombination happens only in the epilogue below.  The kernel and its
// schedule are in gemm_persist.cuh.
#pragma once
#include "intops.cuh"
#include "tc.cuh"
#include "host_util.h"

namespace vela {

enum { SRC_I8 = 0, SRC_X32 = 1, SRC_CONV32 = 2 };
enum { EPI_PLAIN = 0, EPI_SPLIT3 = 1, EPI_GEGLU = 2, EPI_GELU = 3, EPI_QKV = 4 };

struct GemmArgs {
    CUtensorMap tmA_hi, tmA_lo, tmW;
    CUtensorMap tmX;                                        // int32 sources staged by TMA (xtma = 1): X rows or the NHWC image
    int xtma;                                               // 1: int32 operand through tmX + staging ring; 0: per-thread loads
    int conv_rows_per_img;                                  // SRC_CONV32 with xtma: output rows per image (Ho*Wo)
    int Mreal, Nreal, Np, Mp, Kp, nkb, kb_per_split;
    const int32_t* e;                                       // SRC_I8 / SRC_CONV32: per-row exponent
    const int32_t* x; int ldx; const uint32_t* rowmax_in; int K;   // SRC_X32 (and K bound of int32 sources)
    const int32_t* img; int H, W, C, stride, Ho, Wo;        // SRC_CONV32, tap-major K = (ky*3+kx)*C + c
    const int4* cst;                                        // {m, s, b, wsum} per column (Np entries)
    int32_t* Y; int ldy; const int32_t* R; int gelu; const int32_t* Lphi; uint32_t* rowmax_out;
    int Cs; int32_t* Y1; int32_t* Y2;                       // EPI_SPLIT3 / EPI_QKV (v)
    int heads, T, TpQ, TpK, Cq;                             // EPI_QKV (Cq = heads * 64)
    int8_t *qhi, *qlo, *khi, *klo; int32_t *qe, *ke; int64_t *qhs, *qls, *qts, *khs, *kls, *kts;
    int32_t* partial;                                       // split-K: raw s32 [split][2][Mp][Np]
    int rvec;                                               // residual rows 16-byte aligned (int4 loads)
    CUtensorMap tmY;                                        // plain epilogue with ytma = 1: Y [Mreal][Nreal] int32, box 16 x 32, 64B swizzle
    int ytma;
    unsigned* err;
    long long wait_limit;                                   // SM clock cycles before a barrier wait gives up
    int stall;                                              // failure-path tests: the TMA producers issue nothing
};

__device__ __forceinline__ int ws128(int4 c) { return 128 * c.w; }

// An epilogue warp's shared-memory boxes (2 KB each) for the TMA stores of Y.  One box: a plain pointer, each store
// waits until the previous one has read the box.  Several boxes (YBox, by reference): n boxes used in turn, i counts
// the warp's stores, and with two boxes a store waits only for the one before the previous.  A null base means no
// TMA stores.
struct YBox { uint8_t* base; int n; int i; };
__device__ __forceinline__ bool ybox_on(const uint8_t* p) { return p != nullptr; }
__device__ __forceinline__ bool ybox_on(const YBox& b) { return b.base != nullptr; }
__device__ __forceinline__ uint8_t* ybox_cur(uint8_t* p) { return p; }
__device__ __forceinline__ uint8_t* ybox_cur(const YBox& b) { return b.base + (b.i & (b.n - 1)) * 2048; }
__device__ __forceinline__ void ybox_wait(const uint8_t*) { bulk_wait_read0(); }
__device__ __forceinline__ void ybox_wait(const YBox& b) { if (b.n == 2) bulk_wait_read1(); else bulk_wait_read0(); }
__device__ __forceinline__ void ybox_next(uint8_t*) {}
__device__ __forceinline__ void ybox_next(YBox& b) { ++b.i; }


// Epilogue of one 128 x BN tile for one thread = one output row (rl) and the NC columns [c0, c0 + NC) of the tile
// (q|k|v: NC = 64, one head): reads the hi / lo accumulators from TMEM (tl = the thread's lane-quarter base),
// applies the per-column constants (cst[j] = column n0 + j) and writes the epilogue's outputs.  er is the row's
// exponent; L2 the GELU table staged in shared memory (null: read a.Lphi from global memory); yb the warp's boxes for
// the TMA stores of a plain epilogue (uint8_t* or YBox2&, see above).
template <int BN, int SRC, int EPI, int NC, bool FAST, class YB>
__device__ __forceinline__ void gemm_epilogue_t(const GemmArgs& a, uint32_t tl, const int4* __restrict__ cst, const int2* __restrict__ L2,
                                                int m0, int n0, int rl, int c0, int split, int er, YB yb) {
    static_assert(NC % 16 == 0, "16-column chunks");
    const int grow = m0 + rl;
    const bool live = grow < a.Mreal;
    if constexpr (EPI == EPI_QKV) {
        static_assert(NC == 64, "q|k|v epilogue works on one 64-column head per thread");
        int y[64];
        #pragma unroll
        for (int c = 0; c < 4; ++c) {
            int hi[16], lo[16];
            tmem_ld16(tl + c0 + c * 16, hi); tmem_ld16(tl + BN + c0 + c * 16, lo); tmem_ld_wait();
            #pragma unroll
            for (int j = 0; j < 16; ++j) { const int4 cc = cst[c0 + c * 16 + j]; y[c * 16 + j] = FAST ? epi_y_fast(hi[j], lo[j], cc.x, cc.y - er, cc.z, ws128(cc)) : epi_y(hi[j], lo[j], cc.x, cc.y - er, cc.z, ws128(cc)); }
        }
        const int nh = n0 + c0;
        // the head's row exponent and the warp's choice of rounding form, voted by every lane (rows past Mreal vote
        // for the short form) before the per-lane branch below
        u32 hm = 0;
        #pragma unroll
        for (int j = 0; j < 64; ++j) hm = max(hm, uabs(y[j]));
        const int ee = row_exp(hm);
        const bool e15 = __all_sync(0xffffffffu, !live || ee <= 15);
        if (live && nh < a.Nreal) {
            const int part = nh / a.Cq, head = (nh - part * a.Cq) >> 6;
            if (part == 2) {
                int4* dst = reinterpret_cast<int4*>(a.Y2 + size_t(grow) * a.Cq + head * 64);
                #pragma unroll
                for (int j = 0; j < 16; ++j) dst[j] = make_int4(y[4 * j], y[4 * j + 1], y[4 * j + 2], y[4 * j + 3]);
            } else {
                const int b = grow / a.T, t = grow - b * a.T;
                const int Tp = part == 0 ? a.TpQ : a.TpK;
                const size_t gt = size_t(b * a.heads + head) * Tp + t;
                int8_t* hip = (part == 0 ? a.qhi : a.khi) + gt * 64; int8_t* lop = (part == 0 ? a.qlo : a.klo) + gt * 64;
                // quant16 of the head's 64 values, four at a time into hi / lo byte words (quant_pack4; the two-operation
                // rounding when every live row of the warp has e <= 15); the plane sums from the packed bytes (dp4a), and
                // sum q = 256 sum hi + sum lo + 128 * 64 since q = 256 hi + lo + 128
                const int qs1 = ee > 0 ? ee - 1 : 0, qr = ee > 0 ? 1 : 0, qh = (1 << ee) >> 1;
                int hs = 0, ls = 0;
                #pragma unroll
                for (int j = 0; j < 16; j += 4) {
                    uint32_t hw[4], lw[4];
                    #pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int b4 = (j + u) * 4;
                        if (e15) quant_pack4_e15(y[b4], y[b4 + 1], y[b4 + 2], y[b4 + 3], qh, ee, hw[u], lw[u]);
                        else quant_pack4(y[b4], y[b4 + 1], y[b4 + 2], y[b4 + 3], qs1, qr, qr, hw[u], lw[u]);
                        hs = __dp4a(int(hw[u]), 0x01010101, hs);
                        ls = __dp4a(int(lw[u]), 0x01010101, ls);
                    }
                    *reinterpret_cast<uint4*>(hip + j * 4) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                    *reinterpret_cast<uint4*>(lop + j * 4) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
                }
                const int ts = 256 * hs + ls + 128 * 64;
                (part == 0 ? a.qe : a.ke)[gt] = ee;
                (part == 0 ? a.qhs : a.khs)[gt] = hs;
                (part == 0 ? a.qls : a.kls)[gt] = ls;
                (part == 0 ? a.qts : a.kts)[gt] = ts;
            }
        }
    } else {
        u32 mx = 0;
        #pragma unroll 1
        for (int c = 0; c < NC / 16; ++c) {
            const int col = c0 + c * 16, n = n0 + col;
            if (n >= a.Nreal) break;                  // warp-uniform: the rest of the slice lies past N
            const bool act = live;
            const bool full16 = n + 16 <= a.Nreal;
            // residual of this chunk in flight while the accumulators are read (int4 when rows are 16-byte aligned)
            int4 rv[4];
            if constexpr (EPI == EPI_PLAIN) {
                if (act && a.R && a.rvec && full16) {
                    const int4* rp = reinterpret_cast<const int4*>(a.R + size_t(grow) * a.ldy + n);
                    #pragma unroll
                    for (int j = 0; j < 4; ++j) rv[j] = __ldg(rp + j);
                }
            }
            int hi[16], lo[16];
            tmem_ld16(tl + col, hi); tmem_ld16(tl + BN + col, lo); tmem_ld_wait();
            // a TMA-stored plain chunk is written by the whole warp (rows past Mreal are clipped by the store)
            const bool tstore = EPI == EPI_PLAIN && ybox_on(yb);
            if (!act && !tstore) continue;
            if (a.partial) {             // split-K: raw accumulators, reduced by gemm_splitk_reduce
                int32_t* ph = a.partial + (size_t(split) * 2 * a.Mp + grow) * a.Np + n;
                int32_t* pl = ph + size_t(a.Mp) * a.Np;
                #pragma unroll
                for (int j = 0; j < 16; j += 4) {
                    *reinterpret_cast<int4*>(ph + j) = make_int4(hi[j], hi[j + 1], hi[j + 2], hi[j + 3]);
                    *reinterpret_cast<int4*>(pl + j) = make_int4(lo[j], lo[j + 1], lo[j + 2], lo[j + 3]);
                }
                continue;
            }
            if constexpr (EPI == EPI_PLAIN) {
                // four columns at a time: y, GELU, + residual, then out (shared-memory box or global) and the row max
                const int lane = rl & 31;
                uint8_t* box = ybox_cur(yb);
                if (tstore) {                            // the store that last used this box has finished reading it
                    if (lane == 0) ybox_wait(yb);
                    __syncwarp();
                }
                const int32_t* rp = a.R + size_t(grow) * a.ldy + n;
                int32_t* dst = a.Y + size_t(grow) * a.ldy + n;
                #pragma unroll
                for (int g4 = 0; g4 < 4; ++g4) {
                    int y4[4];
                    #pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int j = 4 * g4 + u;
                        const int4 cc = cst[col + j];
                        y4[u] = FAST ? epi_y_fast(hi[j], lo[j], cc.x, cc.y - er, cc.z, ws128(cc)) : epi_y(hi[j], lo[j], cc.x, cc.y - er, cc.z, ws128(cc));
                    }
                    if (a.gelu) {
                        #pragma unroll
                        for (int u = 0; u < 4; ++u) y4[u] = L2 ? lut_act_s(y4[u], L2) : lut_act(y4[u], a.Lphi);
                    }
                    if (a.R && act) {
                        if (a.rvec && full16) {
                            y4[0] = add_sat(y4[0], rv[g4].x); y4[1] = add_sat(y4[1], rv[g4].y);
                            y4[2] = add_sat(y4[2], rv[g4].z); y4[3] = add_sat(y4[3], rv[g4].w);
                        } else {
                            #pragma unroll
                            for (int u = 0; u < 4; ++u) if (full16 || n + 4 * g4 + u < a.Nreal) y4[u] = add_sat(y4[u], __ldg(rp + 4 * g4 + u));
                        }
                    }
                    if (tstore) {
                        *reinterpret_cast<int4*>(box + sw64_off(lane, g4)) = make_int4(y4[0], y4[1], y4[2], y4[3]);
                    } else if (full16 && (a.ldy & 3) == 0) {
                        *reinterpret_cast<int4*>(dst + 4 * g4) = make_int4(y4[0], y4[1], y4[2], y4[3]);
                    } else {
                        #pragma unroll
                        for (int u = 0; u < 4; ++u) if (n + 4 * g4 + u < a.Nreal) dst[4 * g4 + u] = y4[u];
                    }
                    if (act) {
                        #pragma unroll
                        for (int u = 0; u < 4; ++u) if (full16 || n + 4 * g4 + u < a.Nreal) mx = max(mx, uabs(y4[u]));
                    }
                }
                if (tstore) {                            // the warp's 32 rows x 16 columns: one TMA store (rows past Mreal clipped)
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0) { tma_store_2d(&a.tmY, box, n, m0 + (rl & ~31)); bulk_commit(); }
                    ybox_next(yb);
                }
            } else {
                int y[16];
                #pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int4 cc = cst[col + j];
                    y[j] = FAST ? epi_y_fast(hi[j], lo[j], cc.x, cc.y - er, cc.z, ws128(cc)) : epi_y(hi[j], lo[j], cc.x, cc.y - er, cc.z, ws128(cc));
                }
                if constexpr (EPI == EPI_GEGLU) {      // interleaved columns 2c = a_c, 2c+1 = g_c
                    int v[8];
                    #pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const int ge = L2 ? lut_act_s(y[2 * j + 1], L2) : lut_act(y[2 * j + 1], a.Lphi);
                        // sat32(rshr(a * ge, 16)): the funnel shift gives the low word, the high word decides saturation
                        const i64 t = i64(y[2 * j]) * ge + 32768;
                        const int lo = int(__funnelshift_r(uint32_t(t), uint32_t(t >> 32), 16));
                        v[j] = (int(t >> 32) >> 16) == (lo >> 31) ? lo : (t < 0 ? INT_MIN : INT_MAX);
                        mx = max(mx, uabs(v[j]));
                    }
                    int32_t* dst = a.Y + size_t(grow) * a.ldy + (n >> 1);
                    *reinterpret_cast<int4*>(dst) = make_int4(v[0], v[1], v[2], v[3]);
                    *reinterpret_cast<int4*>(dst + 4) = make_int4(v[4], v[5], v[6], v[7]);
                } else if constexpr (EPI == EPI_SPLIT3) {
                    const int part = n >= 2 * a.Cs ? 2 : (n >= a.Cs ? 1 : 0);
                    int32_t* dst = (part == 0 ? a.Y : (part == 1 ? a.Y1 : a.Y2)) + size_t(grow) * a.Cs + (n - part * a.Cs);
                    #pragma unroll
                    for (int j = 0; j < 16; j += 4) *reinterpret_cast<int4*>(dst + j) = make_int4(y[j], y[j + 1], y[j + 2], y[j + 3]);
                }
            }
        }
        if (a.rowmax_out && live && mx) atomicMax(a.rowmax_out + grow, mx);
    }
}

// The shifts s[n] - e[row] of a tile all in [1, 31] (the usual case) take the short epilogue arithmetic; the
// decision is warp-uniform (srange = the tile's min and max s; the caller votes).
// (the general arithmetic stays out of line: it is rare and would otherwise raise the register count of the
// common path)
template <int BN, int SRC, int EPI, int NC, class YB>
__device__ __noinline__ void gemm_epilogue_general(const GemmArgs& a, uint32_t tl, const int4* __restrict__ cst, const int2* __restrict__ L2,
                                                   int m0, int n0, int rl, int c0, int split, int er, YB yb) {
    gemm_epilogue_t<BN, SRC, EPI, NC, false, YB>(a, tl, cst, L2, m0, n0, rl, c0, split, er, yb);
}
template <int BN, int SRC, int EPI, int NC, class YB>
__device__ __forceinline__ void gemm_epilogue(const GemmArgs& a, uint32_t tl, const int4* __restrict__ cst, const int2* __restrict__ L2,
                                              int m0, int n0, int rl, int c0, int split, int er, bool fast, YB yb) {
    if (fast) gemm_epilogue_t<BN, SRC, EPI, NC, true, YB>(a, tl, cst, L2, m0, n0, rl, c0, split, er, yb);
    else gemm_epilogue_general<BN, SRC, EPI, NC, YB>(a, tl, cst, L2, m0, n0, rl, c0, split, er, yb);
}

// Split-K reduction: sum the raw hi/lo partials of every split, then the plain epilogue
// (+ GELU, + residual, + row max).  One thread per 4 columns.
__global__ void gemm_splitk_reduce(const int32_t* __restrict__ partial, int splits, int Mp, int Np, int Mreal, int Nreal,
                                   const int4* __restrict__ cst, const int32_t* __restrict__ e, const uint32_t* __restrict__ rowmax_in, int srcx32,
                                   int32_t* Y, int ldy, const int32_t* R, int gelu, const int32_t* __restrict__ Lphi, uint32_t* rowmax_out);
}  // namespace vela
