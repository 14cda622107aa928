// W8A16 hi/lo GEMM on the sm_100a tensor cores (tcgen05.mma kind::i8).
//
// Computes, for output row r and column n (the semantics of the reference's
// gemm_hl kernel, src/gemm_hl.cu:40-52,175-309):
//     acc = 256 * (Ahi[r] . W[n]) + Alo[r] . W[n] + 128 * wsum[n]      (= sum_k q[r,k] W[n,k])
//     y   = sat32(rshr(acc * m[n], s[n] - e[r]) + b[n])
// followed by one of the fused epilogues (plain / GELU / + residual / row max,
// GEGLU, q|k|v head quantisation, 3-way split), or raw s32 partials for split-K.
//
// Layout on chip.  A CTA owns a 128-row x BN-column output tile.  Each K step
// of 64 bytes stages three K-major tiles with the 64-byte swizzle in shared
// memory: A-hi [128 x 64], A-lo [128 x 64] and W [BN x 64].  One elected
// thread issues, per 32-byte K slice, two tcgen05.mma (M=128, N=BN, K=32):
// A-hi x W into TMEM columns [0, BN) and A-lo x W into [BN, 2 BN), so the
// two s32 accumulators never leave the tensor memory until the epilogue.
//
// Warp roles (320 threads):
//   warp 0      TMA producer: W (and A-hi / A-lo for planar int8 operands)
//   warp 1      TMEM allocator and MMA issuer
//   warps 2..9  for int32 operands (SRC_X32, SRC_CONV32) the A producers:
//               each thread loads 32 int32 of one row, quantises them with
//               the row's exponent and writes the hi/lo bytes into the
//               swizzled tiles (TMA cannot quantise); then all eight warps run
//               the epilogue: tcgen05.ld of their 32 TMEM lanes (warp % 4 picks
//               the lane quarter, the two warps of a quarter split the columns).
// Every barrier wait is bounded; a timeout writes the error word and the
// CTA drains to the common exit, where TMEM is released.
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
    unsigned* err;
};

template <int BN, int STAGES> struct GemmCfg {
    static constexpr int BM = 128, BK = 64;
    static constexpr int A_BYTES = BM * BK;                  // one plane, 8 KB
    static constexpr int W_BYTES = BN * BK;
    static constexpr int STAGE = 2 * A_BYTES + W_BYTES;      // multiple of 1024
    static constexpr int TMEM_COLS = (2 * BN <= 32) ? 32 : (2 * BN <= 64 ? 64 : (2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512)));
    static constexpr int CTRL = 1024;                        // barriers + TMEM slot
    static constexpr int SMEM = 1024 /*align slack*/ + STAGES * STAGE + CTRL + BN * 16 /*column constants*/;
    // int32 staging ring (SRC_X32 / SRC_CONV32 through TMA): one k-block = two boxes of 128 rows x 32 int32
    // (128-byte rows, 128-byte swizzle), as many stages as fit beside the MMA ring (at most 4)
    static constexpr int X_HALF = BM * 128;
    static constexpr int X_STAGE = 2 * X_HALF;
    static constexpr int OFF_X = (STAGES * STAGE + CTRL + BN * 16 + 1023) / 1024 * 1024;
    static constexpr int X_FIT = (227 * 1024 - 1024 - OFF_X) / X_STAGE;
    static constexpr int X_STAGES = X_FIT > 4 ? 4 : X_FIT;
    static constexpr int SMEM_X = 1024 + OFF_X + (X_STAGES > 0 ? X_STAGES : 0) * X_STAGE;
    static constexpr int THREADS = 320;
    static_assert(BN % 16 == 0 && BN >= 32 && BN <= 256, "MMA N");
    static_assert(STAGE % 1024 == 0, "stage alignment");
};

__device__ __forceinline__ int ws128(int4 c) { return 128 * c.w; }

template <int BN, int STAGES, int SRC, int EPI>
__global__ void __launch_bounds__(320, 1) gemm_w8a16_kernel(const __grid_constant__ GemmArgs a) {
    using Cfg = GemmCfg<BN, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE);
    uint64_t* empty = full + STAGES;
    uint64_t* accb = empty + STAGES;
    uint64_t* xfull = accb + 1;                      // int32 staging ring (xtma)
    uint64_t* xempty = xfull + 4;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xempty + 4);
    uint8_t* xstage = smem + Cfg::OFF_X;
    int4* s_cst = reinterpret_cast<int4*>(smem + STAGES * Cfg::STAGE + Cfg::CTRL);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * Cfg::BM;
    const int kb0 = blockIdx.z * a.kb_per_split;
    const int kb1 = min(a.nkb, kb0 + a.kb_per_split);
    const int nk = kb1 - kb0;
    constexpr bool REG = SRC != SRC_I8;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1 + (REG ? 8 : 0)); mbar_init(&empty[s], 1); }
        mbar_init(accb, 1);
        for (int s = 0; s < 4; ++s) { mbar_init(&xfull[s], 1); mbar_init(&xempty[s], 8); }
        mbar_fence_init();
    }
    if (warp == 1) { tmem_alloc(tmem_slot, Cfg::TMEM_COLS); tmem_relinquish(); }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&a.tmW);
        if (SRC == SRC_I8) { tma_prefetch_desc(&a.tmA_hi); tma_prefetch_desc(&a.tmA_lo); }
        if (REG && a.xtma) tma_prefetch_desc(&a.tmX);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            int cb = 0, cy0 = 0;                     // SRC_CONV32 + xtma: image and first output row of this tile
            if (SRC == SRC_CONV32 && a.xtma) { cb = m0 / a.conv_rows_per_img; cy0 = (m0 - cb * a.conv_rows_per_img) / a.Wo; }
            for (int i = 0; i < nk; ++i) {
                const int s = i % STAGES; const uint32_t ph = (i / STAGES) & 1;
                const int k = (kb0 + i) * Cfg::BK;
                if constexpr (REG && Cfg::X_STAGES > 0) {
                    if (a.xtma) {
                        // stage the int32 operand of this k-block (zeros outside the matrix / image)
                        const int xs = i % Cfg::X_STAGES;
                        if (!mbar_wait(&xempty[xs], ((i / Cfg::X_STAGES) & 1) ^ 1, a.err, DEVERR_TIMEOUT_EMPTY)) break;
                        mbar_arrive_expect_tx(&xfull[xs], Cfg::X_STAGE);
                        #pragma unroll
                        for (int hf = 0; hf < 2; ++hf) {
                            uint8_t* dst = xstage + xs * Cfg::X_STAGE + hf * Cfg::X_HALF;
                            const int kk = k + hf * 32;
                            if (SRC == SRC_X32) tma_load_2d(dst, &a.tmX, &xfull[xs], kk, m0);
                            else {
                                const int tap = kk / a.C, c0 = kk - tap * a.C, ky = tap / 3, kx = tap - ky * 3;
                                // taps past the ninth (K padding) read a box wholly below the image: zeros
                                const int yy = tap < 9 ? cy0 * a.stride + ky - 1 : a.H + 8;
                                tma_load_4d(dst, &a.tmX, &xfull[xs], tap < 9 ? c0 : 0, kx - 1, yy, cb);
                            }
                        }
                    }
                }
                if (!mbar_wait(&empty[s], ph ^ 1, a.err, DEVERR_TIMEOUT_EMPTY)) break;
                uint8_t* st = smem + s * Cfg::STAGE;
                mbar_arrive_expect_tx(&full[s], Cfg::W_BYTES + (SRC == SRC_I8 ? 2 * Cfg::A_BYTES : 0));
                tma_load_2d(st + 2 * Cfg::A_BYTES, &a.tmW, &full[s], k, n0);
                if (SRC == SRC_I8) {
                    tma_load_2d(st, &a.tmA_hi, &full[s], k, m0);
                    tma_load_2d(st + Cfg::A_BYTES, &a.tmA_lo, &full[s], k, m0);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_i8(128, BN);
            bool ok = true;
            for (int i = 0; i < nk && ok; ++i) {
                const int s = i % STAGES; const uint32_t ph = (i / STAGES) & 1;
                if (!mbar_wait(&full[s], ph, a.err, DEVERR_TIMEOUT_FULL)) { ok = false; break; }
                tc_fence_after();
                const uint32_t sa = smem_u32(smem + s * Cfg::STAGE);
                #pragma unroll
                for (int kk = 0; kk < 2; ++kk) {
                    const uint64_t bd = sdesc_sw64(sa + 2 * Cfg::A_BYTES + kk * 32);
                    mma_i8(tmem, sdesc_sw64(sa + kk * 32), bd, idesc, (i | kk) != 0);
                    mma_i8(tmem + BN, sdesc_sw64(sa + Cfg::A_BYTES + kk * 32), bd, idesc, (i | kk) != 0);
                }
                mma_commit(&empty[s]);
            }
            mma_commit(accb);     // fires once every MMA above has completed (also when nothing was issued)
        }
    } else {
        const int ct = threadIdx.x - 64;          // 0..255
        // stage the column constants while the main loop runs
        for (int i = ct; i < BN; i += 256) { const int n = n0 + i; s_cst[i] = n < a.Np ? a.cst[n] : make_int4(1, 0, 0, 0); }
        if constexpr (REG) {
            // -------------------------------------------------------- A producers: int32 -> hi/lo planes
            const int row = ct & 127, half = ct >> 7;      // thread = one row, 32 of the 64 K bytes
            const int grow = m0 + row;
            const bool live = grow < a.Mreal;
            int er = 0;
            int cb = 0, iy0 = 0, ix0 = 0;
            if (SRC == SRC_X32) { er = live ? row_exp(a.rowmax_in[grow]) : 0; }
            else {
                er = live ? a.e[grow] : 0;
                const int hw = a.Ho * a.Wo; cb = grow / hw; const int p = grow - cb * hw; const int oy = p / a.Wo, ox = p - oy * a.Wo;
                iy0 = oy * a.stride - 1; ix0 = ox * a.stride - 1;
            }
            for (int i = 0; i < nk; ++i) {
                const int s = i % STAGES; const uint32_t ph = (i / STAGES) & 1;
                int4 v[8];
                bool staged = false;
                if constexpr (Cfg::X_STAGES > 0) {
                    if (a.xtma) {
                        // this thread's 32 int32 from the staging ring (128-byte swizzle: chunk j at j ^ (row & 7))
                        const int xs = i % Cfg::X_STAGES;
                        if (!__all_sync(0xffffffffu, mbar_wait(&xfull[xs], (i / Cfg::X_STAGES) & 1, a.err, DEVERR_TIMEOUT_FULL))) break;
                        const uint8_t* xr = xstage + xs * Cfg::X_STAGE + half * Cfg::X_HALF + row * 128;
                        #pragma unroll
                        for (int j = 0; j < 8; ++j) v[j] = *reinterpret_cast<const int4*>(xr + ((j ^ (row & 7)) << 4));
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&xempty[xs]);
                        staged = true;
                    }
                }
                if (!mbar_wait(&empty[s], ph ^ 1, a.err, DEVERR_TIMEOUT_EMPTY)) break;
                if (!staged) {
                    const int k = (kb0 + i) * Cfg::BK + half * 32;
                    const int32_t* src = nullptr;
                    if (live && k < a.K) {
                        if (SRC == SRC_X32) src = a.x + size_t(grow) * a.ldx + k;
                        else {
                            const int tap = k / a.C, c0 = k - tap * a.C, ky = tap / 3, kx = tap - ky * 3;
                            const int iy = iy0 + ky, ix = ix0 + kx;
                            if (iy >= 0 && iy < a.H && ix >= 0 && ix < a.W) src = a.img + ((size_t(cb) * a.H + iy) * a.W + ix) * a.C + c0;
                        }
                    }
                    if (src) {
                        #pragma unroll
                        for (int j = 0; j < 8; ++j) v[j] = __ldg(reinterpret_cast<const int4*>(src) + j);
                    } else {
                        #pragma unroll
                        for (int j = 0; j < 8; ++j) v[j] = make_int4(0, 0, 0, 0);
                    }
                }
                uint32_t hw[8], lw[8];
                #pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int q0 = quant16(v[j].x, er), q1 = quant16(v[j].y, er), q2 = quant16(v[j].z, er), q3 = quant16(v[j].w, er);
                    hw[j] = pack_hi4(q0, q1, q2, q3); lw[j] = pack_lo4(q0, q1, q2, q3);
                }
                uint8_t* st = smem + s * Cfg::STAGE;
                *reinterpret_cast<uint4*>(st + sw64_off(row, half * 2)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                *reinterpret_cast<uint4*>(st + sw64_off(row, half * 2 + 1)) = make_uint4(hw[4], hw[5], hw[6], hw[7]);
                *reinterpret_cast<uint4*>(st + Cfg::A_BYTES + sw64_off(row, half * 2)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
                *reinterpret_cast<uint4*>(st + Cfg::A_BYTES + sw64_off(row, half * 2 + 1)) = make_uint4(lw[4], lw[5], lw[6], lw[7]);
                fence_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&full[s]);
            }
        }
        // ------------------------------------------------------------ epilogue
        asm volatile("bar.sync 1, 256;" ::: "memory");          // column constants staged (epilogue warps only)
        const bool ok = __all_sync(0xffffffffu, mbar_wait(accb, 0, a.err, DEVERR_TIMEOUT_ACC));   // warp-uniform: tcgen05.ld is warp-collective
        tc_fence_after();
        if (ok) {
            const int q = warp & 3, h = (warp - 2) >> 2;
            const int rl = q * 32 + lane, grow = m0 + rl;
            const uint32_t tl = tmem + (uint32_t(q * 32) << 16);
            const bool live = grow < a.Mreal;
            int er = 0;
            if (live) er = (SRC == SRC_X32) ? row_exp(a.rowmax_in[grow]) : a.e[grow];
            constexpr int HALF = BN / 2;
            if constexpr (EPI == EPI_QKV) {
                static_assert(BN == 128, "q|k|v epilogue works on one 64-column head per thread");
                int y[64];
                #pragma unroll
                for (int c = 0; c < 4; ++c) {
                    int hi[16], lo[16];
                    tmem_ld16(tl + h * 64 + c * 16, hi); tmem_ld16(tl + BN + h * 64 + c * 16, lo); tmem_ld_wait();
                    #pragma unroll
                    for (int j = 0; j < 16; ++j) { const int4 cc = s_cst[h * 64 + c * 16 + j]; y[c * 16 + j] = epi_y(hi[j], lo[j], cc.x, cc.y - er, cc.z, ws128(cc)); }
                }
                const int nh = n0 + h * 64;
                if (live && nh < a.Nreal) {
                    const int part = nh / a.Cq, head = (nh - part * a.Cq) >> 6;
                    if (part == 2) {
                        int4* dst = reinterpret_cast<int4*>(a.Y2 + size_t(grow) * a.Cq + head * 64);
                        #pragma unroll
                        for (int j = 0; j < 16; ++j) dst[j] = make_int4(y[4 * j], y[4 * j + 1], y[4 * j + 2], y[4 * j + 3]);
                    } else {
                        u32 m = 0;
                        #pragma unroll
                        for (int j = 0; j < 64; ++j) m = max(m, uabs(y[j]));
                        const int ee = row_exp(m);
                        const int b = grow / a.T, t = grow - b * a.T;
                        const int Tp = part == 0 ? a.TpQ : a.TpK;
                        const size_t gt = size_t(b * a.heads + head) * Tp + t;
                        int8_t* hip = (part == 0 ? a.qhi : a.khi) + gt * 64; int8_t* lop = (part == 0 ? a.qlo : a.klo) + gt * 64;
                        int hs = 0, ls = 0, ts = 0;
                        #pragma unroll
                        for (int j = 0; j < 16; j += 4) {
                            uint32_t hw[4], lw[4];
                            #pragma unroll
                            for (int u = 0; u < 4; ++u) {
                                const int b4 = (j + u) * 4;
                                const int q0 = quant16(y[b4], ee), q1 = quant16(y[b4 + 1], ee), q2 = quant16(y[b4 + 2], ee), q3 = quant16(y[b4 + 3], ee);
                                hw[u] = pack_hi4(q0, q1, q2, q3); lw[u] = pack_lo4(q0, q1, q2, q3);
                                hs += (q0 >> 8) + (q1 >> 8) + (q2 >> 8) + (q3 >> 8);
                                ls += ((q0 & 255) - 128) + ((q1 & 255) - 128) + ((q2 & 255) - 128) + ((q3 & 255) - 128);
                                ts += q0 + q1 + q2 + q3;
                            }
                            *reinterpret_cast<uint4*>(hip + j * 4) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                            *reinterpret_cast<uint4*>(lop + j * 4) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
                        }
                        (part == 0 ? a.qe : a.ke)[gt] = ee;
                        (part == 0 ? a.qhs : a.khs)[gt] = hs;
                        (part == 0 ? a.qls : a.kls)[gt] = ls;
                        (part == 0 ? a.qts : a.kts)[gt] = ts;
                    }
                }
            } else {
                u32 mx = 0;
                #pragma unroll 1
                for (int c = 0; c < HALF / 16; ++c) {
                    const int col = h * HALF + c * 16, n = n0 + col;
                    int hi[16], lo[16];
                    tmem_ld16(tl + col, hi); tmem_ld16(tl + BN + col, lo); tmem_ld_wait();
                    if (!live || n >= a.Nreal) continue;
                    if (a.partial) {             // split-K: raw accumulators, reduced by gemm_splitk_reduce
                        int32_t* ph = a.partial + (size_t(blockIdx.z) * 2 * a.Mp + grow) * a.Np + n;
                        int32_t* pl = ph + size_t(a.Mp) * a.Np;
                        #pragma unroll
                        for (int j = 0; j < 16; j += 4) {
                            *reinterpret_cast<int4*>(ph + j) = make_int4(hi[j], hi[j + 1], hi[j + 2], hi[j + 3]);
                            *reinterpret_cast<int4*>(pl + j) = make_int4(lo[j], lo[j + 1], lo[j + 2], lo[j + 3]);
                        }
                        continue;
                    }
                    int y[16];
                    #pragma unroll
                    for (int j = 0; j < 16; ++j) { const int4 cc = s_cst[col + j]; y[j] = epi_y(hi[j], lo[j], cc.x, cc.y - er, cc.z, ws128(cc)); }
                    if constexpr (EPI == EPI_PLAIN) {
                        const bool full16 = n + 16 <= a.Nreal;
                        if (a.gelu) {
                            #pragma unroll
                            for (int j = 0; j < 16; ++j) y[j] = lut_act(y[j], a.Lphi);
                        }
                        if (a.R) {
                            const int32_t* rp = a.R + size_t(grow) * a.ldy + n;
                            #pragma unroll
                            for (int j = 0; j < 16; ++j) if (full16 || n + j < a.Nreal) y[j] = int(sat32(i64(y[j]) + __ldg(rp + j)));
                        }
                        int32_t* dst = a.Y + size_t(grow) * a.ldy + n;
                        if (full16 && (a.ldy & 3) == 0) {
                            #pragma unroll
                            for (int j = 0; j < 16; j += 4) *reinterpret_cast<int4*>(dst + j) = make_int4(y[j], y[j + 1], y[j + 2], y[j + 3]);
                        } else {
                            for (int j = 0; j < 16; ++j) if (n + j < a.Nreal) dst[j] = y[j];
                        }
                        #pragma unroll
                        for (int j = 0; j < 16; ++j) if (full16 || n + j < a.Nreal) mx = max(mx, uabs(y[j]));
                    } else if constexpr (EPI == EPI_GEGLU) {      // interleaved columns 2c = a_c, 2c+1 = g_c
                        int v[8];
                        #pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const int ge = lut_act(y[2 * j + 1], a.Lphi);
                            v[j] = int(rshr_pos(i64(y[2 * j]) * ge, 16));
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
                if (a.rowmax_out && live && mx) atomicMax(a.rowmax_out + grow, mx);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) { tc_fence_after(); tmem_dealloc(tmem, Cfg::TMEM_COLS); }
}

// Split-K reduction: sum the raw hi/lo partials of every split, then the plain epilogue
// (+ GELU, + residual, + row max).  One thread per 4 columns.
__global__ void gemm_splitk_reduce(const int32_t* __restrict__ partial, int splits, int Mp, int Np, int Mreal, int Nreal,
                                   const int4* __restrict__ cst, const int32_t* __restrict__ e, const uint32_t* __restrict__ rowmax_in, int srcx32,
                                   int32_t* Y, int ldy, const int32_t* R, int gelu, const int32_t* __restrict__ Lphi, uint32_t* rowmax_out);
template <int BN, int STAGES, int SRC, int EPI>
void launch_gemm(const GemmArgs& a, int splits, cudaStream_t st) {
    using Cfg = GemmCfg<BN, STAGES>;
    auto kern = gemm_w8a16_kernel<BN, STAGES, SRC, EPI>;
    constexpr int SMEM_MAX = (SRC != SRC_I8 && Cfg::X_STAGES > 0) ? Cfg::SMEM_X : Cfg::SMEM;
    static int attr_done[64] = {0};
    const int dev = current_device();
    if (dev >= 64 || !attr_done[dev]) {
        VELA_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_MAX));
        if (dev < 64) attr_done[dev] = 1;
    }
    VELA_REQUIRE(!a.xtma || (SRC != SRC_I8 && Cfg::X_STAGES > 0), "gemm: TMA-staged int32 operand without a staging ring");
    dim3 grid(ceil_div(a.Np, BN), ceil_div(a.Mp, 128), splits);
    kern<<<grid, Cfg::THREADS, a.xtma ? Cfg::SMEM_X : Cfg::SMEM, st>>>(a);
    VELA_CUDA(cudaGetLastError());
}

}  // namespace vela
