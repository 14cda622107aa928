// Persistent W8A16 GEMM on the sm_100a tensor cores: one CTA per SM walks the output tiles
// t = blockIdx.x, blockIdx.x + gridDim.x, ... (column tiles fastest, so the CTAs in flight share A rows in L2).
//
// The arithmetic, operand sources and epilogues are those of gemm_kernel.cuh; this file is the schedule.  Two
// TMEM accumulator buffers (2 x [hi | lo] x BN columns, when 4 BN <= 512) let the epilogue of tile i run while
// the MMAs of tile i+1 accumulate, and the TMA / converter rings run continuously across tile boundaries, so
// the short-K GEMMs of the UNet (K = 320..1280, 5-20 k-blocks per tile) pay no pipeline fill and no TMEM
// allocation per tile.
//
// Warp roles (THREADS = 32 x (2 + NCW + EW + XW)):
//   warp 0            TMA producer: W (and the A-hi / A-lo planes of int8 sources)
//   warp 1            TMEM allocator and MMA issuer (one elected lane)
//   warps 2 .. 1+NCW  int32 sources only (NCW = 8): quantise the staged rows into the swizzled A tiles
//   next 8 or 16      epilogue: warp % 4 selects the TMEM lane quarter, the warps of a quarter split the columns
//   last warp         int32 sources only: TMA of the raw operand into the staging ring, decoupled from the W ring so
//                     the staging runs X_STAGES k-blocks ahead of the converters whatever the MMA progress
// Every wait is bounded; on a timeout the error word is set and each role stops issuing work.
#pragma once
#include "gemm_kernel.cuh"
#include <algorithm>
#include <climits>

namespace vela {

template <int BN, int STAGES, int SRC, int EPI> struct PersistCfg {
    static constexpr bool REG = SRC != SRC_I8;
    static constexpr int BM = 128, BK = 64;
    static constexpr int A_BYTES = BM * BK, W_BYTES = BN * BK;
    static constexpr int STAGE = 2 * A_BYTES + W_BYTES;
    static constexpr int ACC_COLS = 2 * BN;                     // hi | lo of one tile
    static constexpr int ACC_BUFS = 4 * BN <= 512 ? 2 : 1;      // wide tiles (BN > 128) keep one accumulator
    static constexpr int TCOLS = ACC_BUFS * ACC_COLS;
    static constexpr int TMEM_COLS = TCOLS <= 32 ? 32 : (TCOLS <= 64 ? 64 : (TCOLS <= 128 ? 128 : (TCOLS <= 256 ? 256 : 512)));
    static constexpr int NCW = REG ? 8 : 0;
    // epilogue warps: 16 (four per TMEM lane quarter) for planar sources, 8 where converters share the SM, a
    // q|k|v head (64 columns) is one thread's unit, or the tile width is not a multiple of 64 (160 columns: each
    // thread takes 80, a multiple of the 16-column loads)
    static constexpr int EW = (REG || EPI == EPI_QKV || BN % 64 != 0) ? 8 : 16;
    // with two accumulator buffers and 16 epilogue warps, two groups of 8 take alternate tiles (group g drains
    // buffer g), so the latency chains of two tiles' epilogues (constants, residual, TMEM loads, stores) overlap
    // (the GEGLU and split epilogues; the plain one measured faster with all 16 warps on every tile)
    static constexpr int EG = (EW == 16 && ACC_BUFS == 2 && EPI != EPI_PLAIN) ? 2 : 1;
    static constexpr int EWG = EW / EG;                         // epilogue warps per group
    static constexpr int NCOL = BN / (EWG / 4);                // columns of a tile per epilogue thread
    static constexpr int EPI_WARP0 = 2 + NCW;
    static constexpr int XW = REG ? 1 : 0;                      // int32 sources: one more warp issues the staging TMA
    static constexpr int X_WARP = EPI_WARP0 + EW;
    static constexpr int THREADS = 32 * (2 + NCW + EW + XW);
    static constexpr int CTRL = 1024;
    static constexpr bool SLUT = !REG;                          // GELU table staged in shared memory
    static constexpr int OFF_CST = STAGES * STAGE + CTRL;       // [EG][2][BN] column constants (per group, double-buffered)
    static constexpr int OFF_LUT = OFF_CST + EG * 2 * BN * 16;  // int2[LUT_S_ENTRIES]
    // plain epilogue: 32 x 16 int32 boxes (2 KB, 64-byte swizzle) per epilogue warp for the TMA stores of Y.  A
    // thread with several 16-column chunks per tile takes two boxes per warp, one filled while the other's store
    // drains, where they fit (for int32 sources: without costing the staging ring a stage); one chunk, one box.
    static constexpr int YB_ONE = EPI == EPI_PLAIN ? EW * 2048 : 0;
    static constexpr int OFF_YB = (OFF_LUT + (SLUT ? LUT_S_ENTRIES * 8 : 0) + 1023) / 1024 * 1024;
    static constexpr int X_HALF = BM * 128, X_STAGE = 2 * X_HALF;
    static constexpr int XF1 = REG ? (227 * 1024 - 1024 - OFF_YB - YB_ONE) / X_STAGE : 0;
    static constexpr int XF2 = REG ? (227 * 1024 - 1024 - OFF_YB - 2 * YB_ONE) / X_STAGE : 0;
    static constexpr int YB_N = EPI != EPI_PLAIN || NCOL < 32 ? 1
                              : REG ? ((XF2 < 4 ? XF2 : 4) >= (XF1 < 4 ? XF1 : 4) ? 2 : 1)
                                    : (1024 + OFF_YB + 2 * YB_ONE <= 227 * 1024 ? 2 : 1);
    static constexpr int YB_BYTES = YB_N * YB_ONE;
    static constexpr int OFF_X = OFF_YB + YB_BYTES;
    static constexpr int X_FIT = REG ? (227 * 1024 - 1024 - OFF_X) / X_STAGE : 0;
    static constexpr int X_STAGES = X_FIT > 4 ? 4 : X_FIT;
    static constexpr int XR = X_STAGES > 0 ? X_STAGES : 1;     // ring modulus (int8 sources have no staging ring)
    static constexpr int SMEM = 1024 + OFF_X + (X_STAGES > 0 ? X_STAGES : 0) * X_STAGE;
    static_assert(BN % 16 == 0 && BN >= 32 && BN <= 256, "MMA N");
    static_assert(NCOL % 16 == 0 && (EPI != EPI_QKV || NCOL == 64), "epilogue column split");
    static_assert(STAGE % 1024 == 0, "stage alignment");
    static_assert(!REG || X_STAGES >= 2, "int32 sources need a staging ring of at least two stages");
    static_assert(SMEM <= 227 * 1024, "shared memory");
};

template <int BN, int STAGES, int SRC, int EPI>
__global__ void __launch_bounds__(PersistCfg<BN, STAGES, SRC, EPI>::THREADS, 1) gemm_persist_kernel(const __grid_constant__ GemmArgs a) {
    using Cfg = PersistCfg<BN, STAGES, SRC, EPI>;
    constexpr bool REG = Cfg::REG;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align_smem_1024(smem_raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE);
    uint64_t* empty = full + STAGES;
    uint64_t* accf = empty + STAGES;            // [2] accumulator buffer b holds a finished tile
    uint64_t* acce = accf + 2;                  // [2] the epilogue has drained buffer b
    uint64_t* xfull = acce + 2;                 // [4] int32 staging ring
    uint64_t* xempty = xfull + 4;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xempty + 4);
    uint8_t* xstage = smem + Cfg::OFF_X;
    int4* s_cst = reinterpret_cast<int4*>(smem + Cfg::OFF_CST);
    int2* s_lut = reinterpret_cast<int2*>(smem + Cfg::OFF_LUT);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nN = (a.Np + BN - 1) / BN, nM = (a.Mp + Cfg::BM - 1) / Cfg::BM;
    // work unit t = (K split z, row tile, column tile), column tiles fastest; split-K writes raw partials
    const int nMN = nN * nM, kbs = a.kb_per_split, nsplit = (a.nkb + kbs - 1) / kbs;
    const int ntiles = nMN * nsplit;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1 + Cfg::NCW); mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(&accf[b], 1); mbar_init(&acce[b], Cfg::EWG); }
        for (int s = 0; s < 4; ++s) { mbar_init(&xfull[s], 1); mbar_init(&xempty[s], Cfg::NCW > 0 ? Cfg::NCW : 1); }
        mbar_fence_init();
    }
    if (warp == 1) { tmem_alloc(tmem_slot, Cfg::TMEM_COLS); tmem_relinquish(); }
    int lut_in_range = 1;
    if (Cfg::SLUT && a.Lphi) lut_in_range = stage_lut_s(s_lut, a.Lphi);
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&a.tmW);
        if (SRC == SRC_I8) { tma_prefetch_desc(&a.tmA_hi); tma_prefetch_desc(&a.tmA_lo); }
        if (REG && a.xtma) tma_prefetch_desc(&a.tmX);
    }
    tc_fence_before();
    lut_in_range = __syncthreads_and(lut_in_range);
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0 && !a.stall) {
            int g = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
                const int z = t / nMN, r = t - z * nMN, m0 = (r / nN) * Cfg::BM, n0 = (r % nN) * BN;
                const int kb0 = z * kbs, nk = min(a.nkb, kb0 + kbs) - kb0;
                for (int i = 0; i < nk; ++i, ++g) {
                    const int k = (kb0 + i) * Cfg::BK;
                    const int s = g % STAGES;
                    if (!mbar_wait(&empty[s], ((g / STAGES) & 1) ^ 1, a.err, DEVERR_TIMEOUT_EMPTY, a.wait_limit)) { ok = false; break; }
                    uint8_t* st = smem + s * Cfg::STAGE;
                    mbar_arrive_expect_tx(&full[s], Cfg::W_BYTES + (SRC == SRC_I8 ? 2 * Cfg::A_BYTES : 0));
                    tma_load_2d(st + 2 * Cfg::A_BYTES, &a.tmW, &full[s], k, n0);
                    if (SRC == SRC_I8) {
                        tma_load_2d(st, &a.tmA_hi, &full[s], k, m0);
                        tma_load_2d(st + Cfg::A_BYTES, &a.tmA_lo, &full[s], k, m0);
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_i8(128, BN);
            int g = 0, tl = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++tl) {
                const int b = Cfg::ACC_BUFS == 2 ? (tl & 1) : 0, u = Cfg::ACC_BUFS == 2 ? (tl >> 1) : tl;
                if (!mbar_wait(&acce[b], (u & 1) ^ 1, a.err, DEVERR_TIMEOUT_EMPTY, a.wait_limit)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d = tmem + uint32_t(b * Cfg::ACC_COLS);
                const int z = t / nMN, kb0 = z * kbs, nk = min(a.nkb, kb0 + kbs) - kb0;
                for (int i = 0; i < nk; ++i, ++g) {
                    const int s = g % STAGES;
                    if (!mbar_wait(&full[s], (g / STAGES) & 1, a.err, DEVERR_TIMEOUT_FULL, a.wait_limit)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + s * Cfg::STAGE);
                    #pragma unroll
                    for (int kk = 0; kk < 2; ++kk) {
                        const uint64_t bd = sdesc_sw64(sa + 2 * Cfg::A_BYTES + kk * 32);
                        mma_i8(d, sdesc_sw64(sa + kk * 32), bd, idesc, (i | kk) != 0);
                        mma_i8(d + BN, sdesc_sw64(sa + Cfg::A_BYTES + kk * 32), bd, idesc, (i | kk) != 0);
                    }
                    mma_commit(&empty[s]);
                }
                mma_commit(&accf[b]);     // fires when every MMA of this tile has completed
            }
        }
    } else if (REG && warp == Cfg::X_WARP) {
        // ------------------------------------------------------------ int32 staging TMA (runs ahead of the W ring)
        if (lane == 0 && a.xtma && !a.stall) {
            int g = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
                const int z = t / nMN, r = t - z * nMN, m0 = (r / nN) * Cfg::BM;
                const int kb0 = z * kbs, nk = min(a.nkb, kb0 + kbs) - kb0;
                int cb = 0, cy0 = 0;
                if (SRC == SRC_CONV32) { cb = m0 / a.conv_rows_per_img; cy0 = (m0 - cb * a.conv_rows_per_img) / a.Wo; }
                for (int i = 0; i < nk; ++i, ++g) {
                    const int k = (kb0 + i) * Cfg::BK;
                    const int xs = g % Cfg::XR;
                    if (!mbar_wait(&xempty[xs], ((g / Cfg::XR) & 1) ^ 1, a.err, DEVERR_TIMEOUT_EMPTY, a.wait_limit)) { ok = false; break; }
                    mbar_arrive_expect_tx(&xfull[xs], Cfg::X_STAGE);
                    #pragma unroll
                    for (int hf = 0; hf < 2; ++hf) {
                        uint8_t* dst = xstage + xs * Cfg::X_STAGE + hf * Cfg::X_HALF;
                        const int kk = k + hf * 32;
                        if (SRC == SRC_X32) tma_load_2d(dst, &a.tmX, &xfull[xs], kk, m0);
                        else {
                            const int tap = kk / a.C, c0 = kk - tap * a.C, ky = tap / 3, kx = tap - ky * 3;
                            const int yy = tap < 9 ? cy0 * a.stride + ky - 1 : a.H + 8;   // K padding: a box below the image
                            tma_load_4d(dst, &a.tmX, &xfull[xs], tap < 9 ? c0 : 0, kx - 1, yy, cb);
                        }
                    }
                }
            }
        }
    } else if (REG && warp < Cfg::EPI_WARP0) {
        // ------------------------------------------------------------ A producers (int32 sources)
        const int ct = threadIdx.x - 64;                  // 0..255: row = ct & 127, K half = ct >> 7
        volatile uint32_t* xsink = reinterpret_cast<uint32_t*>(smem + STAGES * Cfg::STAGE + 512) + warp;
        const int row = ct & 127, half = ct >> 7;
        int g = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
            const int z = t / nMN, m0 = ((t - z * nMN) / nN) * Cfg::BM;
            const int kb0 = z * kbs, nk = min(a.nkb, kb0 + kbs) - kb0;
            const int grow = m0 + row;
            const bool live = grow < a.Mreal;
            int er = 0, cb = 0, iy0 = 0, ix0 = 0;
            if (SRC == SRC_X32) er = live ? row_exp(a.rowmax_in[grow]) : 0;
            else {
                er = live ? a.e[grow] : 0;
                const int hw = a.Ho * a.Wo; cb = grow / hw; const int p = grow - cb * hw; const int oy = p / a.Wo, ox = p - oy * a.Wo;
                iy0 = oy * a.stride - 1; ix0 = ox * a.stride - 1;
            }
            // quant16(v, e) = clamp(((v >> (e-1)) + 1) >> 1) for e >= 1, clamp(v) for e = 0
            const int qs1 = er > 0 ? er - 1 : 0, qr = er > 0 ? 1 : 0, qs2 = er > 0 ? 1 : 0;
            const int qh = (1 << er) >> 1;
            const bool e15 = __all_sync(0xffffffffu, er <= 15);      // every row of the warp: the two-operation rounding
            for (int i = 0; i < nk; ++i, ++g) {
                int4 v[8];
                const int xs = g % Cfg::XR;
                if (a.xtma) {
                    if (!__all_sync(0xffffffffu, mbar_wait(&xfull[xs], (g / Cfg::XR) & 1, a.err, DEVERR_TIMEOUT_FULL, a.wait_limit))) { ok = false; break; }
                    const uint8_t* xr = xstage + xs * Cfg::X_STAGE + half * Cfg::X_HALF + row * 128;
                    #pragma unroll
                    for (int j = 0; j < 8; ++j) v[j] = *reinterpret_cast<const int4*>(xr + ((j ^ (row & 7)) << 4));
                } else if (SRC == SRC_CONV32 && a.C == 4) {
                    // 4-channel image: the 32 K values are the taps k / 4 .. k / 4 + 7 of one 16-byte pixel each
                    // (taps from 9 on are K padding and read as zero)
                    const int tap0 = ((kb0 + i) * Cfg::BK + half * 32) >> 2;
                    #pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const int tap = tap0 + j, ky = tap / 3, kx = tap - ky * 3, iy = iy0 + ky, ix = ix0 + kx;
                        v[j] = live && tap < 9 && iy >= 0 && iy < a.H && ix >= 0 && ix < a.W
                             ? __ldg(reinterpret_cast<const int4*>(a.img + ((size_t(cb) * a.H + iy) * a.W + ix) * 4)) : make_int4(0, 0, 0, 0);
                    }
                } else {
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
                if (e15) {
                    #pragma unroll
                    for (int j = 0; j < 8; ++j) quant_pack4_e15(v[j].x, v[j].y, v[j].z, v[j].w, qh, er, hw[j], lw[j]);
                } else {
                    #pragma unroll
                    for (int j = 0; j < 8; ++j) quant_pack4(v[j].x, v[j].y, v[j].z, v[j].w, qs1, qr, qs2, hw[j], lw[j]);
                }
                if (a.xtma) {
                    // release the staging slot: a shared-memory store that needs a value of every staged load (hw[j]
                    // depends on load j) precedes the arrive, so no read of the slot is in flight when the TMA refills it
                    if (lane == 0) {
                        *xsink = hw[0] | hw[1] | hw[2] | hw[3] | hw[4] | hw[5] | hw[6] | hw[7];
                        mbar_arrive(&xempty[xs]);
                    }
                }
                const int s = g % STAGES;
                if (!__all_sync(0xffffffffu, mbar_wait(&empty[s], ((g / STAGES) & 1) ^ 1, a.err, DEVERR_TIMEOUT_EMPTY, a.wait_limit))) { ok = false; break; }
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
    } else if (warp < Cfg::EPI_WARP0 + Cfg::EW) {
        // ------------------------------------------------------------ epilogue
        const int ew = warp - Cfg::EPI_WARP0;            // 0 .. EW-1
        const int grp = Cfg::EG == 1 ? 0 : ew / Cfg::EWG, ewg = ew - grp * Cfg::EWG;   // group (tile parity when EG = 2), warp in it
        const int et = ewg * 32 + lane;
        const int q = warp & 3, hq = ewg >> 2;           // TMEM lane quarter (fixed by warp % 4), column slice
        const uint32_t tq = tmem + (uint32_t(q * 32) << 16);
        const int2* lut = (Cfg::SLUT && a.Lphi && lut_in_range) ? s_lut : nullptr;   // else the table in global memory
        uint8_t* yb = (Cfg::YB_BYTES > 0 && a.ytma) ? smem + Cfg::OFF_YB + ew * 2048 * Cfg::YB_N : nullptr;
        YBox yb2{yb, Cfg::YB_N, 0};
        bool ok = true;
        // Every epilogue warp runs every tile of its group and every named barrier, also after a timed-out wait (it
        // then skips the work), so no warp waits on a barrier that another one has left.
        for (int t = blockIdx.x + grp * gridDim.x, tl = grp; t < ntiles; t += Cfg::EG * gridDim.x, tl += Cfg::EG) {
            const int b = Cfg::ACC_BUFS == 2 ? (tl & 1) : 0, u = Cfg::ACC_BUFS == 2 ? (tl >> 1) : tl;
            const int z = t / nMN, r = t - z * nMN, m0 = (r / nN) * Cfg::BM, n0 = (r % nN) * BN;
            // this tile's column constants and the row exponent, fetched while the MMAs run
            int4* cb = s_cst + (Cfg::EG == 1 ? (tl & 1) : grp * 2 + ((tl >> 1) & 1)) * BN;
            for (int i = et; i < BN; i += Cfg::EWG * 32) cb[i] = n0 + i < a.Np ? __ldg(a.cst + n0 + i) : make_int4(1, 0, 0, 0);
            const int grow = m0 + q * 32 + lane;
            int er = 0;
            if (grow < a.Mreal) er = (SRC == SRC_X32) ? row_exp(__ldg(a.rowmax_in + grow)) : __ldg(a.e + grow);
            if (Cfg::EG == 1) asm volatile("bar.sync 2, %0;" :: "r"(Cfg::EWG * 32) : "memory");
            else asm volatile("bar.sync %0, %1;" :: "r"(2 + grp), "r"(Cfg::EWG * 32) : "memory");
            // the tile's range of column shifts s (each lane scans a slice of the staged constants)
            // and of |m| (the short arithmetic forms 256 m in 32 bits)
            int smin = INT_MAX, smax = INT_MIN;
            u32 mbig = 0;
            for (int i = lane; i < BN; i += 32) { const int4 cv = cb[i]; smin = min(smin, cv.y); smax = max(smax, cv.y); mbig |= uabs(cv.x) >> 23; }
            smin = __reduce_min_sync(0xffffffffu, smin); smax = __reduce_max_sync(0xffffffffu, smax);
            const bool fast = a.partial == nullptr && __all_sync(0xffffffffu, smin - er >= 1 && smax - er <= 31 && mbig == 0);
            if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&accf[b], u & 1, a.err, DEVERR_TIMEOUT_ACC, a.wait_limit));
            if (!ok) continue;
            tc_fence_after();
            if constexpr (Cfg::YB_N == 2) gemm_epilogue<BN, SRC, EPI, Cfg::NCOL, YBox&>(a, tq + uint32_t(b * Cfg::ACC_COLS), cb, lut, m0, n0, q * 32 + lane, hq * Cfg::NCOL, z, er, fast, yb2);
            else gemm_epilogue<BN, SRC, EPI, Cfg::NCOL, uint8_t*>(a, tq + uint32_t(b * Cfg::ACC_COLS), cb, lut, m0, n0, q * 32 + lane, hq * Cfg::NCOL, z, er, fast, yb);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acce[b]);
        }
        if (yb && lane == 0) bulk_wait0();        // every TMA store of Y has completed before the CTA exits
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) { tc_fence_after(); tmem_dealloc(tmem, Cfg::TMEM_COLS); }
}

template <int BN, int STAGES, int SRC, int EPI>
void launch_gemm_persist(const GemmArgs& a, cudaStream_t st) {
    using Cfg = PersistCfg<BN, STAGES, SRC, EPI>;
    auto kern = gemm_persist_kernel<BN, STAGES, SRC, EPI>;
    static std::atomic<int> attr_done[64];
    once_per_device(attr_done, [&] { VELA_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM)); });
    VELA_REQUIRE(a.kb_per_split > 0 && (a.partial != nullptr) == (a.kb_per_split < a.nkb) && (EPI == EPI_PLAIN || a.partial == nullptr),
                 "gemm: split-K needs a workspace and the plain epilogue");
    const int tiles = ceil_div(a.Np, BN) * ceil_div(a.Mp, 128) * ceil_div(a.nkb, a.kb_per_split);
    const int grid = std::min(tiles, sm_count());
    kern<<<grid, Cfg::THREADS, Cfg::SMEM, st>>>(a);
    VELA_CUDA(cudaGetLastError());
}

}  // namespace vela
