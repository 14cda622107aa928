// Host dispatch of the tcgen05 W8A16 GEMM and its C-ABI entry points.
// Replaces the reference's k_gemm_hl / k_gemm_hl2 (src/gemm_hl.h:27-33) and,
// for deep K, its cuBLASLt + k_epilogue path (src/engine.cu:153-157).
#include "gemm_kernel.cuh"
#include "gemm_persist.cuh"
#include "host_util.h"
#include "ops.h"
#include "vela_b200.h"
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <string>

namespace vela {

static __device__ unsigned g_gemm_err;

__global__ void gemm_splitk_reduce(const int32_t* __restrict__ partial, int splits, int Mp, int Np, int Mreal, int Nreal,
                                   const int4* __restrict__ cst, const int32_t* __restrict__ e, const uint32_t* __restrict__ rowmax_in, int srcx32,
                                   int32_t* Y, int ldy, const int32_t* R, int gelu, const int32_t* __restrict__ Lphi, uint32_t* rowmax_out) {
    const int tpr = Nreal >> 2;
    const size_t idx = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= size_t(Mreal) * tpr) return;
    const int r = int(idx / tpr), n = int(idx - size_t(r) * tpr) * 4;
    int4 hs = make_int4(0, 0, 0, 0), ls = make_int4(0, 0, 0, 0);
    for (int s = 0; s < splits; ++s) {
        const int4 h = *reinterpret_cast<const int4*>(partial + (size_t(s) * 2 * Mp + r) * Np + n);
        const int4 l = *reinterpret_cast<const int4*>(partial + ((size_t(s) * 2 + 1) * Mp + r) * Np + n);
        hs.x += h.x; hs.y += h.y; hs.z += h.z; hs.w += h.w; ls.x += l.x; ls.y += l.y; ls.z += l.z; ls.w += l.w;
    }
    const int er = srcx32 ? row_exp(rowmax_in[r]) : e[r];
    const int hv[4] = {hs.x, hs.y, hs.z, hs.w}, lv[4] = {ls.x, ls.y, ls.z, ls.w};
    int y[4]; u32 mx = 0;
    #pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int4 c = cst[n + j];
        int v = epi_y(hv[j], lv[j], c.x, c.y - er, c.z, 128 * c.w);
        if (gelu) v = lut_act(v, Lphi);
        if (R) v = int(sat32(i64(v) + R[size_t(r) * ldy + n + j]));
        y[j] = v; mx = max(mx, uabs(v));
    }
    *reinterpret_cast<int4*>(Y + size_t(r) * ldy + n) = make_int4(y[0], y[1], y[2], y[3]);
    if (rowmax_out && mx) atomicMax(rowmax_out + r, mx);
}

// the instantiations live in gemm_inst_*.cu
#define VELA_PERSIST_EXTERN(BN, ST, SRC, EPI) extern template void launch_gemm_persist<BN, ST, SRC, EPI>(const GemmArgs&, cudaStream_t);
VELA_PERSIST_EXTERN(64, 6, SRC_I8, EPI_PLAIN) VELA_PERSIST_EXTERN(128, 6, SRC_I8, EPI_PLAIN) VELA_PERSIST_EXTERN(160, 6, SRC_I8, EPI_PLAIN) VELA_PERSIST_EXTERN(256, 5, SRC_I8, EPI_PLAIN) VELA_PERSIST_EXTERN(128, 6, SRC_I8, EPI_GEGLU)
VELA_PERSIST_EXTERN(128, 6, SRC_I8, EPI_SPLIT3) VELA_PERSIST_EXTERN(128, 6, SRC_I8, EPI_QKV)
#define VELA_PERSIST_REG(SRC) VELA_PERSIST_EXTERN(64, 4, SRC, EPI_PLAIN) VELA_PERSIST_EXTERN(128, 4, SRC, EPI_PLAIN) \
    VELA_PERSIST_EXTERN(160, 4, SRC, EPI_PLAIN)
VELA_PERSIST_REG(SRC_X32) VELA_PERSIST_REG(SRC_CONV32)

namespace {
// int32 sources: up to 160 columns (two 160-wide hi | lo accumulators fill the tensor memory; wider tiles measured
// slower on the UNet's convs, their one accumulator buffer leaving the MMAs idle for a longer epilogue)
constexpr int REG_BNS[3] = {64, 128, 160};

template <int SRC> void dispatch_reg(int BN, const GemmArgs& a, cudaStream_t st) {
    switch (BN) {
        case 64: launch_gemm_persist<64, 4, SRC, EPI_PLAIN>(a, st); break;
        case 128: launch_gemm_persist<128, 4, SRC, EPI_PLAIN>(a, st); break;
        default: launch_gemm_persist<160, 4, SRC, EPI_PLAIN>(a, st); break;
    }
}

struct Plan { int bn, splits; };

// Tile width and K splits from a cost model of the persistent kernel, in units of one 128 x 64 x 64 MMA k-block:
// a work unit (tile, K range) costs its k-blocks x (operand cost + BN / 64); int32 sources pay the quantising of the
// 128 x 64 A block again for every column tile (measured ~10 units), planar sources only the TMA (~0.5).  The units
// are spread over the SMs in waves; a K split adds the partial-sum traffic of its reduction.
// Planar sources with deep K (>= 32 k-blocks, where the epilogue is rare) are bound by the operands' flow into shared
// memory instead: ~40 bytes per SM clock measured whatever the tile width, against 512 clocks of MMAs per k-block (two
// planes x two K steps of 32, each B operand fetched once for both planes) -- per k-block max(512, (2 x 128 + BN) x 64
// / 40) clocks = 1.5 / 1.8 / 1.95 / 2.4 units at BN = 64 / 128 / 160 / 256.  160- and 256-column tiles keep a single
// accumulator buffer (the epilogue does not overlap the next tile's MMAs): 160 is weighed for deep K only, 256 only
// when every unit runs in one wave.
Plan plan(int src, int epi, int Mp, int Mreal, int Np, int Nreal, int nkb, size_t workspace, int sms) {
    if (epi != EPI_PLAIN) return {128, 1};
    const bool reg = src != VELA_SRC_I8, deep = !reg && nkb >= 32;
    const double per_kb = reg ? 10.0 : 0.5, us_per_unit = 0.065;
    const int nM = ceil_div(Mp, 128);
    Plan best{reg ? 128 : 64, 1};
    double best_t = 1e30;
    const int nb = reg ? 3 : (deep ? 4 : 2);
    const int i8_bns[4] = {64, 128, 160, 256};
    const double deep_cost[4] = {1.5, 1.8, 1.95, 2.4};
    for (int i = 0; i < nb; ++i) {
        const int bn = reg ? REG_BNS[i] : i8_bns[i];
        if (!reg && bn == 128 && Nreal % 128 != 0 && Nreal > 128) continue;
        const int nN = ceil_div(Np, bn);
        for (int s = 1; s <= 8; ++s) {
            if (s > 1 && (size_t(s) * 2 * Mp * Np * 4 > workspace || ceil_div(nkb, s) < 4)) break;
            const int kbs = ceil_div(nkb, s), units = nN * nM * s;
            if (bn == 256 && units > sms) break;
            const double waves = double(ceil_div(units, sms));
            double t = waves * kbs * (deep ? deep_cost[i] : per_kb + bn / 64.0) * us_per_unit;
            if (s > 1) t += (double(s) * 8 + 8) * Mreal * Nreal / 6.0e6 + 3.0;     // partials in and out of HBM + a launch
            if (t < best_t * 0.98) { best_t = t; best = {bn, s}; }
        }
    }
    return best;
}
}  // namespace

void gemm_w8a16(cudaStream_t st, const vela_asrc& A, int Mp, int Mreal, const int8_t* W, int ldw, int Np, int Nreal, int Kp,
                const int32_t* cst, const vela_aepi& E, const LaunchOpts& o) {
    VELA_REQUIRE(Mp > 0 && Mreal > 0 && Mreal <= Mp && Nreal > 0 && Nreal <= Np && Kp > 0, "gemm: bad M/N/K");
    VELA_REQUIRE(Kp % 16 == 0 && ldw % 16 == 0 && ldw >= Kp && Np % 16 == 0, "gemm: Kp, ldw and Np must be multiples of 16");
    VELA_REQUIRE(W && cst, "gemm: null weights");
    VELA_REQUIRE((reinterpret_cast<uintptr_t>(W) & 15) == 0, "gemm: W must be 16-byte aligned");
    GemmArgs a;
    std::memset(static_cast<void*>(&a), 0, sizeof(a));
    a.Mreal = Mreal; a.Nreal = Nreal; a.Np = Np; a.Mp = Mp; a.Kp = Kp;
    a.nkb = ceil_div(Kp, 64);
    a.cst = reinterpret_cast<const int4*>(cst);
    a.Y = E.Y; a.ldy = E.ldy; a.R = E.residual; a.Lphi = E.Lphi; a.rowmax_out = E.rowmax;
    a.rvec = E.residual && (E.ldy & 3) == 0 && (reinterpret_cast<uintptr_t>(E.residual) & 15) == 0;
    a.gelu = E.epi == VELA_EPI_GELU;
    a.Cs = E.Cs; a.Y1 = E.Y1; a.Y2 = E.Y2;
    a.heads = E.heads; a.T = E.T; a.TpQ = E.TpQ; a.TpK = E.TpK; a.Cq = E.C;
    a.qhi = E.qhi; a.qlo = E.qlo; a.khi = E.khi; a.klo = E.klo; a.qe = E.qe; a.ke = E.ke;
    a.qhs = E.qhs; a.qls = E.qls; a.qts = E.qts; a.khs = E.khs; a.kls = E.kls; a.kts = E.kts;
    a.err = o.err ? o.err : device_error_word(&g_gemm_err);
    a.wait_limit = o.wait_limit > 0 ? o.wait_limit : WAIT_LIMIT_CYCLES;
    a.stall = o.stall;
    const int epi = E.epi == VELA_EPI_GELU ? EPI_PLAIN : E.epi;
    VELA_REQUIRE(epi >= 0 && epi <= EPI_QKV, "gemm: unknown epilogue");
    if (epi == EPI_PLAIN) VELA_REQUIRE(E.Y && E.ldy >= Nreal, "gemm: plain epilogue needs Y and ldy >= N");
    if (epi == EPI_GELU || E.epi == VELA_EPI_GELU || epi == EPI_GEGLU) VELA_REQUIRE(E.Lphi != nullptr, "gemm: GELU/GEGLU need the phi LUT");
    if (epi == EPI_GEGLU) VELA_REQUIRE(Nreal % 16 == 0 && E.Y && E.ldy >= Nreal / 2 && E.ldy % 4 == 0, "gemm: GEGLU needs N % 16 == 0 and ldy >= N/2, ldy % 4 == 0");
    if (epi == EPI_SPLIT3) VELA_REQUIRE(E.Cs % 16 == 0 && Nreal == 3 * E.Cs && E.Y && E.Y1 && E.Y2, "gemm: split3 needs N = 3*Cs, Cs % 16 == 0");
    if (epi == EPI_QKV) VELA_REQUIRE(E.C % 64 == 0 && (Nreal == 3 * E.C || Nreal == E.C) && E.C == E.heads * 64 && E.T > 0 && Mreal % E.T == 0 && E.qhi &&
                                     (Nreal == E.C || (E.Y2 && E.khi)), "gemm: q|k|v epilogue needs N = 3C (or N = C: q only), C = 64*heads, rows = B*T");

    const int src = A.src;
    if (src == VELA_SRC_I8) {
        VELA_REQUIRE(A.hi && A.lo && A.e && A.ld8 % 16 == 0 && A.ld8 >= Kp, "gemm: int8 planes need hi, lo, e and ld8 % 16 == 0");
        VELA_REQUIRE((reinterpret_cast<uintptr_t>(A.hi) & 15) == 0 && (reinterpret_cast<uintptr_t>(A.lo) & 15) == 0, "gemm: planes must be 16-byte aligned");
        a.e = A.e;
        a.tmA_hi = tmap2d(A.hi, CU_TENSOR_MAP_DATA_TYPE_UINT8, uint64_t(Kp), uint64_t(Mp), uint64_t(A.ld8), 64, 128, Swz::B64);
        a.tmA_lo = tmap2d(A.lo, CU_TENSOR_MAP_DATA_TYPE_UINT8, uint64_t(Kp), uint64_t(Mp), uint64_t(A.ld8), 64, 128, Swz::B64);
    } else if (src == VELA_SRC_X32) {
        VELA_REQUIRE(A.x && A.rowmax && A.K > 0 && A.K % 32 == 0 && A.K <= Kp && A.ldx >= A.K && A.ldx % 4 == 0, "gemm: int32 source needs K % 32 == 0, ldx % 4 == 0");
        VELA_REQUIRE((reinterpret_cast<uintptr_t>(A.x) & 15) == 0, "gemm: int32 source must be 16-byte aligned");
        a.x = A.x; a.ldx = A.ldx; a.rowmax_in = A.rowmax; a.K = A.K;
        // staged by TMA: boxes of 128 rows x 32 int32 (128-byte rows, 128-byte swizzle), zeros past Mreal and K
        a.tmX = tmap2d(A.x, CU_TENSOR_MAP_DATA_TYPE_INT32, uint64_t(A.K), uint64_t(Mreal), uint64_t(A.ldx) * 4, 32, 128, Swz::B128);
        a.xtma = 1;
    } else if (src == VELA_SRC_CONV32) {
        VELA_REQUIRE(A.img && A.e && (A.C % 32 == 0 || A.C == 4) && A.K == 9 * A.C && A.K <= Kp && A.stride >= 1,
                     "gemm: conv source needs C % 32 == 0 or C == 4, K = 9C");
        VELA_REQUIRE(A.Ho == (A.H - 1) / A.stride + 1 && A.Wo == (A.W - 1) / A.stride + 1, "gemm: conv output size");
        VELA_REQUIRE((reinterpret_cast<uintptr_t>(A.img) & 15) == 0, "gemm: image must be 16-byte aligned");
        a.img = A.img; a.H = A.H; a.W = A.W; a.C = A.C; a.stride = A.stride; a.Ho = A.Ho; a.Wo = A.Wo; a.K = A.K; a.e = A.e;
        // Implicit im2col through TMA.  For tap (ky, kx) and 32 channels from c0, the 128 output pixels of a tile
        // read the NHWC box starting at (c0, kx - 1, oy0*s + ky - 1, b0) with element strides (1, s, s, 1); the
        // padding ring (coordinates -1 and past the edge) reads zeros.  Tiles must be whole output rows of one
        // image (Ho*Wo % 128 == 0 and 128 % Wo == 0) or whole images (128 % (Ho*Wo) == 0); other shapes keep
        // the per-thread loads, and so does the 4-channel input image (nine 16-byte pixels per row in one k-block).
        const int howo = A.Ho * A.Wo, s = A.stride;
        int bw = 0, bh = 0, bb = 0;
        if (howo % 128 == 0 && 128 % A.Wo == 0) { bw = A.Wo * s; bh = (128 / A.Wo) * s; bb = 1; }
        else if (128 % howo == 0) { bw = A.Wo * s; bh = A.Ho * s; bb = 128 / howo; }
        if (A.C % 32 == 0 && bw > 0 && bw <= 256 && bh <= 256 && s <= 8) {
            const int Bimg = ceil_div(Mreal, howo);
            a.tmX = tmap_nhwc(A.img, uint64_t(Bimg), uint64_t(A.H), uint64_t(A.W), uint64_t(A.C), 32, uint32_t(bw), uint32_t(bh), uint32_t(bb),
                              uint32_t(s), Swz::B128);
            a.xtma = 1; a.conv_rows_per_img = howo;
        }
    } else {
        throw Error(VELA_ERR_ARG, "gemm: unknown A source");
    }
    if (epi != EPI_PLAIN) VELA_REQUIRE(src == VELA_SRC_I8, "gemm: GEGLU / split3 / q|k|v epilogues take planar int8 operands");

    const bool splittable = epi == EPI_PLAIN && E.workspace && Nreal % 4 == 0 && E.ldy % 4 == 0;
    const Plan pl = plan(src, epi, Mp, Mreal, Np, Nreal, a.nkb, splittable ? E.workspace_bytes : 0, sm_count());
    const int BN = pl.bn;
    a.tmW = tmap2d(W, CU_TENSOR_MAP_DATA_TYPE_UINT8, uint64_t(Kp), uint64_t(Np), uint64_t(ldw), 64, uint32_t(BN), Swz::B64);
    a.kb_per_split = ceil_div(a.nkb, pl.splits);
    const int splits = ceil_div(a.nkb, a.kb_per_split);
    if (splits > 1) a.partial = static_cast<int32_t*>(E.workspace);
    // plain epilogue without split-K: Y leaves through per-warp shared-memory boxes and TMA stores
    if (epi == EPI_PLAIN && splits == 1 && E.Y && (E.ldy & 3) == 0 && (reinterpret_cast<uintptr_t>(E.Y) & 15) == 0) {
        a.tmY = tmap2d(E.Y, CU_TENSOR_MAP_DATA_TYPE_INT32, uint64_t(Nreal), uint64_t(Mreal), uint64_t(E.ldy) * 4, 16, 32, Swz::B64);
        a.ytma = 1;
    }

    if (epi == EPI_PLAIN) {
        if (src == VELA_SRC_I8) {
            if (BN == 256) launch_gemm_persist<256, 5, SRC_I8, EPI_PLAIN>(a, st);
            else if (BN == 160) launch_gemm_persist<160, 6, SRC_I8, EPI_PLAIN>(a, st);
            else if (BN == 128) launch_gemm_persist<128, 6, SRC_I8, EPI_PLAIN>(a, st);
            else launch_gemm_persist<64, 6, SRC_I8, EPI_PLAIN>(a, st);
        }
        else if (src == VELA_SRC_X32) dispatch_reg<SRC_X32>(BN, a, st);
        else dispatch_reg<SRC_CONV32>(BN, a, st);
    } else if (epi == EPI_GEGLU) launch_gemm_persist<128, 6, SRC_I8, EPI_GEGLU>(a, st);
    else if (epi == EPI_SPLIT3) launch_gemm_persist<128, 6, SRC_I8, EPI_SPLIT3>(a, st);
    else launch_gemm_persist<128, 6, SRC_I8, EPI_QKV>(a, st);
    if (splits > 1) {
        const size_t n = size_t(Mreal) * (Nreal / 4);
        gemm_splitk_reduce<<<unsigned((n + 255) / 256), 256, 0, st>>>(a.partial, splits, Mp, Np, Mreal, Nreal, a.cst, a.e, a.rowmax_in, src == VELA_SRC_X32,
                                                                     E.Y, E.ldy, E.residual, E.epi == VELA_EPI_GELU, E.Lphi, E.rowmax);
        VELA_CUDA(cudaGetLastError());
    }
}

// conv_e: e[row] = row_exp(max of the pixel maxima over the 3x3 window) (src/gemm_hl.cu:335-341)
__global__ void conv_e_kernel(const uint32_t* __restrict__ pm, int B, int H, int W, int stride, int Ho, int Wo, int32_t* __restrict__ e) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= B * Ho * Wo) return;
    const int hw = Ho * Wo, b = r / hw, p = r - b * hw, oy = p / Wo, ox = p - oy * Wo;
    u32 m = 0;
    #pragma unroll
    for (int ky = 0; ky < 3; ++ky)
        #pragma unroll
        for (int kx = 0; kx < 3; ++kx) {
            const int iy = oy * stride - 1 + ky, ix = ox * stride - 1 + kx;
            if (iy >= 0 && iy < H && ix >= 0 && ix < W) m = max(m, __ldg(pm + (size_t(b) * H + iy) * W + ix));
        }
    e[r] = row_exp(m);
}
void conv_e(cudaStream_t st, const uint32_t* pm, int B, int H, int W, int stride, int32_t* e) {
    VELA_REQUIRE(pm && e && B > 0 && H > 0 && W > 0 && stride >= 1, "conv_e: bad arguments");
    const int Ho = (H - 1) / stride + 1, Wo = (W - 1) / stride + 1, rows = B * Ho * Wo;
    conv_e_kernel<<<ceil_div(rows, 256), 256, 0, st>>>(pm, B, H, W, stride, Ho, Wo, e);
}
}  // namespace vela

using namespace vela;

extern "C" int vela_gemm_w8a16(void* stream, const vela_asrc* A, int Mp, int Mreal, const int8_t* W, int ldw, int Np, int Nreal, int Kp,
                               const int32_t* cst, const vela_aepi* E) {
    return guarded("vela_gemm_w8a16", [&] {
        VELA_REQUIRE(A && E, "null descriptor");
        gemm_w8a16(static_cast<cudaStream_t>(stream), *A, Mp, Mreal, W, ldw, Np, Nreal, Kp, cst, *E);
    });
}
// Failure-path test of the bounded waits: the same launch with the TMA producers idle and a wait limit of
// wait_limit_cycles, so every consumer's wait runs out, the kernel drains and returns and the timeout is reported in
// the device error word (vela_device_error).  Nothing is in flight when the waits give up.
extern "C" int vela_gemm_w8a16_stalled(void* stream, const vela_asrc* A, int Mp, int Mreal, const int8_t* W, int ldw, int Np, int Nreal, int Kp,
                                       const int32_t* cst, const vela_aepi* E, long long wait_limit_cycles) {
    return guarded("vela_gemm_w8a16_stalled", [&] {
        VELA_REQUIRE(A && E && wait_limit_cycles > 0, "null descriptor or non-positive wait limit");
        LaunchOpts o; o.wait_limit = wait_limit_cycles; o.stall = 1;
        gemm_w8a16(static_cast<cudaStream_t>(stream), *A, Mp, Mreal, W, ldw, Np, Nreal, Kp, cst, *E, o);
    });
}
extern "C" int vela_gemm_hl(void* stream, const int8_t* Ahi, const int8_t* Alo, int lda, int Mp, int Mreal, const int8_t* W, int ldw, int Np, int Nreal, int Kp,
                            const int32_t* cst, const int32_t* e, int32_t* Y, int ldy, const int32_t* residual, int epi, int Cs, int32_t* Y1, int32_t* Y2,
                            const int32_t* Lphi) {
    return guarded("vela_gemm_hl", [&] {
        vela_asrc A; std::memset(&A, 0, sizeof(A));
        A.src = VELA_SRC_I8; A.hi = Ahi; A.lo = Alo; A.ld8 = lda; A.e = e;
        vela_aepi E; std::memset(&E, 0, sizeof(E));
        E.epi = epi; E.Y = Y; E.ldy = ldy; E.residual = residual; E.Cs = Cs; E.Y1 = Y1; E.Y2 = Y2; E.Lphi = Lphi;
        gemm_w8a16(static_cast<cudaStream_t>(stream), A, Mp, Mreal, W, ldw, Np, Nreal, Kp, cst, E);
    });
}
extern "C" int vela_conv_e(void* stream, const uint32_t* pm, int B, int H, int W, int stride, int32_t* e) {
    return guarded("vela_conv_e", [&] { conv_e(static_cast<cudaStream_t>(stream), pm, B, H, W, stride, e); });
}
extern "C" unsigned vela_device_error(int clear) {
    try { return read_device_errors(clear != 0); } catch (...) { return 0xFFFFFFFFu; }
}
