// Memory-bound integer kernels of the UNet step and their C-ABI entry points:
// row quantisation, pixel max, explicit im2col, GroupNorm (stats + apply),
// LayerNorm, LUT activations, concat / upsample, ChaCha20 noise, finalize,
// text embedding and the attention operand quantisers.  Semantics follow the
// reference's src/kernels.cu (cited per kernel); the layouts are B200-first:
// int4 (16-byte) coalesced loads and stores, warp-per-row reductions held in
// registers, per-channel accumulation instead of per-element atomics.
#include "intops.cuh"
#include "host_util.h"
#include "vela_b200.h"
#include <algorithm>
#include <climits>
#include <cstring>

namespace vela {
namespace {

__device__ __forceinline__ i64 warp_sum64(i64 v) { for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o); return v; }
__device__ __forceinline__ int warp_min(int v) { for (int o = 16; o; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o)); return v; }
__device__ __forceinline__ int warp_max(int v) { for (int o = 16; o; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o)); return v; }
__device__ __forceinline__ u32 warp_umax(u32 v) { for (int o = 16; o; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o)); return v; }

// floor(a / d) for d >= 1 and |a| < 2^63 with inv = floor((2^64 - 1) / d):
// q0 = floor(|a| * inv / 2^64) is floor(|a| / d) or one less, one correction step fixes it;
// a negative numerator uses floor(-x/d) = -floor(x/d) - [x mod d != 0].
__device__ __forceinline__ i64 floor_div_inv(i64 a, uint64_t d, uint64_t inv) {
    const uint64_t m = a < 0 ? uint64_t(0) - uint64_t(a) : uint64_t(a);
    uint64_t q = __umul64hi(m, inv);
    uint64_t r = m - q * d;
    if (r >= d) { ++q; r -= d; }
    if (a >= 0) return i64(q);
    return r ? -i64(q) - 1 : -i64(q);
}

// 16 quantised values of one row written as hi / lo bytes at column c (c % 4 == 0)
__device__ __forceinline__ void store_q4(int8_t* hi, int8_t* lo, int c, int q0, int q1, int q2, int q3) {
    *reinterpret_cast<u32*>(hi + c) = pack_hi4(q0, q1, q2, q3);
    *reinterpret_cast<u32*>(lo + c) = pack_lo4(q0, q1, q2, q3);
}
// pad columns [C, Kp) of a quantised row with the value 0 = (hi 0, lo -128)
__device__ __forceinline__ void pad_cols(int8_t* hi, int8_t* lo, int C, int Kp, int lane) {
    for (int c = C + lane; c < Kp; c += 32) { hi[c] = 0; lo[c] = -128; }
}

// ---------------------------------------------------------------- row quantisation (src/kernels.cu:42-57,488-497)
// one warp per row; rows [M, Mpad) become value 0
__global__ void quant_rows_kernel(const int32_t* __restrict__ X, int M, int Mpad, int K, int ldx, int8_t* __restrict__ hi, int8_t* __restrict__ lo,
                                  int32_t* __restrict__ e, int Kp) {
    const int lane = threadIdx.x & 31;
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= Mpad) return;
    int8_t* h = hi + size_t(r) * Kp; int8_t* l = lo + size_t(r) * Kp;
    if (r >= M) { for (int k = lane; k < Kp; k += 32) { h[k] = 0; l[k] = -128; } return; }
    const int32_t* x = X + size_t(r) * ldx;
    const bool vec = ((K | ldx) & 3) == 0;
    u32 m = 0;
    if (vec) { for (int c = lane * 4; c < K; c += 128) { const int4 v = __ldg(reinterpret_cast<const int4*>(x + c)); m = max(m, max(max(uabs(v.x), uabs(v.y)), max(uabs(v.z), uabs(v.w)))); } }
    else { for (int c = lane; c < K; c += 32) m = max(m, uabs(__ldg(x + c))); }
    const int ee = row_exp(warp_umax(m));
    if (lane == 0) e[r] = ee;
    if (vec) {
        for (int c = lane * 4; c < K; c += 128) { const int4 v = __ldg(reinterpret_cast<const int4*>(x + c)); store_q4(h, l, c, quant16(v.x, ee), quant16(v.y, ee), quant16(v.z, ee), quant16(v.w, ee)); }
    } else {
        for (int c = lane; c < K; c += 32) { const int q = quant16(__ldg(x + c), ee); h[c] = int8_t(q >> 8); l[c] = int8_t((q & 255) - 128); }
    }
    pad_cols(h, l, K, Kp, lane);
}

// Row quantisation with the row maxima already known (the producing epilogue's row max): one read of X.
// One warp per row (grid-stride), four columns per lane and step: the quantised quad is formed with the packed
// saturating narrowing of quant_pack4 (the two-operation rounding for exponents up to 15) and stored as one
// 32-bit word of hi bytes and one of lo bytes; K % 4 == 0, columns [K, Kp) and rows [M, Mpad) become value 0.
__global__ void quant_rows_rm_kernel(const int32_t* __restrict__ X, const u32* __restrict__ rowmax, int M, int Mpad, int K, int ldx,
                                     int8_t* __restrict__ hi, int8_t* __restrict__ lo, int32_t* __restrict__ e, int Kp) {
    const int lane = threadIdx.x & 31, wpb = blockDim.x >> 5;
    for (int r = blockIdx.x * wpb + (threadIdx.x >> 5); r < Mpad; r += gridDim.x * wpb) {
        u32* h = reinterpret_cast<u32*>(hi + size_t(r) * Kp);
        u32* l = reinterpret_cast<u32*>(lo + size_t(r) * Kp);
        const int ee = r < M ? row_exp(__ldg(rowmax + r)) : 0;
        if (lane == 0) e[r] = ee;
        const int kq = r < M ? (K >> 2) : 0;
        const int qs1 = ee > 0 ? ee - 1 : 0, qr = ee > 0 ? 1 : 0, qs2 = qr, qh = (1 << ee) >> 1;
        const int32_t* x = X + size_t(r) * ldx;
        for (int c4 = lane; c4 < (Kp >> 2); c4 += 32) {
            uint32_t hw = 0u, lw = 0x80808080u;
            if (c4 < kq) {
                const int4 v = __ldg(reinterpret_cast<const int4*>(x) + c4);
                if (ee <= 15) quant_pack4_e15(v.x, v.y, v.z, v.w, qh, ee, hw, lw);
                else quant_pack4(v.x, v.y, v.z, v.w, qs1, qr, qs2, hw, lw);
            }
            h[c4] = hw; l[c4] = lw;
        }
    }
}

// ---------------------------------------------------------------- pixel max (src/kernels.cu:106-115)
__global__ void pixmax_kernel(const int32_t* __restrict__ X, int rows, int C, u32* __restrict__ pm) {
    const int lane = threadIdx.x & 31, r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= rows) return;
    const int32_t* x = X + size_t(r) * C;
    u32 m = 0;
    if ((C & 3) == 0) { for (int c = lane * 4; c < C; c += 128) { const int4 v = __ldg(reinterpret_cast<const int4*>(x + c)); m = max(m, max(max(uabs(v.x), uabs(v.y)), max(uabs(v.z), uabs(v.w)))); } }
    else { for (int c = lane; c < C; c += 32) m = max(m, uabs(__ldg(x + c))); }
    m = warp_umax(m);
    if (lane == 0) pm[r] = m;
}

// ---------------------------------------------------------------- explicit 3x3 im2col (src/kernels.cu:117-170)
// one warp per output row, K index tap*C + c; rows [rows, Mpad) value 0
__global__ void im2col3_kernel(const int32_t* __restrict__ X, const u32* __restrict__ pm, int B, int H, int W, int C, int stride, int Ho, int Wo,
                               int rows, int Mpad, int8_t* __restrict__ hi, int8_t* __restrict__ lo, int32_t* __restrict__ e, int Kp) {
    const int lane = threadIdx.x & 31, r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= Mpad) return;
    int8_t* h = hi + size_t(r) * Kp; int8_t* l = lo + size_t(r) * Kp;
    if (r >= rows) { for (int k = lane; k < Kp; k += 32) { h[k] = 0; l[k] = -128; } return; }
    const int hw = Ho * Wo, b = r / hw, p = r - b * hw, oy = p / Wo, ox = p - oy * Wo;
    u32 m = 0;
    for (int t = 0; t < 9; ++t) {
        const int iy = oy * stride - 1 + t / 3, ix = ox * stride - 1 + t % 3;
        if (iy >= 0 && iy < H && ix >= 0 && ix < W) m = max(m, __ldg(pm + (size_t(b) * H + iy) * W + ix));
    }
    const int ee = row_exp(m);
    if (lane == 0) e[r] = ee;
    const int K = 9 * C;
    for (int k = lane; k < K; k += 32) {
        const int tap = k / C, c = k - tap * C, iy = oy * stride - 1 + tap / 3, ix = ox * stride - 1 + tap % 3;
        const int q = (iy >= 0 && iy < H && ix >= 0 && ix < W) ? quant16(__ldg(X + ((size_t(b) * H + iy) * W + ix) * C + c), ee) : 0;
        h[k] = int8_t(q >> 8); l[k] = int8_t((q & 255) - 128);
    }
    pad_cols(h, l, K, Kp, lane);
}

// One tap of one im2col row: its C / 4 16-byte groups quantised with the row's exponent into four hi and four lo
// bytes each.  Full-warp steps (two loads in flight) carry no predicate, the last partial step one; a tap on the
// padding (warp-uniform) writes the zero value (hi 0, lo 0x80).
// Q: 0 = exponent <= 15 and no saturation possible (quant_nosat), 1 = exponent <= 15, 2 = any exponent.
template <int Q>
__device__ __forceinline__ void im2col_tap(const int4* __restrict__ x, bool in, u32* __restrict__ hp, u32* __restrict__ lp, int q4, int lane,
                                           int qa, int qb) {
    auto put = [&](const int4& v, int c) {
        uint32_t hv, lv;
        if constexpr (Q == 0) quant_pack4_e15_nosat(v.x, v.y, v.z, v.w, qa, qb, hv, lv);
        else if constexpr (Q == 1) quant_pack4_e15(v.x, v.y, v.z, v.w, qa, qb, hv, lv);
        else quant_pack4(v.x, v.y, v.z, v.w, qa, qb, qb, hv, lv);
        hp[c] = hv; lp[c] = lv;
    };
    if (!in) {
        for (int c = lane; c < q4; c += 32) { hp[c] = 0u; lp[c] = 0x80808080u; }
        return;
    }
    const int nfull = q4 >> 5;
    int c = lane;
    for (int j = 0; j + 2 <= nfull; j += 2, c += 64) {
        const int4 v0 = __ldg(x + c), v1 = __ldg(x + c + 32);
        put(v0, c); put(v1, c + 32);
    }
    if (nfull & 1) { put(__ldg(x + c), c); c += 32; }
    if (c < q4) put(__ldg(x + c), c);
}

// The same for C % 4 == 0 and Kp % 4 == 0.  ALL_TAPS: one warp per output row, the nine taps in turn (large images:
// the row's setup and window exponent are paid once); else one warp per (row, tap) (small images: nine times the
// warps to fill the SMs).  The window exponent comes from the nine pixel maxima (a warp max), written by the warp of
// tap 0; the warp of tap 8 fills the K padding [9C, Kp).  The quantisation form is chosen once per row: without the
// saturation when the window maximum rules it out (quant_nosat), the common case.
template <bool ALL_TAPS>
__global__ void im2col3_q4_kernel(const int32_t* __restrict__ X, const u32* __restrict__ pm, int B, int H, int W, int C, int stride, int Ho,
                                  int Wo, int rows, int Mpad, int8_t* __restrict__ hi, int8_t* __restrict__ lo, int32_t* __restrict__ e, int Kp) {
    const int lane = threadIdx.x & 31, wg = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int r = ALL_TAPS ? wg : wg / 9, t0 = ALL_TAPS ? 0 : wg - r * 9, t1 = ALL_TAPS ? 9 : t0 + 1;
    if (r >= Mpad) return;
    u32* h = reinterpret_cast<u32*>(hi + size_t(r) * Kp);
    u32* l = reinterpret_cast<u32*>(lo + size_t(r) * Kp);
    const int q4 = C >> 2, kq = 9 * q4;
    if (r >= rows) {
        for (int c4 = t0 * q4 + lane; c4 < (t1 == 9 ? (Kp >> 2) : t1 * q4); c4 += 32) { h[c4] = 0u; l[c4] = 0x80808080u; }
        return;
    }
    const int hw = Ho * Wo, b = r / hw, p = r - b * hw, oy = p / Wo, ox = p - oy * Wo;
    const int4* img = reinterpret_cast<const int4*>(X + size_t(b) * H * W * C);
    u32 m = 0;
    if (lane < 9) {
        const int py = oy * stride - 1 + lane / 3, px = ox * stride - 1 + lane % 3;
        if (py >= 0 && py < H && px >= 0 && px < W) m = __ldg(pm + (size_t(b) * H + py) * W + px);
    }
    const u32 wm = __reduce_max_sync(0xffffffffu, m);
    const int ee = row_exp(wm);
    if (t0 == 0 && lane == 0) e[r] = ee;
    const int qf = ee > 15 ? 2 : (quant_nosat(wm, ee) ? 0 : 1);       // warp-uniform
    for (int t = t0; t < t1; ++t) {
        const int iy = oy * stride - 1 + t / 3, ix = ox * stride - 1 + t % 3;
        const bool in = iy >= 0 && iy < H && ix >= 0 && ix < W;
        const int4* x = img + (size_t(in ? iy : 0) * W + (in ? ix : 0)) * q4;
        if (qf == 0) im2col_tap<0>(x, in, h + t * q4, l + t * q4, q4, lane, (1 << ee) >> 1, ee);
        else if (qf == 1) im2col_tap<1>(x, in, h + t * q4, l + t * q4, q4, lane, (1 << ee) >> 1, ee);
        else im2col_tap<2>(x, in, h + t * q4, l + t * q4, q4, lane, ee - 1, 1);
    }
    if (t1 == 9)
        for (int c4 = kq + lane; c4 < (Kp >> 2); c4 += 32) { h[c4] = 0u; l[c4] = 0x80808080u; }
}

// ---------------------------------------------------------------- GroupNorm (src/kernels.cu:173-221,285-305,420-487)
// Per-(sample, group) accumulation record = vela_gnstat {sum, mn, mx, mean, e, ss, sd}: zeroed, then the two
// statistics passes accumulate into it with atomics, then the finish kernel derives mean, e and sd.
__global__ void gn_init_kernel(vela_gnstat* gs, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) { gs[i].sum = 0; gs[i].mn = INT_MAX; gs[i].mx = INT_MIN; gs[i].mean = 0; gs[i].e = 0; gs[i].pad_ = 0; gs[i].ss = 0; gs[i].sd = 0; }
}
// mean and exponent of one group, src/kernels.cu:185-191
__device__ __forceinline__ void gn_mean_e(const vela_gnstat& s, i64 n, i64& mean, int& e) {
    mean = floor_div(s.sum + n / 2, n);
    const i64 m = max(i64(s.mx) - mean, mean - i64(s.mn));
    e = max(0, (m >= (i64(1) << 32) ? 17 : row_exp(u32(m))) - 5);
}
// mean, e, ss -> var, eps, sd (src/kernels.cu:204-211)
__device__ __forceinline__ void gn_finish_one(vela_gnstat* g, i64 n, i64 den) {
    vela_gnstat s = *g;
    i64 mean; int e; gn_mean_e(s, n, mean, e);
    s.mean = mean; s.e = e; s.pad_ = 0;
    const i64 var = floor_div(s.ss, n);
    const int sh = 32 - 2 * e; const i64 one = sh >= 0 ? (i64(1) << sh) : 0;
    const i64 eps = floor_div(one + den / 2, den);
    s.sd = isqrt((var + eps) << 16);
    *g = s;
}
// Statistics passes.  Block = Q x RP threads (Q = C / 4 column quads, RP row lanes); a thread keeps one quad
// (four channels, fixed groups) over every RP-th row of the block's rows, four rows in flight, then the block
// combines per group in shared memory and adds to the (sample, group) record once.
// Pass 2 also finishes the records: every block counts itself in gs[0].pad_ (zeroed by gn_init) after its
// atomics, and the block that counts last (no block waits for another) derives mean, e and sd of all B x 32
// records and clears the counter.
template <int PASS>
__global__ void __launch_bounds__(1024) gn_stats_kernel(const int32_t* __restrict__ X, int T, int C, int rowsPerBlock, vela_gnstat* gs,
                                                        int cnt, i64 den) {
    __shared__ long long sacc[32]; __shared__ int smn[32], smx[32]; __shared__ long long smean[32]; __shared__ int se[32];
    __shared__ bool sfast[32];
    const int Q = C >> 2, RP = blockDim.x / Q, cg = C >> 5;
    const int b = blockIdx.y, t0 = blockIdx.x * rowsPerBlock, t1 = min(T, t0 + rowsPerBlock);
    if (threadIdx.x < 32) {
        sacc[threadIdx.x] = 0; smn[threadIdx.x] = INT_MAX; smx[threadIdx.x] = INT_MIN;
        if (PASS == 2) {
            const vela_gnstat g = gs[b * 32 + threadIdx.x];
            i64 mean; int e; gn_mean_e(g, i64(T) * cg, mean, e); smean[threadIdx.x] = mean; se[threadIdx.x] = e;
            sfast[threadIdx.x] = max(i64(g.mx) - mean, mean - i64(g.mn)) < (i64(1) << 30);
        }
    }
    __syncthreads();
    const int c4 = threadIdx.x % Q, rr = threadIdx.x / Q;
    if (rr < RP) {
        const int c = c4 * 4;
        int gi[4]; i64 mean[4] = {0, 0, 0, 0}; int e[4] = {0, 0, 0, 0};
        #pragma unroll
        for (int k = 0; k < 4; ++k) { gi[k] = (c + k) / cg; if (PASS == 2) { mean[k] = smean[gi[k]]; e[k] = se[gi[k]]; } }
        // pass 2 with every deviation below 2^30 in magnitude (the groups' ranges, checked in the prologue): the
        // rounded deviation (d + 2^(e-1)) >> e and its square accumulate in 32 / 64 bits without 64-bit shifts
        bool small = PASS == 2;
        int mean32[4], half[4];
        #pragma unroll
        for (int k = 0; k < 4; ++k) { small = small && sfast[gi[k]]; mean32[k] = int(mean[k]); half[k] = e[k] ? 1 << (e[k] - 1) : 0; }
        i64 acc[4] = {0, 0, 0, 0}; int mn[4] = {INT_MAX, INT_MAX, INT_MAX, INT_MAX}, mx[4] = {INT_MIN, INT_MIN, INT_MIN, INT_MIN};
        const int32_t* x = X + (size_t(b) * T) * C + c;
        auto take = [&](const int4 v) {
            const int vv[4] = {v.x, v.y, v.z, v.w};
            #pragma unroll
            for (int k = 0; k < 4; ++k) {
                if (PASS == 1) { acc[k] += vv[k]; mn[k] = min(mn[k], vv[k]); mx[k] = max(mx[k], vv[k]); }
                else if (small) { const int dd = (vv[k] - mean32[k] + half[k]) >> e[k]; acc[k] += i64(dd) * dd; }
                else { const i64 d = i64(vv[k]) - mean[k]; const i64 dd = e[k] ? ((d >> e[k]) + ((d >> (e[k] - 1)) & 1)) : d; acc[k] += dd * dd; }
            }
        };
        int t = t0 + rr;
        for (; t + 3 * RP < t1; t += 4 * RP) {
            const int4 v0 = __ldg(reinterpret_cast<const int4*>(x + size_t(t) * C));
            const int4 v1 = __ldg(reinterpret_cast<const int4*>(x + size_t(t + RP) * C));
            const int4 v2 = __ldg(reinterpret_cast<const int4*>(x + size_t(t + 2 * RP) * C));
            const int4 v3 = __ldg(reinterpret_cast<const int4*>(x + size_t(t + 3 * RP) * C));
            take(v0); take(v1); take(v2); take(v3);
        }
        for (; t < t1; t += RP) take(__ldg(reinterpret_cast<const int4*>(x + size_t(t) * C)));
        // channels of one group within the quad first (groups of >= 4 channels: at most two groups per quad)
        #pragma unroll
        for (int k = 0; k < 4; ++k) {
            if (k > 0 && gi[k] == gi[k - 1]) continue;
            i64 a = acc[k]; int lo = mn[k], hi = mx[k];
            #pragma unroll
            for (int k2 = k + 1; k2 < 4; ++k2) if (gi[k2] == gi[k]) { a += acc[k2]; lo = min(lo, mn[k2]); hi = max(hi, mx[k2]); }
            atomicAdd(reinterpret_cast<unsigned long long*>(&sacc[gi[k]]), (unsigned long long)a);
            if (PASS == 1) { atomicMin(&smn[gi[k]], lo); atomicMax(&smx[gi[k]], hi); }
        }
    }
    __syncthreads();
    if (threadIdx.x < 32 && t1 > t0) {
        vela_gnstat* st = gs + b * 32 + threadIdx.x;
        if (PASS == 1) {
            atomicAdd(reinterpret_cast<unsigned long long*>(&st->sum), (unsigned long long)sacc[threadIdx.x]);
            atomicMin(&st->mn, smn[threadIdx.x]); atomicMax(&st->mx, smx[threadIdx.x]);
        } else {
            atomicAdd(reinterpret_cast<unsigned long long*>(&st->ss), (unsigned long long)sacc[threadIdx.x]);
        }
    }
    if constexpr (PASS == 2) {
        __shared__ bool s_last;
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) {
            const unsigned done = atomicAdd(reinterpret_cast<unsigned*>(&gs[0].pad_), 1u);
            s_last = done == gridDim.x * gridDim.y - 1;
        }
        __syncthreads();
        if (s_last) {
            __threadfence();
            const i64 n = i64(T) * cg;
            for (int i = threadIdx.x; i < cnt; i += blockDim.x) gn_finish_one(gs + i, n, den);
        }
    }
}

// Normalisation constants of one (sample, group) or one row, for the exact binary64 division of norm_val.
// c = 1.5 * 2^52 + mean (exact: |mean| < 2^31), scale = 2^(25-e), D = 2 sd, rcp = 1 / D rounded.
constexpr double MAGIC52 = 6755399441055744.0;   // 1.5 * 2^52: integers k with |k| < 2^51 sit in its low mantissa bits
struct NormP { double c, scale, sd, D, rcp; };
__device__ __forceinline__ NormP norm_params(i64 mean, int e, i64 sd) {
    NormP p;
    p.c = MAGIC52 + double(mean); p.scale = double(i64(1) << (25 - e)); p.sd = double(sd); p.D = 2.0 * double(sd); p.rcp = 1.0 / p.D;
    return p;
}
// normalise one value: sat32(sat32(rshr(floor((d * 2^(25-e) + sd) / (2 sd)) * g, 16)) + beta), d = x - mean.
// The quotient is formed in binary64, where every intermediate is an integer below 2^53: |d| <= the group's
// range m < 2^(20+e) (2^33 when e = 12), so |d 2^(25-e)| < 2^46.  No conversion instruction is needed: the bits
// of 1.5*2^52 + x are x in the low word and 0x43380000 (minus the sign) in the high word, so x - mean is one
// exact subtraction of c; the quotient is rounded to an integer by adding 1.5*2^52 in the same fma, which puts
// it in the low word of the sum.  That rounding of num * rcp (within 2^-28 of num / D) is the floor or the floor
// plus one, and one exact residual test (fma) settles it.  sd >= 1 always (sd = 0 would need var + eps = 0,
// impossible: a constant group has e = 0 and eps > 0), and the quotient fits 32 bits: sd = isqrt((var + eps) << 16)
// of the group's (row's) own deviations keeps |d| 2^(24-e) / sd near 2^16 sqrt(n) at most (n <= 2^20 values).
__device__ __forceinline__ int norm_val(int x, const NormP& p, int g, int beta) {
    const double xb = __hiloint2double(0x43380000 + (x >> 31), x);     // 1.5 * 2^52 + x
    const double num = fma(xb - p.c, p.scale, p.sd);
    const double t = fma(num, p.rcp, MAGIC52);
    int q = __double2loint(t);
    const double r = fma(-(t - MAGIC52), p.D, num);
    q += int(r >= p.D) - int(r < 0.0);
    const i64 u = i64(q) * g + 32768;
    const int lo = int(__funnelshift_r(uint32_t(u), uint32_t(u >> 32), 16));
    return add_sat((int(u >> 32) >> 16) == (lo >> 31) ? lo : (u < 0 ? INT_MIN : INT_MAX), beta);
}
// SiLU: sat32(rshr(x lut16(x), 16)), lut16 from the sentinel table staged in shared memory (lut16_s); without the
// saturation when every table entry lies in [0, 65536] (then |result| <= |x|)
__device__ __forceinline__ int silu_s(int x, const int2* __restrict__ T, bool in_range) { return in_range ? lut_act_s(x, T) : lut_act_s_sat(x, T); }
// Apply.  Block = PT x RP threads over rowsPerBlock consecutive rows, GN_RPT rows per thread: a thread owns the
// channel pairs pr, pr + PT, ... (int2; PT = min(C/2, 512)); the pair's group constants (one group unless C/32
// is odd and the pair straddles two) of the samples the block touches (at most GN_SPAN) are staged in shared
// memory, the SiLU table as (L[i], L[i+1] - L[i]); the pixel max of each row is combined with shared-memory
// atomics.  QUANT: the normalised rows are kept in shared memory (dynamic, rowsPerBlock x C int32) until their
// maxima give the exponents, then hi / lo planes are written.
constexpr int GN_RPT = 8, GN_SPAN = 4;
template <bool QUANT>
__global__ void __launch_bounds__(512) gn_apply_kernel(const int32_t* __restrict__ X, int M, int T, int C, const vela_gnstat* __restrict__ gs,
                                                       const int32_t* __restrict__ g, const int32_t* __restrict__ beta, const int32_t* __restrict__ Lsig,
                                                       int32_t* __restrict__ Y, u32* __restrict__ pm, int8_t* __restrict__ hi, int8_t* __restrict__ lo,
                                                       int32_t* __restrict__ e, int Kp, int rowsPerBlock) {
    __shared__ int2 s_lut[LUT_S_ENTRIES];
    __shared__ NormP s_p[GN_SPAN][32];
    __shared__ u32 s_rmax[256];
    extern __shared__ int32_t s_rows[];            // QUANT: [rowsPerBlock][C]
    const int P2 = C >> 1, PT = min(P2, 512), RP = blockDim.x / PT, cg = C >> 5;
    const bool lut_in_range = __syncthreads_and(Lsig ? stage_lut_s(s_lut, Lsig) : 1);
    const int rr = threadIdx.x / PT;
    // PT % 32 == 0 (C % 64 == 0, every UNet width): a warp's lanes share the row, so its row max is reduced first
    const bool warp_rows = (PT & 31) == 0;
    const int nchunks = (M + rowsPerBlock - 1) / rowsPerBlock;
    // the block walks row chunks (the table above is staged once per block)
    for (int chunk = blockIdx.x; chunk < nchunks; chunk += gridDim.x) {
        const int r0 = chunk * rowsPerBlock, r1 = min(M, r0 + rowsPerBlock), b0 = r0 / T;
        for (int i = threadIdx.x; i < rowsPerBlock; i += blockDim.x) s_rmax[i] = 0;
        for (int i = threadIdx.x; i < GN_SPAN * 32; i += blockDim.x) {
            const int sb = b0 + (i >> 5);
            if (sb * T < r1) { const vela_gnstat st = gs[sb * 32 + (i & 31)]; s_p[i >> 5][i & 31] = norm_params(st.mean, st.e, st.sd); }
        }
        __syncthreads();
        if (rr < RP) {
            for (int pr = threadIdx.x % PT; pr < P2; pr += PT) {
                const int c = 2 * pr, g0 = c / cg, g1 = (c + 1) / cg;
                const int2 gv = __ldg(reinterpret_cast<const int2*>(g + c)), bv = __ldg(reinterpret_cast<const int2*>(beta + c));
                int cur = -1;
                NormP p0, p1;
                #pragma unroll 4
                for (int i = 0; i < GN_RPT; ++i) {
                    const int r = r0 + rr + i * RP;
                    if (r >= r1) break;
                    int sl = 0;                                 // sample slot of row r (the chunk spans at most GN_SPAN)
                    #pragma unroll
                    for (int k = 1; k < GN_SPAN; ++k) sl += r >= (b0 + k) * T;
                    if (sl != cur) { p0 = s_p[sl][g0]; p1 = s_p[sl][g1]; cur = sl; }
                    const int2 xv = __ldg(reinterpret_cast<const int2*>(X + size_t(r) * C + c));
                    int v0 = norm_val(xv.x, p0, gv.x, bv.x), v1 = norm_val(xv.y, p1, gv.y, bv.y);
                    if (Lsig) { v0 = silu_s(v0, s_lut, lut_in_range); v1 = silu_s(v1, s_lut, lut_in_range); }
                    if constexpr (QUANT) *reinterpret_cast<int2*>(s_rows + (r - r0) * C + c) = make_int2(v0, v1);
                    else *reinterpret_cast<int2*>(Y + size_t(r) * C + c) = make_int2(v0, v1);
                    u32 m = max(uabs(v0), uabs(v1));
                    if (warp_rows) { m = __reduce_max_sync(0xffffffffu, m); if ((threadIdx.x & 31) == 0 && m) atomicMax(&s_rmax[r - r0], m); }
                    else if (m) atomicMax(&s_rmax[r - r0], m);
                }
            }
        }
        __syncthreads();
        if constexpr (!QUANT) {
            for (int i = threadIdx.x; i < r1 - r0; i += blockDim.x) pm[r0 + i] = s_rmax[i];
        } else {
            for (int i = threadIdx.x; i < r1 - r0; i += blockDim.x) e[r0 + i] = row_exp(s_rmax[i]);
            // planes: one thread per 4 columns of a row, value 0 = (hi 0, lo -128) in the padding columns [C, Kp)
            const int K4 = Kp >> 2;
            for (int i = threadIdx.x; i < (r1 - r0) * K4; i += blockDim.x) {
                const int rl = i / K4, c = (i - rl * K4) * 4;
                const int ee = row_exp(s_rmax[rl]);
                int v[4];
                #pragma unroll
                for (int k = 0; k < 4; ++k) v[k] = c + k < C ? s_rows[rl * C + c + k] : 0;
                uint32_t hw, lw;
                quant_pack4(v[0], v[1], v[2], v[3], ee > 0 ? ee - 1 : 0, ee > 0 ? 1 : 0, ee > 0 ? 1 : 0, hw, lw);
                *reinterpret_cast<u32*>(hi + size_t(r0 + rl) * Kp + c) = hw;
                *reinterpret_cast<u32*>(lo + size_t(r0 + rl) * Kp + c) = lw;
            }
        }
        __syncthreads();      // s_rmax, s_p and s_rows are reused by the next chunk
    }
}

// ---------------------------------------------------------------- LayerNorm (src/kernels.cu:223-284,350-419)
// one warp per row, the row held in registers (C <= 128 * R4, C % 4 == 0)
// Per-launch constants of the row statistics: floor((2^64 - 1) / d) for the exact divisions by d = C and d = den.
struct LnConst { uint64_t inv_n; i64 den; uint64_t inv_den; };
template <int R4, bool QUANT, typename GT>
__global__ void lnorm_kernel(const int32_t* __restrict__ X, int M, int C, const GT* __restrict__ g, const GT* __restrict__ beta, const LnConst k,
                             int8_t* __restrict__ hi, int8_t* __restrict__ lo, int32_t* __restrict__ e, int Kp, int32_t* __restrict__ Y) {
    const int lane = threadIdx.x & 31, r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= M) return;
    const int C4 = C >> 2;
    const int32_t* x = X + size_t(r) * C;
    int v[4 * R4];
    i64 sum = 0; int mn = INT_MAX, mx = INT_MIN;
    #pragma unroll
    for (int j = 0; j < R4; ++j) {
        const int c4 = lane + 32 * j;
        int4 t = make_int4(0, 0, 0, 0);
        if (c4 < C4) {
            t = __ldg(reinterpret_cast<const int4*>(x + c4 * 4));
            sum += i64(t.x) + t.y + t.z + t.w;
            mn = min(mn, min(min(t.x, t.y), min(t.z, t.w))); mx = max(mx, max(max(t.x, t.y), max(t.z, t.w)));
        }
        v[4 * j] = t.x; v[4 * j + 1] = t.y; v[4 * j + 2] = t.z; v[4 * j + 3] = t.w;
    }
    sum = warp_sum64(sum); mn = warp_min(mn); mx = warp_max(mx);
    const i64 n = C, mean = floor_div_inv(sum + n / 2, uint64_t(n), k.inv_n);
    const i64 rng = max(i64(mx) - mean, mean - i64(mn));
    const int ex = max(0, (rng >= (i64(1) << 32) ? 17 : row_exp(u32(rng))) - 5);
    i64 ss = 0;
    if (rng < (i64(1) << 30)) {            // every deviation below 2^30: rounded shift and square in 32 / 64 bits
        const int m32 = int(mean), h = ex ? 1 << (ex - 1) : 0;
        #pragma unroll
        for (int j = 0; j < R4; ++j) {
            if (lane + 32 * j >= C4) break;
            #pragma unroll
            for (int k = 0; k < 4; ++k) { const int dd = (v[4 * j + k] - m32 + h) >> ex; ss += i64(dd) * dd; }
        }
    } else {
        #pragma unroll
        for (int j = 0; j < R4; ++j) {
            if (lane + 32 * j >= C4) break;
            #pragma unroll
            for (int k = 0; k < 4; ++k) { const i64 d = i64(v[4 * j + k]) - mean; const i64 dd = ex ? ((d >> ex) + ((d >> (ex - 1)) & 1)) : d; ss += dd * dd; }
        }
    }
    ss = warp_sum64(ss);
    const i64 var = floor_div_inv(ss, uint64_t(n), k.inv_n);
    const int shb = 32 - 2 * ex;
    const i64 eps = floor_div_inv((shb >= 0 ? (i64(1) << shb) : 0) + k.den / 2, uint64_t(k.den), k.inv_den);
    const i64 sd = isqrt((var + eps) << 16);
    const NormP np = norm_params(mean, ex, sd);
    u32 m = 0;
    #pragma unroll
    for (int j = 0; j < R4; ++j) {
        const int c4 = lane + 32 * j;
        if (c4 >= C4) break;
        int gv[4], bv[4];
        if (sizeof(GT) == 4 && ((reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(beta)) & 15) == 0) {
            const int4 g4 = __ldg(reinterpret_cast<const int4*>(reinterpret_cast<const int32_t*>(g) + c4 * 4));
            const int4 b4 = __ldg(reinterpret_cast<const int4*>(reinterpret_cast<const int32_t*>(beta) + c4 * 4));
            gv[0] = g4.x; gv[1] = g4.y; gv[2] = g4.z; gv[3] = g4.w; bv[0] = b4.x; bv[1] = b4.y; bv[2] = b4.z; bv[3] = b4.w;
        } else {
            #pragma unroll
            for (int k = 0; k < 4; ++k) { gv[k] = int(g[c4 * 4 + k]); bv[k] = int(beta[c4 * 4 + k]); }
        }
        #pragma unroll
        for (int k = 0; k < 4; ++k) {
            v[4 * j + k] = norm_val(v[4 * j + k], np, gv[k], bv[k]);
            m = max(m, uabs(v[4 * j + k]));
        }
        if (!QUANT) *reinterpret_cast<int4*>(Y + size_t(r) * C + c4 * 4) = make_int4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    }
    if (!QUANT) return;
    const int ee = row_exp(warp_umax(m));
    int8_t* h = hi + size_t(r) * Kp; int8_t* l = lo + size_t(r) * Kp;
    if (lane == 0) e[r] = ee;
    // the row is this warp's: one rounding form for all its lanes (the two-operation one when e <= 15)
    const int qs1 = ee > 0 ? ee - 1 : 0, qr = ee > 0 ? 1 : 0, qh = (1 << ee) >> 1;
    #pragma unroll
    for (int j = 0; j < R4; ++j) {
        const int c4 = lane + 32 * j;
        if (c4 >= C4) break;
        uint32_t hw, lw;
        if (ee <= 15) quant_pack4_e15(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3], qh, ee, hw, lw);
        else quant_pack4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3], qs1, qr, qr, hw, lw);
        *reinterpret_cast<u32*>(h + c4 * 4) = hw;
        *reinterpret_cast<u32*>(l + c4 * 4) = lw;
    }
    pad_cols(h, l, C, Kp, lane);
}

// ---------------------------------------------------------------- elementwise (src/kernels.cu:537-561)
__global__ void act_kernel(int32_t* X, size_t n, const int32_t* __restrict__ L) {
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) X[i] = lut_act(X[i], L);
}
__global__ void geglu_kernel(int32_t* A, const int32_t* __restrict__ G, size_t n, const int32_t* __restrict__ L) {
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
        A[i] = int(rshr_pos(i64(A[i]) * lut_act(G[i], L), 16));
}
__global__ void add_kernel(int32_t* X, const int32_t* __restrict__ Y, size_t n) {
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) X[i] = int(sat32(i64(X[i]) + Y[i]));
}
// channel concat, 4 channels per thread (Ca, Cb multiples of 4)
__global__ void concat_kernel(const int32_t* __restrict__ A, int Ca, const int32_t* __restrict__ Bm, int Cb, size_t rows, int32_t* __restrict__ out) {
    const int Co4 = (Ca + Cb) >> 2, Ca4 = Ca >> 2;
    const size_t tot = rows * Co4;
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < tot; i += size_t(gridDim.x) * blockDim.x) {
        const size_t r = i / Co4; const int c4 = int(i - r * Co4);
        const int4 v = c4 < Ca4 ? __ldg(reinterpret_cast<const int4*>(A + r * Ca) + c4) : __ldg(reinterpret_cast<const int4*>(Bm + r * Cb) + (c4 - Ca4));
        reinterpret_cast<int4*>(out)[i] = v;
    }
}
// nearest x2 upsample, 4 channels per thread
__global__ void upsample2_kernel(const int32_t* __restrict__ X, int B, int H, int W, int C, int32_t* __restrict__ out) {
    const int C4 = C >> 2;
    const size_t tot = size_t(B) * 4 * H * W * C4;
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < tot; i += size_t(gridDim.x) * blockDim.x) {
        const int c4 = int(i % C4); size_t p = i / C4;
        const int xo = int(p % (2 * W)); p /= 2 * W; const int yo = int(p % (2 * H)); const int b = int(p / (2 * H));
        reinterpret_cast<int4*>(out)[i] = __ldg(reinterpret_cast<const int4*>(X + ((size_t(b) * H + (yo >> 1)) * W + (xo >> 1)) * C) + c4);
    }
}

// ---------------------------------------------------------------- ChaCha20 noise and finalize (src/kernels.cu:563-599)
// ChaCha20 block function (RFC 7539 section 2.3): 16-word state = 4 constant words, the 8 key words, block counter,
// 3 nonce words (zero here); 10 double rounds, each a column round and a diagonal round of quarter rounds; output
// word i = round state i + initial state i.
__device__ __forceinline__ void chacha_qround(u32& a, u32& b, u32& c, u32& d) {
    a += b; d = __funnelshift_l(d ^ a, d ^ a, 16);
    c += d; b = __funnelshift_l(b ^ c, b ^ c, 12);
    a += b; d = __funnelshift_l(d ^ a, d ^ a, 8);
    c += d; b = __funnelshift_l(b ^ c, b ^ c, 7);
}
__device__ __forceinline__ void chacha20_block(const u32* key, u32 counter, u32 (&out)[16]) {
    u32 x[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u, key[0], key[1], key[2], key[3],
                 key[4], key[5], key[6], key[7], counter, 0u, 0u, 0u};
    #pragma unroll
    for (int i = 0; i < 16; ++i) out[i] = x[i];
    #pragma unroll
    for (int dr = 0; dr < 10; ++dr) {
        #pragma unroll
        for (int col = 0; col < 4; ++col) chacha_qround(x[col], x[4 + col], x[8 + col], x[12 + col]);
        #pragma unroll
        for (int dg = 0; dg < 4; ++dg) chacha_qround(x[dg], x[4 + (dg + 1) % 4], x[8 + (dg + 2) % 4], x[12 + (dg + 3) % 4]);
    }
    #pragma unroll
    for (int i = 0; i < 16; ++i) out[i] += x[i];
}
// Noise of one sample: 16384 values, value v = gauss[u16 v of the keystream] (little-endian halves of the output
// words, block k holding values 32k .. 32k+31), stored channel-major n[c][p] (v = 4096 c + p), and the scaled latent
// x[p][c] = rshr(n[c][p] cin, 30) in NHWC.  CTA = (a quarter of the 4096 pixels, one sample), 128 threads: thread t
// makes block 128 (t / 32) + 32 quarter + t % 32 -- 32 pixels of channel t / 32 -- writes them to n and to shared
// memory, then the CTA writes its 1024 NHWC pixels as one 16-byte store each.
__global__ void __launch_bounds__(128) noise_kernel(const uint8_t* __restrict__ seeds, const i64* __restrict__ gauss64,
                                                    const int32_t* __restrict__ gauss32, i64 cin, int32_t* __restrict__ n, int32_t* __restrict__ x) {
    __shared__ u32 key[8];
    __shared__ int32_t ns[4][1024];
    const int quarter = blockIdx.x, b = blockIdx.y, t = threadIdx.x;
    if (t < 8) {
        const uint8_t* kp = seeds + 32 * size_t(b) + 4 * t;
        key[t] = u32(kp[0]) | (u32(kp[1]) << 8) | (u32(kp[2]) << 16) | (u32(kp[3]) << 24);
    }
    __syncthreads();
    const int c = t >> 5, j = quarter * 32 + (t & 31);          // channel, block within the channel (0..127)
    u32 ks[16];
    chacha20_block(key, u32(c * 128 + j), ks);
    int v[32];
    #pragma unroll
    for (int i = 0; i < 16; ++i) {
        const u32 lo16 = ks[i] & 0xffffu, hi16 = ks[i] >> 16;
        v[2 * i] = gauss32 ? __ldg(gauss32 + lo16) : int(__ldg(gauss64 + lo16));
        v[2 * i + 1] = gauss32 ? __ldg(gauss32 + hi16) : int(__ldg(gauss64 + hi16));
    }
    int4* nout = reinterpret_cast<int4*>(n + size_t(b) * 16384 + c * 4096 + j * 32);
    #pragma unroll
    for (int i = 0; i < 8; ++i) nout[i] = make_int4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    #pragma unroll
    for (int i = 0; i < 32; ++i) ns[c][(t & 31) * 32 + i] = v[i];
    __syncthreads();
    int4* xout = reinterpret_cast<int4*>(x + size_t(b) * 16384) + quarter * 1024;
    #pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int p = t + 128 * k;
        xout[p] = make_int4(int(rshr(i64(ns[0][p]) * cin, 30)), int(rshr(i64(ns[1][p]) * cin, 30)),
                            int(rshr(i64(ns[2][p]) * cin, 30)), int(rshr(i64(ns[3][p]) * cin, 30)));
    }
}
// x0 = rshr((n - eps) sig, 16), out = clamp(rshr(x0, 8), +-32767) as little-endian int16 in n's channel-major order;
// eps is NHWC.  Thread = two neighbouring pixels of one sample: eps as two 16-byte loads, n as one 8-byte load per
// channel, the output as one packed pair of int16 per channel.
__global__ void finalize_kernel(const int32_t* __restrict__ n, const int32_t* __restrict__ eps, int B, i64 sig, uint32_t* __restrict__ out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * 2048) return;
    const int b = i >> 11, p = (i & 2047) * 2;
    const int4 e0 = __ldg(reinterpret_cast<const int4*>(eps + size_t(b) * 16384 + p * 4));
    const int4 e1 = __ldg(reinterpret_cast<const int4*>(eps + size_t(b) * 16384 + p * 4 + 4));
    const int ea[4] = {e0.x, e0.y, e0.z, e0.w}, eb[4] = {e1.x, e1.y, e1.z, e1.w};
    auto q16 = [&](int nv, int ev) -> uint32_t {
        const i64 x0 = rshr((i64(nv) - ev) * sig, 16);
        return uint32_t(uint16_t(int16_t(min(max(rshr(x0, 8), i64(-32767)), i64(32767)))));
    };
    #pragma unroll
    for (int c = 0; c < 4; ++c) {
        const size_t at = size_t(b) * 16384 + c * 4096 + p;
        const int2 nv = __ldg(reinterpret_cast<const int2*>(n + at));
        out[at >> 1] = q16(nv.x, ea[c]) | (q16(nv.y, eb[c]) << 16);
    }
}
// token embedding of the prompt rows: X[t][d] = sat32(rshr(w[id][d] m[id], s[id] - 16) + pos[t][d]) for t < T, 0 for
// the padding rows.  CTA = one row; thread = four neighbouring d (4-byte weight loads, 16-byte stores).
__global__ void text_embed_kernel(const int32_t* __restrict__ ids, int T, const int8_t* __restrict__ tw, const i64* __restrict__ tm,
                                  const i64* __restrict__ ts, const i64* __restrict__ pos, int D, int32_t* __restrict__ X) {
    const int t = blockIdx.x;
    int4* row = reinterpret_cast<int4*>(X + size_t(t) * D);
    if (t >= T) {
        for (int d4 = threadIdx.x; d4 < D / 4; d4 += blockDim.x) row[d4] = make_int4(0, 0, 0, 0);
        return;
    }
    const int id = __ldg(ids + t);
    const i64 m = __ldg(tm + id), sh = __ldg(ts + id) - 16;
    const char4* w = reinterpret_cast<const char4*>(tw + size_t(id) * D);
    const longlong2* ps = reinterpret_cast<const longlong2*>(pos + size_t(t) * D);
    for (int d4 = threadIdx.x; d4 < D / 4; d4 += blockDim.x) {
        const char4 wv = __ldg(w + d4);
        const longlong2 p01 = __ldg(ps + 2 * d4), p23 = __ldg(ps + 2 * d4 + 1);
        row[d4] = make_int4(int(sat32(rshr(i64(wv.x) * m, sh) + p01.x)), int(sat32(rshr(i64(wv.y) * m, sh) + p01.y)),
                            int(sat32(rshr(i64(wv.z) * m, sh) + p23.x)), int(sat32(rshr(i64(wv.w) * m, sh) + p23.y)));
    }
}

// ---------------------------------------------------------------- attention operands (src/kernels.cu:609-669,799-809)
// Q/K: one warp per (g, t) row of 64 values (2 per lane); rows t >= T value 0
__global__ void quant_heads_kernel(const int32_t* __restrict__ X, int B, int T, int C, int heads, int Tp, int8_t* __restrict__ hi, int8_t* __restrict__ lo,
                                   int32_t* __restrict__ e, i64* __restrict__ hs, i64* __restrict__ ls, i64* __restrict__ tsum, int tFrom) {
    const int lane = threadIdx.x & 31;
    const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int rowsPerG = Tp - tFrom;
    if (w >= B * heads * rowsPerG) return;
    const int g = w / rowsPerG, t = tFrom + w % rowsPerG, b = g / heads, h = g % heads;
    const size_t row = size_t(g) * Tp + t;
    int8_t* hp = hi + row * 64; int8_t* lp = lo + row * 64;
    if (t >= T) {
        *reinterpret_cast<uint16_t*>(hp + 2 * lane) = 0; *reinterpret_cast<uint16_t*>(lp + 2 * lane) = 0x8080;
        if (lane == 0) { e[row] = 0; hs[row] = 0; ls[row] = -128 * 64; tsum[row] = 0; }
        return;
    }
    const int2 v = __ldg(reinterpret_cast<const int2*>(X + (size_t(b) * T + t) * C + h * 64) + lane);
    const int ee = row_exp(warp_umax(max(uabs(v.x), uabs(v.y))));
    const int q0 = quant16(v.x, ee), q1 = quant16(v.y, ee);
    const int h0 = q0 >> 8, h1 = q1 >> 8, l0 = (q0 & 255) - 128, l1 = (q1 & 255) - 128;
    *reinterpret_cast<uint16_t*>(hp + 2 * lane) = uint16_t((h0 & 255) | ((h1 & 255) << 8));
    *reinterpret_cast<uint16_t*>(lp + 2 * lane) = uint16_t((l0 & 255) | ((l1 & 255) << 8));
    const i64 sh = warp_sum64(h0 + h1), sl = warp_sum64(l0 + l1), st = warp_sum64(q0 + q1);
    if (lane == 0) { e[row] = ee; hs[row] = sh; ls[row] = sl; tsum[row] = st; }
}
// V column statistics: block = (g, t-chunk of 256 rows) x 64 dims; column max (atomic)
__global__ void quant_v_max_kernel(const int32_t* __restrict__ X, int Tk, int C, int heads, u32* __restrict__ colmax) {
    __shared__ u32 sm[4][64];
    const int g = blockIdx.y, b = g / heads, h = g % heads, d = threadIdx.x & 63, ts = threadIdx.x >> 6;
    const int t0 = blockIdx.x * 256, t1 = min(Tk, t0 + 256);
    const int32_t* x = X + size_t(b) * Tk * C + h * 64 + d;
    u32 m = 0;
    for (int t = t0 + ts; t < t1; t += 4) m = max(m, uabs(__ldg(x + size_t(t) * C)));
    sm[ts][d] = m;
    __syncthreads();
    if (ts == 0) { m = max(max(sm[0][d], sm[1][d]), max(sm[2][d], sm[3][d])); if (m) atomicMax(colmax + g * 64 + d, m); }
}
// transposed quantised write [G][64][Tkp] + per-column sums of the quantised values: block = (g, 64-row t tile).
// After the tile is staged, each half-warp takes one column d and its 16 lanes four consecutive t each: the four
// values become one word of hi bytes and one of lo bytes (quant_pack4), stored at t..t+3 of row d, and the sum
// of q over them is 256 * (hi byte sum) + (lo byte sum) + 4 * 128 (q = 256 hi + lo + 128; dp4a byte sums),
// reduced over the half-warp before one atomic per column.  Padded t (>= Tk) hold 0 and quantise to 0.
__global__ void quant_v_write_kernel(const int32_t* __restrict__ X, int Tk, int C, int heads, int Tkp, const u32* __restrict__ colmax,
                                     int8_t* __restrict__ vh, int8_t* __restrict__ vl, int32_t* __restrict__ ev, i64* __restrict__ vsum) {
    __shared__ int tile[64][65];
    const int g = blockIdx.y, t0 = blockIdx.x * 64, b = g / heads, h = g % heads;
    const int tx = threadIdx.x & 63, ty = threadIdx.x >> 6;
    for (int r = ty; r < 64; r += 4) { const int t = t0 + r; tile[r][tx] = t < Tk ? __ldg(X + (size_t(b) * Tk + t) * C + h * 64 + tx) : 0; }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, tl = lane & 15;
    for (int d = 2 * warp + (lane >> 4); d < 64; d += 2 * (blockDim.x >> 5)) {
        const int e = row_exp(colmax[g * 64 + d]);
        const int qs1 = e > 0 ? e - 1 : 0, qr = e > 0 ? 1 : 0;
        uint32_t hw, lw;
        quant_pack4(tile[4 * tl][d], tile[4 * tl + 1][d], tile[4 * tl + 2][d], tile[4 * tl + 3][d], qs1, qr, qr, hw, lw);
        const size_t o = (size_t(g) * 64 + d) * Tkp + t0 + 4 * tl;
        *reinterpret_cast<uint32_t*>(vh + o) = hw;
        *reinterpret_cast<uint32_t*>(vl + o) = lw;
        int sq = 256 * __dp4a(int(hw), 0x01010101, 0) + __dp4a(int(lw), 0x01010101, 0) + 4 * 128;
        #pragma unroll
        for (int o2 = 8; o2; o2 >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o2);
        if (tl == 0 && sq) atomicAdd(reinterpret_cast<unsigned long long*>(vsum + g * 64 + d), (unsigned long long)i64(sq));
        if (blockIdx.x == 0 && tl == 0) ev[g * 64 + d] = e;
    }
}

inline unsigned grid1(size_t n, int per = 256) { return unsigned(std::min<size_t>((n + per - 1) / per, size_t(148) * 32)); }
}  // namespace

// ================================================================ host launchers (used by the engine and the C ABI)
void quant_rows(cudaStream_t st, const int32_t* X, int M, int K, int ldx, int8_t* hi, int8_t* lo, int32_t* e, int Kp) {
    VELA_REQUIRE(X && hi && lo && e && M > 0 && K > 0 && Kp >= K && ldx >= K, "quant_rows: bad arguments");
    const int Mpad = (M + 31) / 32 * 32;
    quant_rows_kernel<<<ceil_div(Mpad, 8), 256, 0, st>>>(X, M, Mpad, K, ldx, hi, lo, e, Kp);
}
void quant_rows_rm(cudaStream_t st, const int32_t* X, const uint32_t* rowmax, int M, int K, int ldx, int8_t* hi, int8_t* lo, int32_t* e, int Kp, int Mpad) {
    VELA_REQUIRE(X && rowmax && hi && lo && e && M > 0 && K > 0 && K % 4 == 0 && ldx % 4 == 0 && Kp >= K && Kp % 4 == 0 && Mpad >= M,
                 "quant_rows_rm: needs K, ldx and Kp multiples of 4");
    quant_rows_rm_kernel<<<unsigned(std::min(ceil_div(Mpad, 8), sm_count() * 16)), 256, 0, st>>>(X, rowmax, M, Mpad, K, ldx, hi, lo, e, Kp);
}
void pixmax(cudaStream_t st, const int32_t* X, int rows, int C, uint32_t* pm) {
    VELA_REQUIRE(X && pm && rows > 0 && C > 0, "pixmax: bad arguments");
    pixmax_kernel<<<ceil_div(rows, 8), 256, 0, st>>>(X, rows, C, pm);
}
void im2col3(cudaStream_t st, const int32_t* X, const uint32_t* pm, int B, int H, int W, int C, int stride, int8_t* hi, int8_t* lo, int32_t* e, int Kp) {
    VELA_REQUIRE(X && pm && hi && lo && e && Kp >= 9 * C && stride >= 1, "im2col3: bad arguments");
    const int Ho = (H - 1) / stride + 1, Wo = (W - 1) / stride + 1, rows = B * Ho * Wo, Mpad = (rows + 31) / 32 * 32;
    if (C % 4 == 0 && Kp % 4 == 0 && (reinterpret_cast<uintptr_t>(X) & 15) == 0 && (reinterpret_cast<uintptr_t>(hi) & 3) == 0 &&
        (reinterpret_cast<uintptr_t>(lo) & 3) == 0)
    {
        // whole rows per warp once the rows alone give every SM about 32 warps
        if (Mpad >= 32 * sm_count())
            im2col3_q4_kernel<true><<<ceil_div(Mpad, 8), 256, 0, st>>>(X, pm, B, H, W, C, stride, Ho, Wo, rows, Mpad, hi, lo, e, Kp);
        else
            im2col3_q4_kernel<false><<<ceil_div(Mpad * 9, 8), 256, 0, st>>>(X, pm, B, H, W, C, stride, Ho, Wo, rows, Mpad, hi, lo, e, Kp);
    }
    else
        im2col3_kernel<<<ceil_div(Mpad, 8), 256, 0, st>>>(X, pm, B, H, W, C, stride, Ho, Wo, rows, Mpad, hi, lo, e, Kp);
}
// statistics: accumulate sum/min/max, then the squared deviations, then mean/e/sd per (sample, group)
void gn_stats(cudaStream_t st, const int32_t* X, int B, int T, int C, i64 den, vela_gnstat* gs) {
    VELA_REQUIRE(X && gs && B > 0 && T > 0 && C % 32 == 0 && C <= 4096, "gn_stats: C must be a multiple of 32 (32 groups), at most 4096");
    const int cnt = B * 32, Q = C / 4, RP = std::max(1, 512 / Q);
    // one wave: as many blocks as stay resident (pass 2, the larger register footprint, decides), each a long run
    // of rows, so no second wave waits on the first and every block's prologue and reduction are paid once per SM
    const int resident = sm_count() * blocks_per_sm(reinterpret_cast<const void*>(gn_stats_kernel<2>), Q * RP, 0);
    const int chunks = std::max(1, std::min(ceil_div(T, 4 * RP), resident / B));
    const int rpb = ceil_div(T, chunks);
    gn_init_kernel<<<ceil_div(cnt, 256), 256, 0, st>>>(gs, cnt);
    const dim3 grid(ceil_div(T, rpb), B);
    gn_stats_kernel<1><<<grid, Q * RP, 0, st>>>(X, T, C, rpb, gs, cnt, den);
    gn_stats_kernel<2><<<grid, Q * RP, 0, st>>>(X, T, C, rpb, gs, cnt, den);     // + the finish (last block)
}
void gn_apply(cudaStream_t st, const int32_t* X, int B, int T, int C, const vela_gnstat* gs, const int32_t* g, const int32_t* beta,
              const int32_t* Lsig, int32_t* Y, uint32_t* pm, int8_t* hi, int8_t* lo, int32_t* e, int Kp) {
    VELA_REQUIRE(X && gs && g && beta && C % 32 == 0 && C <= 4096 && B > 0 && T > 0, "gn_apply: C must be a multiple of 32 (32 groups), at most 4096");
    const int M = B * T, PT = std::min(C / 2, 512), RP = std::max(1, 512 / PT);
    // rows per block: RP x GN_RPT (at most 256: row maxima in shared memory), touching at most GN_SPAN samples;
    // the quantised form also keeps its rows in at most 24 KB of shared memory (48 KB per block in all)
    int rpb = std::min(256, RP * GN_RPT);
    if (hi) rpb = std::min(rpb, std::max(1, 24576 / (4 * C)));
    if (rpb > 2 * T) rpb = std::max(1, 2 * T);
    const int rp = std::min(RP, rpb);
    // the blocks walk the row chunks: one wave of resident blocks
    if (hi) {
        VELA_REQUIRE(lo && e && Kp >= C && Kp % 4 == 0 && C <= 6144, "gn_apply: quantised output needs lo, e, C <= 6144 and Kp >= C, Kp % 4 == 0");
        const size_t sm = size_t(rpb) * C * 4;
        const unsigned blocks = std::min(ceil_div(M, rpb), sm_count() * blocks_per_sm(reinterpret_cast<const void*>(gn_apply_kernel<true>), PT * rp, sm));
        gn_apply_kernel<true><<<blocks, PT * rp, sm, st>>>(X, M, T, C, gs, g, beta, Lsig, Y, pm, hi, lo, e, Kp, rpb);
    } else {
        VELA_REQUIRE(Y && pm, "gn_apply: int32 output needs Y and pm");
        const unsigned blocks = std::min(ceil_div(M, rpb), sm_count() * blocks_per_sm(reinterpret_cast<const void*>(gn_apply_kernel<false>), PT * rp, 0));
        gn_apply_kernel<false><<<blocks, PT * rp, 0, st>>>(X, M, T, C, gs, g, beta, Lsig, Y, pm, hi, lo, e, Kp, rpb);
    }
}
template <bool QUANT, typename GT>
static void lnorm_dispatch(cudaStream_t st, const int32_t* X, int M, int C, const GT* g, const GT* beta, i64 den, int8_t* hi, int8_t* lo, int32_t* e, int Kp, int32_t* Y) {
    VELA_REQUIRE(den > 0 && C > 0, "lnorm: den and C must be positive");
    LnConst k;
    k.inv_n = ~uint64_t(0) / uint64_t(C);
    k.den = den; k.inv_den = ~uint64_t(0) / uint64_t(den);
    const unsigned blocks = ceil_div(M, 8);
    if (C <= 384) lnorm_kernel<3, QUANT, GT><<<blocks, 256, 0, st>>>(X, M, C, g, beta, k, hi, lo, e, Kp, Y);
    else if (C <= 640) lnorm_kernel<5, QUANT, GT><<<blocks, 256, 0, st>>>(X, M, C, g, beta, k, hi, lo, e, Kp, Y);
    else if (C <= 1280) lnorm_kernel<10, QUANT, GT><<<blocks, 256, 0, st>>>(X, M, C, g, beta, k, hi, lo, e, Kp, Y);
    else throw Error(VELA_ERR_ARG, "lnorm: C must be <= 1280");
}
void lnorm_q(cudaStream_t st, const int32_t* X, int M, int C, const int32_t* g, const int32_t* beta, i64 den, int8_t* hi, int8_t* lo, int32_t* e, int Kp) {
    VELA_REQUIRE(X && g && beta && hi && lo && e && C % 4 == 0 && Kp >= C, "lnorm_q: bad arguments");
    lnorm_dispatch<true, int32_t>(st, X, M, C, g, beta, den, hi, lo, e, Kp, nullptr);
}
void lnorm(cudaStream_t st, const int32_t* X, int M, int C, const i64* g, const i64* beta, i64 den, int32_t* Y) {
    VELA_REQUIRE(X && g && beta && Y && C % 4 == 0, "lnorm: bad arguments");
    lnorm_dispatch<false, i64>(st, X, M, C, g, beta, den, nullptr, nullptr, nullptr, 0, Y);
}
void act(cudaStream_t st, int32_t* X, size_t n, const int32_t* L) { act_kernel<<<grid1(n), 256, 0, st>>>(X, n, L); }
void geglu(cudaStream_t st, int32_t* A, const int32_t* G, size_t n, const int32_t* L) { geglu_kernel<<<grid1(n), 256, 0, st>>>(A, G, n, L); }
void add(cudaStream_t st, int32_t* X, const int32_t* Y, size_t n) { add_kernel<<<grid1(n), 256, 0, st>>>(X, Y, n); }
void concat(cudaStream_t st, const int32_t* A, int Ca, const int32_t* Bm, int Cb, int rows, int32_t* out) {
    VELA_REQUIRE(A && Bm && out && Ca % 4 == 0 && Cb % 4 == 0, "concat: channel counts must be multiples of 4");
    concat_kernel<<<grid1(size_t(rows) * (Ca + Cb) / 4), 256, 0, st>>>(A, Ca, Bm, Cb, size_t(rows), out);
}
void upsample2(cudaStream_t st, const int32_t* X, int B, int H, int W, int C, int32_t* out) {
    VELA_REQUIRE(X && out && C % 4 == 0, "upsample2: C must be a multiple of 4");
    upsample2_kernel<<<grid1(size_t(B) * 4 * H * W * C / 4), 256, 0, st>>>(X, B, H, W, C, out);
}
void noise(cudaStream_t st, const uint8_t* seeds, int B, const i64* gauss64, const int32_t* gauss32, i64 cin, int32_t* n, int32_t* x) {
    VELA_REQUIRE(seeds && (gauss64 || gauss32) && n && x && B > 0, "noise: bad arguments");
    VELA_REQUIRE((reinterpret_cast<uintptr_t>(n) & 15) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0, "noise: n and x must be 16-byte aligned");
    noise_kernel<<<dim3(4, B), 128, 0, st>>>(seeds, gauss64, gauss32, cin, n, x);
}
void finalize(cudaStream_t st, const int32_t* n, const int32_t* eps, int B, i64 sig, uint8_t* out) {
    VELA_REQUIRE(n && eps && out && B > 0, "finalize: bad arguments");
    VELA_REQUIRE((reinterpret_cast<uintptr_t>(n) & 7) == 0 && (reinterpret_cast<uintptr_t>(eps) & 15) == 0 && (reinterpret_cast<uintptr_t>(out) & 3) == 0,
                 "finalize: n must be 8-byte, eps 16-byte and out 4-byte aligned");
    finalize_kernel<<<ceil_div(B * 2048, 256), 256, 0, st>>>(n, eps, B, sig, reinterpret_cast<uint32_t*>(out));
}
void text_embed(cudaStream_t st, const int32_t* ids, int T, int rowsPad, const int8_t* tw, const i64* tm, const i64* ts, const i64* pos, int D, int32_t* X) {
    VELA_REQUIRE(ids && tw && tm && ts && pos && X, "text_embed: bad arguments");
    VELA_REQUIRE(D % 4 == 0 && rowsPad >= T && T >= 0 && (reinterpret_cast<uintptr_t>(tw) & 3) == 0 && (reinterpret_cast<uintptr_t>(pos) & 15) == 0 &&
                 (reinterpret_cast<uintptr_t>(X) & 15) == 0, "text_embed: D % 4 == 0, rowsPad >= T, aligned tw / pos / X");
    if (rowsPad > 0) text_embed_kernel<<<rowsPad, 256, 0, st>>>(ids, T, tw, tm, ts, pos, D, X);
}
void quant_heads(cudaStream_t st, const int32_t* X, int B, int T, int C, int heads, int Tp, int8_t* hi, int8_t* lo, int32_t* e, i64* hs, i64* ls, i64* tsum, int tFrom) {
    VELA_REQUIRE(hi && lo && e && hs && ls && tsum && C == heads * 64 && Tp >= T, "quant_heads: bad arguments");
    if (tFrom < T) VELA_REQUIRE(X != nullptr, "quant_heads: null X");
    const int rows = B * heads * (Tp - tFrom);
    if (rows > 0) quant_heads_kernel<<<ceil_div(rows, 8), 256, 0, st>>>(X, B, T, C, heads, Tp, hi, lo, e, hs, ls, tsum, tFrom);
}
void quant_v(cudaStream_t st, const int32_t* X, int B, int Tk, int C, int heads, int Tkp, int8_t* vh, int8_t* vl, int32_t* ev, i64* vsum, uint32_t* colmax) {
    VELA_REQUIRE(X && vh && vl && ev && vsum && colmax && C == heads * 64 && Tkp >= Tk && Tkp % 64 == 0, "quant_v: bad arguments");
    VELA_REQUIRE(((reinterpret_cast<uintptr_t>(vh) | reinterpret_cast<uintptr_t>(vl)) & 3) == 0, "quant_v: vh and vl must be 4-byte aligned");
    const int G = B * heads;
    VELA_CUDA(cudaMemsetAsync(colmax, 0, size_t(G) * 64 * 4, st));
    VELA_CUDA(cudaMemsetAsync(vsum, 0, size_t(G) * 64 * 8, st));
    quant_v_max_kernel<<<dim3(ceil_div(Tk, 256), G), 256, 0, st>>>(X, Tk, C, heads, colmax);
    quant_v_write_kernel<<<dim3(Tkp / 64, G), 256, 0, st>>>(X, Tk, C, heads, Tkp, colmax, vh, vl, ev, vsum);
}
}  // namespace vela

// ================================================================ C ABI (src/kernels.h)
using namespace vela;
#define ST static_cast<cudaStream_t>(stream)

extern "C" int vela_quant_rows(void* stream, const int32_t* X, int M, int K, int ldx, int8_t* hi, int8_t* lo, int32_t* e, int Kp) {
    return guarded("vela_quant_rows", [&] { quant_rows(ST, X, M, K, ldx, hi, lo, e, Kp); });
}
extern "C" int vela_quant_rows_rm(void* stream, const int32_t* X, const uint32_t* rowmax, int M, int K, int ldx, int8_t* hi, int8_t* lo, int32_t* e,
                                  int Kp, int Mpad) {
    return guarded("vela_quant_rows_rm", [&] { quant_rows_rm(ST, X, rowmax, M, K, ldx, hi, lo, e, Kp, Mpad); });
}
extern "C" int vela_pixmax(void* stream, const int32_t* X, int rows, int C, uint32_t* pm) {
    return guarded("vela_pixmax", [&] { pixmax(ST, X, rows, C, pm); });
}
extern "C" int vela_im2col3(void* stream, const int32_t* X, const uint32_t* pm, int B, int H, int W, int C, int stride, int8_t* hi, int8_t* lo, int32_t* e, int Kp) {
    return guarded("vela_im2col3", [&] { im2col3(ST, X, pm, B, H, W, C, stride, hi, lo, e, Kp); });
}
extern "C" int vela_gn_stats(void* stream, const int32_t* X, int B, int T, int C, int groups, long long den, vela_gnstat* gs) {
    return guarded("vela_gn_stats", [&] { VELA_REQUIRE(groups == 32, "gn_stats: 32 groups"); gn_stats(ST, X, B, T, C, den, gs); });
}
extern "C" int vela_gn_apply_row(void* stream, const int32_t* X, int B, int T, int C, int groups, const vela_gnstat* gs, const int32_t* g, const int32_t* beta,
                                 const int32_t* Lsig, int32_t* Y, uint32_t* pm, int8_t* hi, int8_t* lo, int32_t* e, int Kp) {
    return guarded("vela_gn_apply_row", [&] {
        VELA_REQUIRE(groups == 32, "gn_apply_row: 32 groups");
        gn_apply(ST, X, B, T, C, gs, g, beta, Lsig, Y, pm, hi, lo, e, Kp);
    });
}
extern "C" int vela_lnorm_q(void* stream, const int32_t* X, int M, int C, const int32_t* g, const int32_t* beta, long long den, int8_t* hi, int8_t* lo, int32_t* e, int Kp) {
    return guarded("vela_lnorm_q", [&] { lnorm_q(ST, X, M, C, g, beta, den, hi, lo, e, Kp); });
}
extern "C" int vela_lnorm(void* stream, const int32_t* X, int M, int C, const int64_t* g, const int64_t* beta, long long den, int32_t* Y) {
    return guarded("vela_lnorm", [&] { lnorm(ST, X, M, C, g, beta, den, Y); });
}
extern "C" int vela_act(void* stream, int32_t* X, size_t n, const int32_t* L) { return guarded("vela_act", [&] { act(ST, X, n, L); }); }
extern "C" int vela_geglu(void* stream, int32_t* A, const int32_t* G, size_t n, const int32_t* L) { return guarded("vela_geglu", [&] { geglu(ST, A, G, n, L); }); }
extern "C" int vela_add(void* stream, int32_t* X, const int32_t* Y, size_t n) { return guarded("vela_add", [&] { add(ST, X, Y, n); }); }
extern "C" int vela_concat(void* stream, const int32_t* A, int Ca, const int32_t* Bm, int Cb, int rows, int32_t* out) {
    return guarded("vela_concat", [&] { concat(ST, A, Ca, Bm, Cb, rows, out); });
}
extern "C" int vela_upsample2(void* stream, const int32_t* X, int B, int H, int W, int C, int32_t* out) {
    return guarded("vela_upsample2", [&] { upsample2(ST, X, B, H, W, C, out); });
}
extern "C" int vela_noise(void* stream, const uint8_t* seeds, int B, const int64_t* gauss, long long cin, int32_t* n, int32_t* x) {
    return guarded("vela_noise", [&] { noise(ST, seeds, B, gauss, nullptr, cin, n, x); });
}
extern "C" int vela_finalize(void* stream, const int32_t* n, const int32_t* eps, int B, long long sig, uint8_t* out) {
    return guarded("vela_finalize", [&] { finalize(ST, n, eps, B, sig, out); });
}
extern "C" int vela_text_embed(void* stream, const int32_t* ids, int T, int rowsPad, const int8_t* tw, const int64_t* tm, const int64_t* ts, const int64_t* pos, int D, int32_t* X) {
    return guarded("vela_text_embed", [&] { text_embed(ST, ids, T, rowsPad, tw, tm, ts, pos, D, X); });
}
extern "C" int vela_quant_heads(void* stream, const int32_t* X, int B, int T, int C, int heads, int Tp, int8_t* hi, int8_t* lo, int32_t* e, int64_t* hs, int64_t* ls, int64_t* tsum) {
    return guarded("vela_quant_heads", [&] { quant_heads(ST, X, B, T, C, heads, Tp, hi, lo, e, hs, ls, tsum, 0); });
}
extern "C" int vela_quant_heads_pad(void* stream, int G, int T, int Tp, int8_t* hi, int8_t* lo, int32_t* e, int64_t* hs, int64_t* ls, int64_t* tsum) {
    return guarded("vela_quant_heads_pad", [&] { quant_heads(ST, nullptr, 1, T, G * 64, G, Tp, hi, lo, e, hs, ls, tsum, T); });
}
extern "C" int vela_quant_v(void* stream, const int32_t* X, int B, int Tk, int C, int heads, int Tkp, int8_t* vt_hi, int8_t* vt_lo, int32_t* ev, int64_t* vsum, uint32_t* scratch) {
    return guarded("vela_quant_v", [&] { quant_v(ST, X, B, Tk, C, heads, Tkp, vt_hi, vt_lo, ev, vsum, scratch); });
}
