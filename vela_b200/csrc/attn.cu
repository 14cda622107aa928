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
// Warp roles: warp 0 TMA (Q once; K tiles + per-key ek/ksum each pass; V^T tiles in pass 2),
// warp 1 TMEM allocation + MMA issue, warps 2..17 softmax (thread = one query row = one TMEM
// lane; the four warps of a lane quarter split each 64-key tile, and the output dims, in quarters).
// TMEM: QK buffers at columns [0,192) and [192,384) (passes 0-1 alternate; pass 2 uses the first),
// P.V accumulators at [192,384) during pass 2.  All barrier waits are bounded.
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
constexpr int VSTAGE = 2 * KT_BYTES;                  // V^T hi + lo
constexpr int P_BYTES = 128 * 64;                     // one plane of P
// shared memory map (offsets from a 1024-aligned base)
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + 2 * Q_BYTES;
constexpr int OFF_V = OFF_K + KS * KSTAGE;
constexpr int OFF_P = OFF_V + VS * VSTAGE;
constexpr int OFF_KAUX = OFF_P + 2 * P_BYTES;          // per K stage: ek int32[64], ksum int64[64]
constexpr int KAUX_BYTES = 64 * 4 + 64 * 8;
constexpr int OFF_LUT = OFF_KAUX + KS * KAUX_BYTES;    // int2[1025]: (L[i], L[i+1] - L[i]); entry 1024 = (0, 0)
constexpr int SW = 16;                                 // softmax warps: four per TMEM lane quarter, 16 keys each
constexpr int THREADS = 32 * (2 + SW);
constexpr int OFF_RED = OFF_LUT + 1032 * 8;            // cross-warp reductions: 4 x 128 x 8 bytes
constexpr int OFF_WK = OFF_RED + 4 * 128 * 8;          // per softmax warp: ek[16], 128*ksum[16] of its keys
constexpr int OFF_BAR = OFF_WK + SW * 32 * 4;
constexpr int NBAR = 1 + 2 * KS + 2 * VS + 2 + 2 + 2 + 1;
constexpr int SMEM = 1024 + OFF_BAR + NBAR * 8 + 16;
constexpr int TMEM_COLS = 512;

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
};

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// s = sat32(rshr(65536 hh + T, sh)) for a shift sh in [5, 19], T = 256 xx + ll + cq + 128 ksum + 2^(sh-1) (the
// rounding term already added).  |S| < 2^36 (64 products of 16-bit values), so S fits 64 bits, S / 2^5 fits 32 bits
// and no saturation can occur: one wide multiply-add and one funnel shift of the 64-bit sum.
__device__ __forceinline__ int score_fast(int hh, int T, int sh) {
    const long long S = (long long)hh * 65536 + T;
    return int(__funnelshift_r(uint32_t(S), uint32_t(S >> 32), sh));
}

// E = expLUT(z) for z = mx - s >= 0 (z < 2^32): index min(z >> 10, 1024), the sentinel entry 1024 = (0, 0) giving
// E = 0 from z = 2^20 on; linear interpolation over the low 10 bits.
__device__ __forceinline__ int lut_exp(uint32_t z, const int2* L2) {
    const int2 e = L2[min(z >> 10, 1024u)];
    return e.x + int(((long long)e.y * int(z & 1023u)) >> 10);
}

// One 16-key quarter tile of one pass for one query row (this thread) -- scores from the three TMEM accumulators
// (HH at taddr, X at +64, LL at +128), then PASS 0: row max; PASS 1: sum of E; PASS 2: P (into pw_h / pw_l).
template <int PASS>
__device__ __forceinline__ void softmax_tile(uint32_t taddr, const int* __restrict__ wk, int shq, int r0, int cq, bool fast, bool unif, int eku,
                                             bool full, int kbase, int q, int Tk, int causal, const int2* __restrict__ L2,
                                             int& mx, uint64_t& sum, uint32_t rlo, uint32_t rhi, int& psum, uint32_t* pw_h, uint32_t* pw_l,
                                             uint64_t* rel_qk, uint64_t* rel_k) {
    // X and LL first, folded into T (16 registers), then HH: the three accumulators are never all live at once
    int s[16];
    {
        int xx[16], ll[16];
        tmem_ld16(taddr + 64, xx); tmem_ld16(taddr + 128, ll);
        tmem_ld_wait();
        if (fast && unif) {
            const int cr = cq + (r0 >> eku);       // one key exponent for the chunk: rounding term of shift shq - eku
            #pragma unroll
            for (int u = 0; u < 16; u += 4) {
                const int4 k4 = *reinterpret_cast<const int4*>(wk + 16 + u);
                s[u] = (xx[u] << 8) + (ll[u] + k4.x + cr); s[u + 1] = (xx[u + 1] << 8) + (ll[u + 1] + k4.y + cr);
                s[u + 2] = (xx[u + 2] << 8) + (ll[u + 2] + k4.z + cr); s[u + 3] = (xx[u + 3] << 8) + (ll[u + 3] + k4.w + cr);
            }
        } else if (fast) {
            #pragma unroll
            for (int u = 0; u < 16; u += 4) {
                const int4 e4 = *reinterpret_cast<const int4*>(wk + u);
                const int4 k4 = *reinterpret_cast<const int4*>(wk + 16 + u);
                s[u] = (xx[u] << 8) + (ll[u] + k4.x + cq) + (r0 >> e4.x); s[u + 1] = (xx[u + 1] << 8) + (ll[u + 1] + k4.y + cq) + (r0 >> e4.y);
                s[u + 2] = (xx[u + 2] << 8) + (ll[u + 2] + k4.z + cq) + (r0 >> e4.z); s[u + 3] = (xx[u + 3] << 8) + (ll[u + 3] + k4.w + cq) + (r0 >> e4.w);
            }
        } else {
            #pragma unroll
            for (int u = 0; u < 16; ++u) s[u] = (xx[u] << 8) + ll[u] + cq + wk[16 + u];
        }
    }
    {
        int hh[16];
        tmem_ld16(taddr, hh);
        tmem_ld_wait();
        if (fast && unif) {
            const int sh = shq - eku;
            #pragma unroll
            for (int u = 0; u < 16; ++u) s[u] = score_fast(hh[u], s[u], sh);
        } else if (fast) {
            #pragma unroll
            for (int u = 0; u < 16; ++u) s[u] = score_fast(hh[u], s[u], shq - wk[u]);
        } else {            // a shift outside [5, 19] somewhere in the tile: the 64-bit rshr with saturation
            #pragma unroll
            for (int u = 0; u < 16; ++u) s[u] = int(rshr((i64(hh[u]) << 16) + s[u], shq - wk[u]));
        }
    }
    // every accumulator of the tile is in registers: hand the QK buffer and the K stage back now, so the next
    // tile's QK products run on the tensor core while this tile's E / P arithmetic runs here
    tc_fence_before();
    __syncwarp();
    if ((threadIdx.x & 31) == 0) { mbar_arrive(rel_qk); mbar_arrive(rel_k); }
    uint32_t vmask = 0xFFFFu;   // validity by key position (a valid score may itself saturate to INT_MIN)
    if (!full) {
        vmask = 0;
        #pragma unroll
        for (int u = 0; u < 16; ++u) { const int key = kbase + u; vmask |= uint32_t(key < Tk && !(causal && key > q)) << u; }
    }
    if constexpr (PASS == 0) {
        if (!full) {
            #pragma unroll
            for (int u = 0; u < 16; ++u) s[u] = (vmask >> u) & 1u ? s[u] : INT_MIN;
        }
        #pragma unroll
        for (int u = 0; u < 16; ++u) mx = max(mx, s[u]);
    } else if constexpr (PASS == 1) {
        // each E < 2^31 (the table holds int32 values >= 0): a pair fits 32 bits
        #pragma unroll
        for (int u = 0; u < 16; u += 2) {
            uint32_t e0 = uint32_t(lut_exp(uint32_t(mx) - uint32_t(s[u]), L2)), e1 = uint32_t(lut_exp(uint32_t(mx) - uint32_t(s[u + 1]), L2));
            if (!full) { e0 = (vmask >> u) & 1u ? e0 : 0u; e1 = (vmask >> (u + 1)) & 1u ? e1 : 0u; }
            sum += e0 + e1;
        }
    } else {
        // P = min(32767, (E r + 2^46) >> 47) with r = rhi 2^32 + rlo.  E <= sum E, so E r <= 2^62 and
        // floor(E r / 2^32) = E rhi + umulhi(E, rlo) <= 2^30 fits 32 bits.  Four keys at a time, packed at once.
        #pragma unroll
        for (int u = 0; u < 16; u += 4) {
            int P[4];
            #pragma unroll
            for (int w = 0; w < 4; ++w) {
                uint32_t e = uint32_t(lut_exp(uint32_t(mx) - uint32_t(s[u + w]), L2));
                if (!full) e = (vmask >> (u + w)) & 1u ? e : 0u;
                const uint32_t h = e * rhi + (__umulhi(e, rlo) + 16384u);
                P[w] = int(min(32767u, h >> 15));
                psum += P[w];
            }
            pw_h[u / 4] = pack_hi4(P[0], P[1], P[2], P[3]);
            pw_l[u / 4] = pack_lo4(P[0], P[1], P[2], P[3]);
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
        mbar_fence_init();
    }
    if (warp == 1) { tmem_alloc(tmem_slot, TMEM_COLS); tmem_relinquish(); }
    for (int i = threadIdx.x; i <= 1024; i += blockDim.x) {
        if (i < 1024) { const int x0 = __ldg(a.lexp + i), x1 = __ldg(a.lexp + i + 1); lut2[i] = make_int2(x0, x1 - x0); }
        else lut2[i] = make_int2(0, 0);
    }
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
                mbar_arrive_expect_tx(&k_full[ks], KSTAGE + KAUX_BYTES);
                tma_load_2d(kst, &a.tmKh, &k_full[ks], 0, g * a.Tkp + j * 64);
                tma_load_2d(kst + KT_BYTES, &a.tmKl, &k_full[ks], 0, g * a.Tkp + j * 64);
                bulk_load(aux, a.ek + size_t(g) * a.Tkp + j * 64, 64 * 4, &k_full[ks]);
                bulk_load(aux + 256, a.ksum + size_t(g) * a.Tkp + j * 64, 64 * 8, &k_full[ks]);
                if (it >= 2 * nT) {
                    const int vs = j % VS;
                    if (!mbar_wait(&v_empty[vs], ((j / VS) & 1) ^ 1, a.err, DEVERR_TIMEOUT_EMPTY, a.wait_limit)) break;
                    mbar_arrive_expect_tx(&v_full[vs], VSTAGE);
                    uint8_t* vst = sm + OFF_V + vs * VSTAGE;
                    tma_load_2d(vst, &a.tmVh, &v_full[vs], j * 64, g * 64);
                    tma_load_2d(vst + KT_BYTES, &a.tmVl, &v_full[vs], j * 64, g * 64);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_i8(128, 64);
            const uint32_t qh = smem_u32(sm + OFF_Q), ql = qh + Q_BYTES;
            const uint32_t ph = smem_u32(sm + OFF_P), pl = ph + P_BYTES;
            const uint32_t pv = tmem + 192;                   // A: [192,256), Y: [256,320), D: [320,384)
            bool ok = mbar_wait(q_full, 0, a.err, DEVERR_TIMEOUT_FULL, a.wait_limit);
            auto issue_pv = [&](int j) -> bool {
                const int vs = j % VS;
                if (!mbar_wait(p_full, j & 1, a.err, DEVERR_TIMEOUT_FULL, a.wait_limit)) return false;
                if (!mbar_wait(&v_full[vs], (j / VS) & 1, a.err, DEVERR_TIMEOUT_FULL, a.wait_limit)) return false;
                tc_fence_after();
                const uint32_t vh = smem_u32(sm + OFF_V + vs * VSTAGE), vl = vh + KT_BYTES;
                #pragma unroll
                for (int kk = 0; kk < 2; ++kk) {
                    const bool acc = (j | kk) != 0;
                    mma_i8(pv, sdesc_sw64(ph + kk * 32), sdesc_sw64(vh + kk * 32), idesc, acc);
                    mma_i8(pv + 64, sdesc_sw64(ph + kk * 32), sdesc_sw64(vl + kk * 32), idesc, acc);
                    mma_i8(pv + 64, sdesc_sw64(pl + kk * 32), sdesc_sw64(vh + kk * 32), idesc, true);
                    mma_i8(pv + 128, sdesc_sw64(pl + kk * 32), sdesc_sw64(vl + kk * 32), idesc, acc);
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
    } else {
        // ---------------------------------------------------------------- softmax / output warps
        const int qq = warp & 3, kq = (warp - 2) >> 2;             // lane quarter; key quarter (and dim quarter)
        const int rl = qq * 32 + lane, q = q0 + rl;
        const uint32_t tl = uint32_t(qq * 32) << 16;
        const size_t rq = size_t(g) * a.Tqp + q;
        const int eqv = __ldg(a.eq + rq);
        const int cq = int(32768 * __ldg(a.qhs + rq) + 128 * __ldg(a.qls + rq));
        const int shq = 19 - eqv;                                   // eq <= 17, so shq >= 2
        const int r0 = 1 << (shq - 1);                              // rounding term of shift shq; >> ek gives that of shq - ek
        const int shq_min = __reduce_min_sync(0xffffffffu, shq);
        int* wk = reinterpret_cast<int*>(sm + OFF_WK) + (warp - 2) * 32;
        i64* red = reinterpret_cast<i64*>(sm + OFF_RED);          // [4][128]
        int mx = INT_MIN; uint64_t sum = 0; uint32_t rlo = 0, rhi = 0; int psum = 0;
        bool ok = true;
        // Every warp runs all iterations and every named barrier, also after a timed-out wait
        // (then it skips the work), so no warp can be left waiting on a barrier the others skipped.
        for (int pass = 0; pass < 3; ++pass) {
            for (int j = 0; j < nT; ++j) {
                const int it = pass * nT + j, ks = it % KS;
                const int b = pass < 2 ? (it & 1) : 0;
                const int ub = it < 2 * nT ? (it >> 1) : it - nT;      // earlier uses of buffer b
                if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&qk_full[b], ub & 1, a.err, DEVERR_TIMEOUT_FULL, a.wait_limit));
                if (ok) {
                    tc_fence_after();
                    // this warp's 16 keys: exponent and 128 * ksum, staged once per tile for vector reads
                    const uint8_t* aux = sm + OFF_KAUX + ks * KAUX_BYTES;
                    const int kk = kq * 16 + (lane & 15);
                    const int ekL = reinterpret_cast<const int32_t*>(aux)[kk];
                    const int kcL = int(128 * reinterpret_cast<const i64*>(aux + 256)[kk]);
                    const int emax = __reduce_max_sync(0xffffffffu, ekL), emin = __reduce_min_sync(0xffffffffu, ekL);
                    if (lane < 16) { wk[lane] = ekL; wk[16 + lane] = kcL; }
                    __syncwarp();
                    const int kbase = j * 64 + kq * 16;
                    const bool full = !a.causal && kbase + 16 <= a.Tk;
                    const bool fast = shq_min - emax >= 5;           // every shift of the tile in [5, 19]
                    const uint32_t taddr = tmem + tl + uint32_t(b * 192 + kq * 16);
                    uint32_t pw_h[4], pw_l[4];                        // P bytes of this thread's 16 keys (pass 2)
                    const bool unif = emin == emax;
                    if (pass == 0) softmax_tile<0>(taddr, wk, shq, r0, cq, fast, unif, emax, full, kbase, q, a.Tk, a.causal, lut2, mx, sum, rlo, rhi, psum, pw_h, pw_l, &qk_free[b], &k_empty[ks]);
                    else if (pass == 1) softmax_tile<1>(taddr, wk, shq, r0, cq, fast, unif, emax, full, kbase, q, a.Tk, a.causal, lut2, mx, sum, rlo, rhi, psum, pw_h, pw_l, &qk_free[b], &k_empty[ks]);
                    else softmax_tile<2>(taddr, wk, shq, r0, cq, fast, unif, emax, full, kbase, q, a.Tk, a.causal, lut2, mx, sum, rlo, rhi, psum, pw_h, pw_l, &qk_free[b], &k_empty[ks]);
                    if (pass == 2) {
                        ok = __all_sync(0xffffffffu, mbar_wait(p_free, (j & 1) ^ 1, a.err, DEVERR_TIMEOUT_EMPTY, a.wait_limit));
                        if (ok) {
                            uint8_t* php = sm + OFF_P; uint8_t* plp = php + P_BYTES;
                            *reinterpret_cast<uint4*>(php + sw64_off(rl, kq)) = make_uint4(pw_h[0], pw_h[1], pw_h[2], pw_h[3]);
                            *reinterpret_cast<uint4*>(plp + sw64_off(rl, kq)) = make_uint4(pw_l[0], pw_l[1], pw_l[2], pw_l[3]);
                            fence_async_smem();
                            __syncwarp();
                            if (lane == 0) mbar_arrive(p_full);
                        }
                    }
                }
                if (j == nT - 1 && pass < 2) {         // combine the four key quarters of each row
                    red[kq * 128 + rl] = pass == 0 ? i64(mx) : i64(sum);
                    asm volatile("bar.sync 1, %0;" :: "r"(SW * 32) : "memory");
                    i64 o[3];
                    #pragma unroll
                    for (int w = 1; w < 4; ++w) o[w - 1] = red[((kq + w) & 3) * 128 + rl];
                    asm volatile("bar.sync 1, %0;" :: "r"(SW * 32) : "memory");
                    if (pass == 0) mx = max(max(mx, int(o[0])), max(int(o[1]), int(o[2])));
                    else {
                        const uint64_t tot = sum + uint64_t(o[0]) + uint64_t(o[1]) + uint64_t(o[2]);
                        const uint64_t r = tot ? (uint64_t(1) << 62) / tot : 0;
                        rlo = uint32_t(r); rhi = uint32_t(r >> 32);
                    }
                }
            }
        }
        // ---------------------------------------------------------------- output
        red[kq * 128 + rl] = psum;
        asm volatile("bar.sync 1, %0;" :: "r"(SW * 32) : "memory");
        const i64 ps = red[rl] + red[128 + rl] + red[256 + rl] + red[384 + rl];
        const bool done = ok && __all_sync(0xffffffffu, mbar_wait(pv_done, 0, a.err, DEVERR_TIMEOUT_ACC, a.wait_limit));
        tc_fence_after();
        if (done) {
            const int bidx = g / a.heads, h = g % a.heads;
            const i64 n = a.Tkp;
            u32 am = 0;
            #pragma unroll
            for (int hv = 0; hv < 2; ++hv) {           // two halves of 8 output dims: fewer live registers
                int A[8], Y[8], D[8];
                const uint32_t col = uint32_t(192 + kq * 16 + hv * 8);
                tmem_ld8(tmem + tl + col, A); tmem_ld8(tmem + tl + col + 64, Y); tmem_ld8(tmem + tl + col + 128, D);
                tmem_ld_wait();
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
