// Test-only harness around the REFERENCE implementation.
//
// oracle/Makefile compiles the reference's own sources (src/kernels.cu,
// src/gemm_hl.cu, src/attn.cu, src/gemm.cu, src/engine.cu, src/poisd.cpp from
// emanwrxsti/vela, unmodified, where they lie) together with this file into
// oracle/_ref/libvela_ref.so.  Tests use it on a B200 to produce golden
// vectors from the reference's own kernels, and bench.py --impl reference
// uses it to time the reference engine through its public API
// (DevModel::load, Engine, setPrompt, submit/collect: src/engine.h:16-124),
// the way the reference's --bench mode does (src/main.cpp:111-162).
// Nothing in the product links this library.
#define private public          // reach Engine's op methods to tap the UNet's intermediates
#include "engine.h"
#undef private
#include "gemm_hl.h"
#include "kernels.h"
#include "poisd.h"
#include "common.h"
#include <cstring>
#include <memory>
#include <string>
#include <thread>
#include <atomic>
#include <chrono>
#include <mutex>
#include <exception>
#include <random>

using namespace meow;

static thread_local std::string g_err;
static thread_local bool g_sync = true;      // false: launches return without waiting (timing loops)
#define GUARD(...) try { __VA_ARGS__; if (g_sync) CUDA_CHECK(cudaDeviceSynchronize()); CUDA_CHECK(cudaGetLastError()); return 0; } \
                    catch (const std::exception& ex) { g_err = ex.what(); return -1; }

extern "C" const char* ref_last_error() { return g_err.c_str(); }
extern "C" void ref_set_sync(int sync) { g_sync = sync != 0; }

// ------------------------------------------------------------------ operators (src/kernels.h, src/gemm_hl.h)
extern "C" int ref_quant_rows(const int32_t* X, int M, int K, int ldx, int8_t* hi, int8_t* lo, int32_t* e, int Kp) {
    GUARD(k_quant_rows(0, X, M, K, ldx, hi, lo, e, Kp));
}
extern "C" int ref_gemm_hl(const int8_t* Ahi, const int8_t* Alo, int lda, int Mp, int Mreal, const int8_t* W, int ldw, int Np, int Nreal, int Kp,
                           const int4* cst, const int32_t* e, int32_t* Y, int ldy, const int32_t* residual, int epi, int Cs, int32_t* Y1, int32_t* Y2,
                           const int32_t* Lphi, uint32_t* rowmax) {
    GUARD({
        ASrc A; A.src = SRC_I8; A.hi = Ahi; A.lo = Alo; A.ld8 = lda; A.e = e;
        AEpi E; E.epi = epi; E.Y = Y; E.ldy = ldy; E.residual = residual; E.Cs = Cs; E.Y1 = Y1; E.Y2 = Y2; E.Lphi = Lphi; E.rowmax = rowmax;
        k_gemm_hl2(0, A, Mp, Mreal, W, ldw, Np, Nreal, Kp, cst, E);
    });
}
extern "C" int ref_gemm_x32(const int32_t* X, int ldx, const uint32_t* rowmaxIn, int K, int Mp, int Mreal, const int8_t* W, int ldw, int Np, int Nreal, int Kp,
                            const int4* cst, int32_t* Y, int ldy, const int32_t* residual, int epi, const int32_t* Lphi, uint32_t* rowmaxOut) {
    GUARD({
        ASrc A; A.src = SRC_X32; A.x = X; A.ldx = ldx; A.rowmax = rowmaxIn; A.K = K;
        AEpi E; E.epi = epi; E.Y = Y; E.ldy = ldy; E.residual = residual; E.Lphi = Lphi; E.rowmax = rowmaxOut;
        k_gemm_hl2(0, A, Mp, Mreal, W, ldw, Np, Nreal, Kp, cst, E);
    });
}
extern "C" int ref_gemm_conv(const int32_t* img, int B, int H, int Wd, int C, int stride, const uint32_t* pm, int32_t* e, int Mp,
                             const int8_t* W, int ldw, int Np, int Nreal, int Kp, const int4* cst, int32_t* Y, int ldy, const int32_t* residual) {
    GUARD({
        const int Ho = (H - 1) / stride + 1, Wo = (Wd - 1) / stride + 1, rows = B * Ho * Wo;
        k_conv_e(0, pm, B, H, Wd, stride, e);
        ASrc A; A.src = SRC_CONV32; A.img = img; A.H = H; A.W = Wd; A.C = C; A.stride = stride; A.Ho = Ho; A.Wo = Wo; A.K = 9 * C; A.e = e;
        AEpi E; E.epi = EPI_PLAIN; E.Y = Y; E.ldy = ldy; E.residual = residual;
        k_gemm_hl2(0, A, Mp, rows, W, ldw, Np, Nreal, Kp, cst, E);
    });
}
extern "C" int ref_gemm_qkv(const int8_t* Ahi, const int8_t* Alo, int lda, const int32_t* e, int Mp, int Mreal, const int8_t* W, int ldw, int Np, int Nreal, int Kp,
                            const int4* cst, int heads, int T, int TpQ, int TpK, int C,
                            int8_t* qhi, int8_t* qlo, int32_t* qe, int64_t* qhs, int64_t* qls, int64_t* qts,
                            int8_t* khi, int8_t* klo, int32_t* ke, int64_t* khs, int64_t* kls, int64_t* kts, int32_t* V) {
    GUARD({
        ASrc A; A.src = SRC_I8; A.hi = Ahi; A.lo = Alo; A.ld8 = lda; A.e = e;
        AEpi E; E.epi = EPI_QKV; E.Y2 = V; E.heads = heads; E.T = T; E.TpQ = TpQ; E.TpK = TpK; E.C = C;
        E.qhi = qhi; E.qlo = qlo; E.qe = qe; E.qhs = qhs; E.qls = qls; E.qts = qts; E.khi = khi; E.klo = klo; E.ke = ke; E.khs = khs; E.kls = kls; E.kts = kts;
        k_gemm_hl2(0, A, Mp, Mreal, W, ldw, Np, Nreal, Kp, cst, E);
        const int B = Mreal / T;
        k_quant_heads_pad(0, B * heads, T, TpQ, qhi, qlo, qe, qhs, qls, qts);
        k_quant_heads_pad(0, B * heads, T, TpK, khi, klo, ke, khs, kls, kts);
    });
}
// deep-K path of the reference: cuBLASLt s8 GEMM on stacked [hi; lo] rows + k_epilogue (src/engine.cu:153-157)
extern "C" int ref_gemm_lt(const int8_t* Ahilo, int Mp, int Mreal, const int8_t* W, int Np, int Nreal, int Kp, const int4* cst, const int32_t* e,
                           int32_t* Cscratch, int32_t* Y, int ldy, const int32_t* residual) {
    GUARD({
        static thread_local std::unique_ptr<Gemm> lt;
        if (!lt) { lt.reset(new Gemm()); lt->init(32 << 20); }
        lt->run(0, Ahilo, Kp, 0, W, Kp, 0, Cscratch, Np, 0, 2 * Mp, Np, Kp);
        k_epilogue(0, Cscratch, Cscratch + size_t(Mp) * Np, Mreal, Nreal, Np, cst, e, Y, ldy, residual);
    });
}
extern "C" int ref_pixmax(const int32_t* X, int rows, int C, uint32_t* pm) { GUARD(k_pixmax(0, X, rows, C, pm)); }
extern "C" int ref_conv_e(const uint32_t* pm, int B, int H, int W, int stride, int32_t* e) { GUARD(k_conv_e(0, pm, B, H, W, stride, e)); }
extern "C" int ref_im2col3(const int32_t* X, const uint32_t* pm, int B, int H, int W, int C, int stride, int8_t* hi, int8_t* lo, int32_t* e, int Kp) {
    GUARD(k_im2col3(0, X, pm, B, H, W, C, stride, hi, lo, e, Kp));
}
extern "C" int ref_gn_stats(const int32_t* X, int B, int T, int C, int groups, long long den, GnStat* gs) {
    GUARD({ k_gn_stats1(0, X, B, T, C, groups, gs); k_gn_stats2(0, X, B, T, C, groups, den, gs); });
}
extern "C" int ref_gn_apply_row(const int32_t* X, int B, int T, int C, int groups, const GnStat* gs, const int32_t* g, const int32_t* beta, const int32_t* Lsig,
                                int32_t* Y, uint32_t* pm, int8_t* hi, int8_t* lo, int32_t* e, int Kp) {
    GUARD(k_gn_apply_row(0, X, B, T, C, groups, gs, g, beta, Lsig, Y, pm, hi, lo, e, Kp));
}
extern "C" int ref_lnorm_q(const int32_t* X, int M, int C, const int32_t* g, const int32_t* beta, long long den, int8_t* hi, int8_t* lo, int32_t* e, int Kp) {
    GUARD(k_lnorm_q(0, X, M, C, g, beta, den, hi, lo, e, Kp));
}
extern "C" int ref_lnorm(const int32_t* X, int M, int C, const int64_t* g, const int64_t* beta, long long den, int32_t* Y) {
    GUARD(k_lnorm(0, X, M, C, g, beta, den, Y));
}
extern "C" int ref_noise(const uint8_t* seeds, int B, const int64_t* gauss, long long cin, int32_t* n, int32_t* x) { GUARD(k_noise(0, seeds, B, gauss, cin, n, x)); }
extern "C" int ref_finalize(const int32_t* n, const int32_t* eps, int B, long long sig, uint8_t* out) { GUARD(k_finalize(0, n, eps, B, sig, out)); }
extern "C" int ref_quant_heads(const int32_t* X, int B, int T, int C, int heads, int Tp, int8_t* hi, int8_t* lo, int32_t* e, int64_t* hs, int64_t* ls, int64_t* tsum) {
    GUARD(k_quant_heads(0, X, B, T, C, heads, Tp, hi, lo, e, hs, ls, tsum));
}
extern "C" int ref_quant_v(const int32_t* X, int B, int Tk, int C, int heads, int Tkp, int8_t* vhi, int8_t* vlo, int32_t* ev, int64_t* vsum, uint32_t* scratch) {
    GUARD(k_quant_v(0, X, B, Tk, C, heads, Tkp, vhi, vlo, ev, vsum, scratch));
}
extern "C" int ref_fused_attention(const int8_t* qhi, const int8_t* qlo, const int32_t* eq, const int64_t* qhs, const int64_t* qls,
                                   const int8_t* khi, const int8_t* klo, const int32_t* ek, const int64_t* ksum,
                                   const int8_t* vthi, const int8_t* vtlo, const int32_t* ev, const int64_t* vsum,
                                   int B, int heads, int Tq, int Tqp, int Tk, int Tkp, int causal, const int64_t* Lexp, int C,
                                   int32_t* gmx, int64_t* gr, int32_t* out, uint32_t* rowmax) {
    GUARD(k_fused_attention(0, qhi, qlo, eq, qhs, qls, khi, klo, ek, ksum, vthi, vtlo, ev, vsum, B, heads, Tq, Tqp, Tk, Tkp, causal != 0, Lexp, C, gmx, gr, out, rowmax));
}
extern "C" int ref_concat(const int32_t* A, int Ca, const int32_t* Bm, int Cb, int rows, int32_t* out) { GUARD(k_concat(0, A, Ca, Bm, Cb, rows, out)); }
extern "C" int ref_upsample2(const int32_t* X, int B, int H, int W, int C, int32_t* out) { GUARD(k_upsample2(0, X, B, H, W, C, out)); }
extern "C" int ref_act(int32_t* X, size_t n, const int32_t* L) { GUARD(k_act(0, X, n, L)); }
extern "C" int ref_geglu(int32_t* A, const int32_t* G, size_t n, const int32_t* L) { GUARD(k_geglu(0, A, G, n, L)); }

// ------------------------------------------------------------------ engine (src/engine.h:16-124)
struct RefEngine {
    Poisd model; DevModel dm; std::vector<std::unique_ptr<Engine>> lanes; int batch = 0;
};
extern "C" void* ref_open(const char* path, int device, int batch, int lanes, int graph) {
    try {
        std::unique_ptr<RefEngine> r(new RefEngine());
        std::string err;
        if (!r->model.load(path, err)) throw std::runtime_error("model: " + err);
        r->dm.load(device, r->model);
        size_t freeB = 0, totB = 0; CUDA_CHECK(cudaMemGetInfo(&freeB, &totB));
        EngineConfig cfg; cfg.batch = batch; cfg.graph = graph != 0;
        cfg.arenaBytes = (freeB - (768u << 20)) / lanes;    // as src/main.cpp:121
        r->batch = batch;
        for (int l = 0; l < lanes; ++l) r->lanes.emplace_back(new Engine(r->dm, cfg));
        return r.release();
    } catch (const std::exception& ex) { g_err = ex.what(); return nullptr; }
}
extern "C" void ref_close(void* h) { delete static_cast<RefEngine*>(h); }
extern "C" int ref_set_prompt(void* h, const int* toks, int n) {
    try { auto* r = static_cast<RefEngine*>(h); std::vector<int> t(toks, toks + n); for (auto& e : r->lanes) e->setPrompt(t); return 0; }
    catch (const std::exception& ex) { g_err = ex.what(); return -1; }
}
extern "C" int ref_run(void* h, int lane, const uint8_t* seeds, uint8_t* x0, float* ms) {
    try { auto* r = static_cast<RefEngine*>(h); r->lanes[lane]->run(seeds, x0); if (ms) *ms = float(r->lanes[lane]->lastMs); return 0; }
    catch (const std::exception& ex) { g_err = ex.what(); return -1; }
}
extern "C" int ref_submit(void* h, int lane, const uint8_t* seeds) {
    try { static_cast<RefEngine*>(h)->lanes[lane]->submit(seeds); return 0; } catch (const std::exception& ex) { g_err = ex.what(); return -1; }
}
extern "C" int ref_collect(void* h, int lane, uint8_t* x0) {
    try { static_cast<RefEngine*>(h)->lanes[lane]->collect(x0); return 0; } catch (const std::exception& ex) { g_err = ex.what(); return -1; }
}
// The reference's --bench loop (src/main.cpp:124-147): per lane one host thread keeping two batches in
// flight (submit / collect), fresh random seeds per batch; both pipeline slots warmed up and captured first.
extern "C" int ref_bench(void* h, int warmup, int iters, double* seconds, long long* inferences) {
    try {
        auto* r = static_cast<RefEngine*>(h); const int B = r->batch, L = int(r->lanes.size());
        std::vector<uint8_t> s0(size_t(B) * 32, 7), x(size_t(B) * 32768);
        for (int w = 0; w < warmup; ++w) for (auto& e : r->lanes) { e->submit(s0.data()); e->submit(s0.data()); e->collect(x.data()); e->collect(x.data()); }
        std::atomic<long long> total{0}; std::exception_ptr err; std::mutex mu; std::vector<std::thread> th;
        auto t0 = std::chrono::steady_clock::now();
        for (int l = 0; l < L; ++l) th.emplace_back([&, l] {
            try {
                std::mt19937_64 rng(100 + l); std::vector<uint8_t> seeds(size_t(B) * 32), x0(size_t(B) * 32768);
                for (auto& b : seeds) b = uint8_t(rng());
                r->lanes[l]->submit(seeds.data());
                for (int it = 0; it < iters; ++it) {
                    if (it + 1 < iters) { for (auto& b : seeds) b = uint8_t(rng()); r->lanes[l]->submit(seeds.data()); }
                    r->lanes[l]->collect(x0.data());
                    total += B;
                }
            } catch (...) { std::lock_guard<std::mutex> lk(mu); if (!err) err = std::current_exception(); }
        });
        for (auto& t : th) t.join();
        if (err) std::rethrow_exception(err);
        *seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        *inferences = total.load();
        return 0;
    } catch (const std::exception& ex) { g_err = ex.what(); return -1; }
}
// text-encoder output for the prompt (src/engine.cu:491-535), 77 x 1024 int32
extern "C" int ref_context(void* h, const int* toks, int n, int32_t* out) {
    try {
        auto* r = static_cast<RefEngine*>(h); Engine& e = *r->lanes[0];
        std::vector<int> ids; ids.push_back(49406); for (int i = 0; i < n; ++i) ids.push_back(toks[i]); ids.push_back(49407);
        while (ids.size() < 77) ids.push_back(0);
        e.arena_.reset();
        Tensor ctx = e.textEncoder(ids);
        CUDA_CHECK(cudaStreamSynchronize(e.st_));
        CUDA_CHECK(cudaMemcpy(out, ctx.d, size_t(77) * 1024 * 4, cudaMemcpyDeviceToHost));
        e.arena_.reset();
        return 0;
    } catch (const std::exception& ex) { g_err = ex.what(); return -1; }
}
// One eager UNet step on lane 0 with every block output handed to `tap`; the block sequence is
// Engine::unet's (src/engine.cu:455-490), each block being the reference's own method.
typedef void (*tap_fn)(void* user, const char* name, const int32_t* host, size_t count);
extern "C" int ref_unet_taps(void* h, const uint8_t* seeds, uint8_t* x0, tap_fn tap, void* user) {
    try {
        auto* r = static_cast<RefEngine*>(h); Engine& e = *r->lanes[0]; const int B = r->batch;
        auto emit = [&](const std::string& name, const Tensor& t) {
            CUDA_CHECK(cudaStreamSynchronize(e.st_));
            std::vector<int32_t> hbuf(t.n()); CUDA_CHECK(cudaMemcpy(hbuf.data(), t.d, t.n() * 4, cudaMemcpyDeviceToHost));
            if (tap) tap(user, name.c_str(), hbuf.data(), hbuf.size());
        };
        CUDA_CHECK(cudaMemcpyAsync(e.dSeeds_, seeds, 32 * B, cudaMemcpyHostToDevice, e.st_));
        e.arena_.reset();
        k_noise(e.st_, e.dSeeds_, B, e.dm_.lutGauss, e.dm_.cCin, e.dNoise_, e.dX_);
        Tensor x; x.d = e.dX_; x.B = B; x.T = 4096; x.C = 4;
        emit("x", x);
        static const int HEADS[4] = {5, 10, 20, 20};
        int H = 64, W = 64;
        Tensor hh = e.conv3(x, H, W, e.dm_.lin("unet.conv_in"), 1);
        emit("conv_in", hh);
        std::vector<Tensor> skips; skips.push_back(hh);
        for (int i = 0; i < 4; ++i) {
            for (int j = 0; j < 2; ++j) {
                std::string n = "unet.down_blocks." + std::to_string(i) + ".resnets." + std::to_string(j);
                hh = e.resnet(hh, H, W, n); emit(n, hh);
                if (i < 3) { n = "unet.down_blocks." + std::to_string(i) + ".attentions." + std::to_string(j); hh = e.transformer(hh, n, HEADS[i]); emit(n, hh); }
                skips.push_back(hh);
            }
            if (i < 3) { std::string n = "unet.down_blocks." + std::to_string(i) + ".downsamplers.0.conv"; hh = e.conv3(hh, H, W, e.dm_.lin(n), 2); emit(n, hh); H /= 2; W /= 2; skips.push_back(hh); }
        }
        hh = e.resnet(hh, H, W, "unet.mid_block.resnets.0"); emit("unet.mid_block.resnets.0", hh);
        hh = e.transformer(hh, "unet.mid_block.attentions.0", 20); emit("unet.mid_block.attentions.0", hh);
        hh = e.resnet(hh, H, W, "unet.mid_block.resnets.1"); emit("unet.mid_block.resnets.1", hh);
        for (int i = 0; i < 4; ++i) {
            for (int j = 0; j < 3; ++j) {
                Tensor s = skips.back(); skips.pop_back();
                Tensor c = e.talloc(hh.B, hh.T, hh.C + s.C);
                k_concat(e.st_, hh.d, hh.C, s.d, s.C, hh.B * hh.T, c.d, nullptr, c.T);
                std::string n = "unet.up_blocks." + std::to_string(i) + ".resnets." + std::to_string(j);
                hh = e.resnet(c, H, W, n); emit(n, hh);
                if (i > 0) { n = "unet.up_blocks." + std::to_string(i) + ".attentions." + std::to_string(j); hh = e.transformer(hh, n, HEADS[3 - i]); emit(n, hh); }
            }
            if (i < 3) {
                Tensor u = e.talloc(hh.B, hh.T * 4, hh.C);
                k_upsample2(e.st_, hh.d, hh.B, H, W, hh.C, u.d); H *= 2; W *= 2;
                std::string n = "unet.up_blocks." + std::to_string(i) + ".upsamplers.0.conv";
                hh = e.conv3(u, H, W, e.dm_.lin(n), 1); emit(n, hh);
            }
        }
        u32* pmo = nullptr;
        Tensor nrm = e.groupnormSilu(hh, e.dm_.norm("unet.conv_norm_out"), pmo);
        Tensor eps; eps.d = e.dEps_; eps.B = B; eps.T = 4096; eps.C = 4;
        e.conv3(nrm, H, W, e.dm_.lin("unet.conv_out"), 1, eps.d, nullptr, pmo);
        emit("eps", eps);
        k_finalize(e.st_, e.dNoise_, e.dEps_, B, e.dm_.cSig, e.dOut_);
        CUDA_CHECK(cudaStreamSynchronize(e.st_)); CUDA_CHECK(cudaGetLastError());
        CUDA_CHECK(cudaMemcpy(x0, e.dOut_, size_t(B) * 32768, cudaMemcpyDeviceToHost));
        e.arena_.reset();
        return 0;
    } catch (const std::exception& ex) { g_err = ex.what(); return -1; }
}
