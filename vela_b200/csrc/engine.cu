// The UNet-step engine on one B200: model loading (POISD), weight preparation, the activation
// arena, the step's composition (noise -> UNet -> finalize), the text encoder / cross-attention K/V
// of a prompt, CUDA-graph capture of the whole step and the two-slot submit / collect pipeline.
//
// Replaces the reference's DevModel / Engine (src/engine.h:16-124, src/engine.cu).  The UNet is a table of blocks
// (unet_plan) walked by one loop; it computes what src/engine.cu:389-490 computes, block for block, and also tells
// the loader which weights are 3x3 kernels and which blocks are transformers.  The text encoder / setPrompt follow
// src/engine.cu:491-574, the step and its pipeline :599-677 (forwardIO, graph per slot, submit / collect / run).
// Differences by design:
//   - every GEMM, convolution and attention runs on the tcgen05 kernels; no cuBLASLt, no score buffers;
//     3x3 convolutions quantise their windows while loading them (implicit GEMM), except the ones with 640 or more
//     output channels at 32x32 and below, which quantise each window once into an im2col buffer for the planar GEMM;
//   - weights are prepared once at load: 3x3 kernels permuted to tap-major K, N padded to 64,
//     K to 16, q|k|v and the GEGLU a|g rows merged (a|g interleaved) exactly as the reference does;
//   - the text encoder computes only the 77 real rows (every op on that path is row-local and the
//     causal attention masks the padding rows), the reference computes 96.
#include "ops.h"
#include "host_util.h"
#include "status.h"
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <map>
#include <set>
#include <memory>
#include <string>
#include <vector>

namespace vela {

// ------------------------------------------------------------------ POISD reader (src/poisd.cpp:11-35)
struct PoisdEntry { uint8_t dtype = 0; std::vector<uint32_t> dims; size_t off = 0, count = 0; };
class Poisd {
public:
    // the file read into memory this object owns
    void load(const std::string& path) {
        FILE* f = std::fopen(path.c_str(), "rb");
        if (!f) throw Error(VELA_ERR_IO, "cannot open model " + path);
        std::fseek(f, 0, SEEK_END); const long sz = std::ftell(f); std::fseek(f, 0, SEEK_SET);
        if (sz < 12) { std::fclose(f); throw Error(VELA_ERR_IO, "model file too small"); }
        own_.resize(size_t(sz));
        const size_t got = std::fread(own_.data(), 1, own_.size(), f);
        std::fclose(f);
        if (got != own_.size()) throw Error(VELA_ERR_IO, "model read error");
        parse(own_.data(), own_.size());
    }
    // a file image the caller keeps alive while this object is used (e.g. the bytes its host already read)
    void view(const uint8_t* bytes, size_t n) {
        if (!bytes || n < 12) throw Error(VELA_ERR_IO, "model image too small");
        parse(bytes, n);
    }
    bool has(const std::string& n) const { return entries_.count(n) != 0; }
    const PoisdEntry& get(const std::string& n) const {
        auto it = entries_.find(n); if (it == entries_.end()) throw Error(VELA_ERR_IO, "model lacks tensor " + n); return it->second;
    }
    const int8_t* i8(const std::string& n) const { const auto& e = get(n); if (e.dtype != 0) throw Error(VELA_ERR_IO, n + " is not int8"); return reinterpret_cast<const int8_t*>(p_ + e.off); }
    std::vector<int32_t> i32(const std::string& n) const {
        const auto& e = get(n); if (e.dtype != 2) throw Error(VELA_ERR_IO, n + " is not int32");
        std::vector<int32_t> v(e.count); std::memcpy(v.data(), p_ + e.off, e.count * 4); return v;
    }
    const std::map<std::string, PoisdEntry>& entries() const { return entries_; }
private:
    // container layout (src/poisd.cpp:17-33): "POISDv1\0", u32 count, then per tensor u16 name length, name, u8 dtype,
    // u8 rank, u32 dims[rank], little-endian data
    void parse(const uint8_t* p, size_t n) {
        p_ = p; n_ = n; entries_.clear();
        static const uint8_t MAGIC[8] = {'P', 'O', 'I', 'S', 'D', 'v', '1', 0};
        if (std::memcmp(p_, MAGIC, 8) != 0) throw Error(VELA_ERR_IO, "bad magic (not a POISDv1 file)");
        size_t pos = 8;
        auto need = [&](size_t k) { if (pos + k > n_) throw Error(VELA_ERR_IO, "truncated model file"); };
        need(4); const uint32_t count = rd32(pos); pos += 4;
        static const size_t SZ[4] = {1, 2, 4, 1};
        for (uint32_t i = 0; i < count; ++i) {
            need(2); const uint16_t nl = uint16_t(p_[pos] | (p_[pos + 1] << 8)); pos += 2;
            need(size_t(nl) + 2); std::string name(reinterpret_cast<const char*>(p_ + pos), nl); pos += nl;
            PoisdEntry e; e.dtype = p_[pos]; const uint8_t nd = p_[pos + 1]; pos += 2;
            if (e.dtype > 3) throw Error(VELA_ERR_IO, "bad dtype in " + name);
            need(size_t(4) * nd); e.count = 1;
            for (int d = 0; d < nd; ++d) { e.dims.push_back(rd32(pos)); e.count *= e.dims.back(); pos += 4; }
            need(e.count * SZ[e.dtype]); e.off = pos; pos += e.count * SZ[e.dtype];
            entries_.emplace(std::move(name), std::move(e));
        }
        if (pos != n_) throw Error(VELA_ERR_IO, "trailing data in model file");
        for (const char* t : {"unet.conv_in.w", "unet.conv_out.w", "te.tok.w", "te.pos", "lut.gauss", "lut.exp", "lut.sigmoid", "lut.phi", "c.sig", "c.cin"})
            if (!has(t)) throw Error(VELA_ERR_IO, std::string("model lacks tensor ") + t);
    }
    uint32_t rd32(size_t q) const { return uint32_t(p_[q]) | (uint32_t(p_[q + 1]) << 8) | (uint32_t(p_[q + 2]) << 16) | (uint32_t(p_[q + 3]) << 24); }
    std::vector<uint8_t> own_;
    const uint8_t* p_ = nullptr; size_t n_ = 0;
    std::map<std::string, PoisdEntry> entries_;
};

// ------------------------------------------------------------------ UNet topology as data
// The step's blocks in execution order, built once from the SD-2.1 channel / head configuration.  Engine::unet walks
// this table; the model loader uses it to find the 3x3 kernels and the transformer blocks.  Block order and tensor
// names follow the reference's UNet (src/engine.cu:455-490), since every block output is compared with it.
enum class BlockKind : uint8_t { ConvIn, Res, Xfmr, Down, Up, Out };
struct UNetBlock {
    BlockKind kind;
    std::string name;        // tensor prefix in the model file
    std::string tap;         // label of the block's output for the parity taps
    int heads = 0;           // Xfmr: 64-dim attention heads
    int xattn = -1;          // Xfmr: index of its prompt cross-attention K/V
    bool push = false;       // the result is kept for the up path
    bool pop = false;        // Res: the newest kept tensor is concatenated to the input first
};
static const std::vector<UNetBlock>& unet_plan() {
    static const std::vector<UNetBlock> plan = [] {
        std::vector<UNetBlock> p;
        const int heads[4] = {5, 10, 20, 20};              // per level; width = 64 x heads (320, 640, 1280, 1280)
        int xa = 0;
        auto add = [&](BlockKind k, std::string name, std::string tap = std::string()) {
            UNetBlock b; b.kind = k; b.tap = tap.empty() ? name : tap; b.name = std::move(name); p.push_back(std::move(b)); return &p.back();
        };
        auto attn = [&](std::string name, int h) { UNetBlock* b = add(BlockKind::Xfmr, std::move(name)); b->heads = h; b->xattn = xa++; return b; };
        add(BlockKind::ConvIn, "unet.conv_in", "conv_in")->push = true;
        for (int lv = 0; lv < 4; ++lv) {                       // down path: two resnets (+ attention above level 3)
            const std::string db = "unet.down_blocks." + std::to_string(lv);
            for (int r = 0; r < 2; ++r) {
                UNetBlock* last = add(BlockKind::Res, db + ".resnets." + std::to_string(r));
                if (lv < 3) last = attn(db + ".attentions." + std::to_string(r), heads[lv]);
                last->push = true;
            }
            if (lv < 3) add(BlockKind::Down, db + ".downsamplers.0.conv")->push = true;
        }
        add(BlockKind::Res, "unet.mid_block.resnets.0");
        attn("unet.mid_block.attentions.0", 20);
        add(BlockKind::Res, "unet.mid_block.resnets.1");
        for (int u = 0; u < 4; ++u) {                           // up path: three resnets on concatenated skips
            const std::string ub = "unet.up_blocks." + std::to_string(u);
            for (int r = 0; r < 3; ++r) {
                add(BlockKind::Res, ub + ".resnets." + std::to_string(r))->pop = true;
                if (u > 0) attn(ub + ".attentions." + std::to_string(r), heads[3 - u]);
            }
            if (u < 3) add(BlockKind::Up, ub + ".upsamplers.0.conv");
        }
        add(BlockKind::Out, "unet.conv_out", "eps");
        return p;
    }();
    return plan;
}
static bool ends_with(const std::string& s, const char* suf) { const size_t l = std::strlen(suf); return s.size() >= l && s.compare(s.size() - l, l, suf) == 0; }
// prefix of a transformer block's single inner block ("<name>.transformer_blocks.0")
static std::string inner_block(const UNetBlock& b) { return b.name + ".transformer_blocks.0"; }

// ------------------------------------------------------------------ device model
struct Lin { int N = 0, K = 0, Np = 0, Kp = 0; bool conv3 = false; int8_t* w = nullptr; int32_t* cst = nullptr; };
struct Norm { int C = 0; int32_t *g = nullptr, *beta = nullptr; i64 *g64 = nullptr, *beta64 = nullptr; i64 den = 0; };
struct HostLin { int N = 0, K = 0, Np = 0, Kp = 0; bool conv3 = false; std::vector<int8_t> w; std::vector<int32_t> cst; };

// The weights of the UNet's 3x3 kernels: every conv block of the plan and both convolutions of each resnet.
static std::set<std::string> kernel3x3_names() {
    std::set<std::string> out;
    for (const UNetBlock& b : unet_plan()) {
        if (b.kind == BlockKind::Res) { out.insert(b.name + ".conv1"); out.insert(b.name + ".conv2"); }
        else if (b.kind != BlockKind::Xfmr) out.insert(b.name);
    }
    return out;
}

// Device layout of one linear (src/engine.cu:20-46 describes the same layout): W rows padded to Np = 64k output
// channels and Kp = 16k inputs, zeros in the padding; a 3x3 kernel, stored with input index c*9 + tap, is re-ordered so
// that input (ky*3+kx)*C + c follows tap by tap (an implicit-GEMM K block then reads 32 channels of one tap); per
// output channel the constants {m, s, b, sum of the channel's weights}, and {1, 0, 0, 0} for padding channels.
static HostLin pack_linear(const Poisd& f, const std::string& base, const PoisdEntry& wt, bool kernel3x3) {
    HostLin h;
    h.N = int(wt.dims[0]); h.K = int(wt.dims[1]); h.conv3 = kernel3x3;
    h.Np = int(align_up(h.N, 64)); h.Kp = int(align_up(h.K, 16));
    if (kernel3x3 && h.K % 9 != 0) throw Error(VELA_ERR_IO, "3x3 kernel " + base + " has " + std::to_string(h.K) + " inputs, not 9 per channel");
    const int chans = kernel3x3 ? h.K / 9 : h.K;
    const int8_t* src = f.i8(base + ".w");
    const std::vector<int32_t> mul = f.i32(base + ".m"), shift = f.i32(base + ".s"), bias = f.i32(base + ".b");
    if (int(mul.size()) != h.N || int(shift.size()) != h.N || int(bias.size()) != h.N) throw Error(VELA_ERR_IO, base + ": per-channel constants do not match its rows");
    h.w.assign(size_t(h.Np) * h.Kp, 0);
    h.cst.assign(size_t(h.Np) * 4, 0);
    for (int o = 0; o < h.Np; ++o) {
        int32_t* cc = &h.cst[4 * size_t(o)];
        if (o >= h.N) { cc[0] = 1; continue; }
        const int8_t* in = src + size_t(o) * h.K;
        int8_t* row = &h.w[size_t(o) * h.Kp];
        if (kernel3x3) {
            for (int tap = 0; tap < 9; ++tap)
                for (int c = 0; c < chans; ++c) row[size_t(tap) * chans + c] = in[size_t(c) * 9 + tap];
        } else {
            std::memcpy(row, in, size_t(h.K));
        }
        int32_t acc = 0;
        for (int k = 0; k < h.K; ++k) acc += in[k];
        cc[0] = mul[o]; cc[1] = shift[o]; cc[2] = bias[o]; cc[3] = acc;
    }
    return h;
}

class Model {
public:
    int device = 0; size_t bytes = 0;
    std::map<std::string, Lin> lins; std::map<std::string, Norm> norms;
    int32_t *lut_sig = nullptr, *lut_phi = nullptr, *lut_exp = nullptr, *lut_gauss = nullptr;
    i64 c_sig = 0, c_cin = 0;
    int8_t* tok_w = nullptr; i64 *tok_m = nullptr, *tok_s = nullptr, *te_pos = nullptr; int te_dim = 0;

    ~Model() { int cur = 0; cudaGetDevice(&cur); cudaSetDevice(device); for (void* p : allocs_) cudaFree(p); cudaSetDevice(cur); }

    const Lin& lin(const std::string& n) const { auto it = lins.find(n); if (it == lins.end()) throw Error(VELA_ERR_IO, "model lacks linear " + n); return it->second; }
    const Norm& norm(const std::string& n) const { auto it = norms.find(n); if (it == norms.end()) throw Error(VELA_ERR_IO, "model lacks norm " + n); return it->second; }
    bool has_lin(const std::string& n) const { return lins.count(n) != 0; }

    void load(int dev, const std::string& path) { Poisd f; f.load(path); load(dev, f); }
    void load(int dev, const Poisd& f) {
        device = dev;
        VELA_CUDA(cudaSetDevice(dev));
        std::map<std::string, HostLin> hl;
        // every linear the file holds: <base>.w int8 [N, K] with per-channel <base>.m / .s / .b
        const std::set<std::string> k3 = kernel3x3_names();
        for (const auto& kv : f.entries()) {
            const std::string& name = kv.first;
            if (kv.second.dtype != 0 || kv.second.dims.size() != 2 || name.size() < 3 || name.compare(name.size() - 2, 2, ".w") != 0) continue;
            const std::string base = name.substr(0, name.size() - 2);
            if (base == "te.tok" || !f.has(base + ".m")) continue;          // the token table is an embedding, not a linear
            hl.emplace(base, pack_linear(f, base, kv.second, k3.count(base) != 0));
        }
        // merged projections (src/engine.cu:63-101): q|k|v rows, GEGLU a|g interleaved
        auto merge = [&](const std::string& name, const std::vector<std::string>& parts, bool interleave) {
            std::vector<const HostLin*> ps;
            for (auto& p : parts) { auto it = hl.find(p); if (it == hl.end()) return; ps.push_back(&it->second); }
            HostLin L; L.K = ps[0]->K; L.Kp = ps[0]->Kp; L.conv3 = false;
            for (auto* p : ps) { if (p->K != L.K) throw Error(VELA_ERR_IO, "merge: K mismatch in " + name); L.N += p->N; }
            L.Np = int(align_up(L.N, 64));
            L.w.assign(size_t(L.Np) * L.Kp, 0); L.cst.assign(size_t(L.Np) * 4, 0);
            for (int n = L.N; n < L.Np; ++n) L.cst[4 * size_t(n)] = 1;
            const int P = int(ps.size());
            int off = 0;
            for (int i = 0; i < P; ++i) {
                const HostLin* p = ps[i];
                for (int n = 0; n < p->N; ++n) {
                    const int dn = interleave ? n * P + i : off + n;
                    std::memcpy(&L.w[size_t(dn) * L.Kp], &p->w[size_t(n) * p->Kp], size_t(L.Kp));
                    std::memcpy(&L.cst[4 * size_t(dn)], &p->cst[4 * size_t(n)], 16);
                }
                off += p->N;
            }
            hl.emplace(name, std::move(L));
        };
        for (const UNetBlock& blk : unet_plan()) {
            if (blk.kind != BlockKind::Xfmr) continue;
            const std::string b = inner_block(blk);
            merge(b + ".attn1.to_qkv", {b + ".attn1.to_q", b + ".attn1.to_k", b + ".attn1.to_v"}, false);
            merge(b + ".ff.net.0.proj.agi", {b + ".ff.net.0.proj.a", b + ".ff.net.0.proj.g"}, true);
        }
        for (int l = 0; l < 23; ++l) {
            const std::string p = "te.layers." + std::to_string(l) + ".self_attn";
            merge(p + ".qkv", {p + ".q_proj", p + ".k_proj", p + ".v_proj"}, false);
        }
        for (auto& kv : hl) {
            Lin L; const HostLin& h = kv.second;
            L.N = h.N; L.K = h.K; L.Np = h.Np; L.Kp = h.Kp; L.conv3 = h.conv3;
            L.w = static_cast<int8_t*>(upload(h.w.data(), h.w.size()));
            L.cst = static_cast<int32_t*>(upload(h.cst.data(), h.cst.size() * 4));
            lins.emplace(kv.first, L);
        }
        // norms: <base>.g / .beta / .eps (src/engine.cu:47-56)
        for (const auto& kv : f.entries()) {
            const std::string& name = kv.first;
            if (!ends_with(name, ".g")) continue;
            const std::string base = name.substr(0, name.size() - 2);
            if (!f.has(base + ".beta") || !f.has(base + ".eps")) continue;
            const auto g = f.i32(name), bt = f.i32(base + ".beta");
            Norm nm; nm.C = int(g.size()); nm.den = f.i32(base + ".eps").at(0);
            nm.g = static_cast<int32_t*>(upload(g.data(), g.size() * 4)); nm.beta = static_cast<int32_t*>(upload(bt.data(), bt.size() * 4));
            std::vector<i64> g64(g.begin(), g.end()), b64(bt.begin(), bt.end());
            nm.g64 = static_cast<i64*>(upload(g64.data(), g64.size() * 8)); nm.beta64 = static_cast<i64*>(upload(b64.data(), b64.size() * 8));
            norms.emplace(base, nm);
        }
        auto up32 = [&](const char* n) { const auto v = f.i32(n); return static_cast<int32_t*>(upload(v.data(), v.size() * 4)); };
        auto up64 = [&](const char* n) { const auto v = f.i32(n); std::vector<i64> w(v.begin(), v.end()); return static_cast<i64*>(upload(w.data(), w.size() * 8)); };
        lut_sig = up32("lut.sigmoid"); lut_phi = up32("lut.phi"); lut_exp = up32("lut.exp"); lut_gauss = up32("lut.gauss");
        if (f.get("lut.exp").count < 1025 || f.get("lut.sigmoid").count < 2049 || f.get("lut.phi").count < 2049 || f.get("lut.gauss").count < 65536)
            throw Error(VELA_ERR_IO, "model LUTs too short");
        c_sig = f.i32("c.sig").at(0); c_cin = f.i32("c.cin").at(0);
        const PoisdEntry& tw = f.get("te.tok.w");
        te_dim = int(tw.dims.at(1));
        tok_w = static_cast<int8_t*>(upload(f.i8("te.tok.w"), tw.count));
        tok_m = up64("te.tok.m"); tok_s = up64("te.tok.s"); te_pos = up64("te.pos");
        VELA_CUDA(cudaDeviceSynchronize());
    }
private:
    std::vector<void*> allocs_;
    void* upload(const void* src, size_t n) {
        void* p = nullptr; VELA_CUDA(cudaMalloc(&p, std::max<size_t>(n, 16))); allocs_.push_back(p); bytes += n;
        VELA_CUDA(cudaMemcpy(p, src, n, cudaMemcpyHostToDevice));
        return p;
    }
};

// ------------------------------------------------------------------ engine
struct Tensor { int32_t* d = nullptr; int B = 0, T = 0, C = 0; uint32_t* rowmax = nullptr; size_t n() const { return size_t(B) * T * C; } };
struct QIn { int8_t *hi = nullptr, *lo = nullptr; int32_t* e = nullptr; int B = 0, T = 0, K = 0, Kp = 0, Mp = 0; int rows() const { return B * T; } };
struct HeadQ { int8_t *hi = nullptr, *lo = nullptr; int32_t* e = nullptr; i64 *hs = nullptr, *ls = nullptr, *ts = nullptr; int B = 0, T = 0, Tp = 0, heads = 0; };
struct KV { int8_t *khi = nullptr, *klo = nullptr, *vhi = nullptr, *vlo = nullptr; int32_t *ek = nullptr, *ev = nullptr; i64 *ksum = nullptr, *vsum = nullptr; int Tk = 0, Tkp = 0; };

struct Arena {
    uint8_t* base = nullptr; size_t cap = 0, off = 0, peak = 0;
    void* alloc(size_t n) {
        n = align_up(n, 256);
        if (off + n > cap) throw Error(VELA_ERR_ARENA, "arena exhausted (" + std::to_string((off + n) >> 20) + " MiB needed, " + std::to_string(cap >> 20) + " MiB reserved)");
        void* p = base + off; off += n; peak = std::max(peak, off); return p;
    }
};

class Engine {
public:
    typedef void (*TapFn)(void*, const char*, const int32_t*, size_t);
    Engine(const Model& m, int batch, bool graph, size_t arenaBytes) : m_(m), B_(batch), graph_(graph) {
        VELA_CUDA(cudaSetDevice(m.device));
        VELA_CUDA(cudaStreamCreateWithFlags(&st_, cudaStreamNonBlocking));
        if (!arenaBytes) arenaBytes = (size_t(1) << 30) + size_t(batch) * (size_t(512) << 20);
        arena_.cap = arenaBytes;
        arena_.base = static_cast<uint8_t*>(palloc(arenaBytes));
        for (int s = 0; s < 2; ++s) {
            dSeeds_[s] = static_cast<uint8_t*>(palloc(size_t(32) * B_)); dOut_[s] = static_cast<uint8_t*>(palloc(size_t(32768) * B_));
            VELA_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&hSeeds_[s]), size_t(32) * B_, cudaHostAllocDefault));
            VELA_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&hOut_[s]), size_t(32768) * B_, cudaHostAllocDefault));
            VELA_CUDA(cudaEventCreateWithFlags(&done_[s], cudaEventDisableTiming | cudaEventBlockingSync));
        }
        dNoise_ = static_cast<int32_t*>(palloc(size_t(B_) * 16384 * 4)); dX_ = static_cast<int32_t*>(palloc(size_t(B_) * 16384 * 4));
        dEps_ = static_cast<int32_t*>(palloc(size_t(B_) * 16384 * 4)); dIds_ = static_cast<int32_t*>(palloc(128 * 4));
        dCtx_ = static_cast<int32_t*>(palloc(size_t(77) * m.te_dim * 4));
        for (const UNetBlock& b : unet_plan()) if (b.kind == BlockKind::Xfmr) cross_.resize(std::max(cross_.size(), size_t(b.xattn) + 1));
        VELA_CUDA(cudaEventCreate(&ev0_)); VELA_CUDA(cudaEventCreateWithFlags(&ev1_, cudaEventBlockingSync));
        // this engine's own device error word: its kernels report a timed-out wait here, and each step copies it out
        // beside x0, so collect / run fail with VELA_ERR_TIMEOUT for exactly the steps that timed out
        dErr_ = static_cast<unsigned*>(palloc(sizeof(unsigned)));
        VELA_CUDA(cudaMemset(dErr_, 0, sizeof(unsigned)));
        for (int s = 0; s < 2; ++s) {
            VELA_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&hErr_[s]), sizeof(unsigned), cudaHostAllocDefault));
            *hErr_[s] = 0;
        }
        lo_.err = dErr_;
    }
    ~Engine() {
        cudaSetDevice(m_.device);
        if (st_) cudaStreamSynchronize(st_);
        if (gexec_dev_) cudaGraphExecDestroy(gexec_dev_);
        for (int s = 0; s < 2; ++s) {
            if (gexec_[s]) cudaGraphExecDestroy(gexec_[s]);
            if (done_[s]) cudaEventDestroy(done_[s]);
            if (hSeeds_[s]) cudaFreeHost(hSeeds_[s]);
            if (hOut_[s]) cudaFreeHost(hOut_[s]);
            if (hErr_[s]) cudaFreeHost(hErr_[s]);
        }
        for (void* p : persist_) cudaFree(p);
        if (ev0_) cudaEventDestroy(ev0_); if (ev1_) cudaEventDestroy(ev1_);
        if (st_) cudaStreamDestroy(st_);
    }
    int batch() const { return B_; }
    size_t arena_peak() const { return arena_.peak; }
    cudaStream_t stream() const { return st_; }
    int in_flight() const { return inflight_; }
    double last_ms = 0;

    // ---- prompt: text encoder + cross-attention K/V per transformer block (src/engine.cu:491-574)
    void set_prompt(const std::vector<int>& tokens) {
        VELA_CUDA(cudaSetDevice(m_.device));
        VELA_REQUIRE(inflight_ == 0, "set_prompt: batches still in flight");
        std::vector<int32_t> ids; ids.push_back(49406); for (int t : tokens) ids.push_back(t); ids.push_back(49407);
        VELA_REQUIRE(ids.size() <= 77, "prompt too long (at most 75 tokens)");
        while (ids.size() < 77) ids.push_back(0);
        arena_.off = 0;
        workspace_ = arena_.alloc(WORKSPACE);
        text_encoder(ids);
        const int T = 77, D = m_.te_dim;
        Tensor ctx; ctx.d = dCtx_; ctx.B = 1; ctx.T = T; ctx.C = D;
        for (const UNetBlock& blk : unet_plan()) {
            if (blk.kind != BlockKind::Xfmr) continue;
            const std::string b = inner_block(blk);
            const int heads = blk.heads, i = blk.xattn;
            const size_t mk = arena_.off;
            Tensor k = lin_x(ctx, m_.lin(b + ".attn2.to_k")), v = lin_x(ctx, m_.lin(b + ".attn2.to_v"));
            const int C = k.C, G1 = heads, Tkp = 128;
            VELA_REQUIRE(C == heads * 64, "cross-attention width");
            KV& kv = cross_.at(size_t(i));
            if (!kv.khi) {
                kv.Tk = T; kv.Tkp = Tkp;
                const size_t G = size_t(B_) * G1;
                kv.khi = static_cast<int8_t*>(palloc(G * Tkp * 64)); kv.klo = static_cast<int8_t*>(palloc(G * Tkp * 64));
                kv.ek = static_cast<int32_t*>(palloc(G * Tkp * 4)); kv.ksum = static_cast<i64*>(palloc(G * Tkp * 8));
                kv.vhi = static_cast<int8_t*>(palloc(G * 64 * Tkp)); kv.vlo = static_cast<int8_t*>(palloc(G * 64 * Tkp));
                kv.ev = static_cast<int32_t*>(palloc(G * 64 * 4)); kv.vsum = static_cast<i64*>(palloc(G * 64 * 8));
            }
            // one copy (B = 1), then replicated over the batch (src/engine.cu:558-568)
            i64* hs = static_cast<i64*>(arena_.alloc(size_t(G1) * Tkp * 8)); i64* ls = static_cast<i64*>(arena_.alloc(size_t(G1) * Tkp * 8));
            quant_heads(st_, k.d, 1, T, C, heads, Tkp, kv.khi, kv.klo, kv.ek, hs, ls, kv.ksum, 0);
            uint32_t* colmax = static_cast<uint32_t*>(arena_.alloc(size_t(G1) * 64 * 4));
            quant_v(st_, v.d, 1, T, C, heads, Tkp, kv.vhi, kv.vlo, kv.ev, kv.vsum, colmax);
            for (int bb = 1; bb < B_; ++bb) {
                const size_t o = size_t(bb) * G1;
                VELA_CUDA(cudaMemcpyAsync(kv.khi + o * Tkp * 64, kv.khi, size_t(G1) * Tkp * 64, cudaMemcpyDeviceToDevice, st_));
                VELA_CUDA(cudaMemcpyAsync(kv.klo + o * Tkp * 64, kv.klo, size_t(G1) * Tkp * 64, cudaMemcpyDeviceToDevice, st_));
                VELA_CUDA(cudaMemcpyAsync(kv.ek + o * Tkp, kv.ek, size_t(G1) * Tkp * 4, cudaMemcpyDeviceToDevice, st_));
                VELA_CUDA(cudaMemcpyAsync(kv.ksum + o * Tkp, kv.ksum, size_t(G1) * Tkp * 8, cudaMemcpyDeviceToDevice, st_));
                VELA_CUDA(cudaMemcpyAsync(kv.vhi + o * 64 * Tkp, kv.vhi, size_t(G1) * 64 * Tkp, cudaMemcpyDeviceToDevice, st_));
                VELA_CUDA(cudaMemcpyAsync(kv.vlo + o * 64 * Tkp, kv.vlo, size_t(G1) * 64 * Tkp, cudaMemcpyDeviceToDevice, st_));
                VELA_CUDA(cudaMemcpyAsync(kv.ev + o * 64, kv.ev, size_t(G1) * 64 * 4, cudaMemcpyDeviceToDevice, st_));
                VELA_CUDA(cudaMemcpyAsync(kv.vsum + o * 64, kv.vsum, size_t(G1) * 64 * 8, cudaMemcpyDeviceToDevice, st_));
            }
            arena_.off = mk;
        }
        VELA_CUDA(cudaStreamSynchronize(st_));
        VELA_CUDA(cudaGetLastError());
        if (const unsigned v = device_error(true))
            throw Error(VELA_ERR_TIMEOUT, "a kernel of the text encoder gave up a bounded wait (device error code " + std::to_string(v) + ")");
        have_prompt_ = true;
    }
    void context(int32_t* host) {
        VELA_REQUIRE(have_prompt_, "context: no prompt set");
        VELA_CUDA(cudaMemcpy(host, dCtx_, size_t(77) * m_.te_dim * 4, cudaMemcpyDeviceToHost));
    }

    // ---- one step: synchronous (src/engine.cu:650-677)
    void run(const uint8_t* seeds, uint8_t* x0) {
        VELA_REQUIRE(have_prompt_, "run: no prompt set");
        VELA_REQUIRE(inflight_ == 0, "run: batches in flight (collect them first)");
        VELA_CUDA(cudaSetDevice(m_.device));
        ensure_slot(0);
        std::memcpy(hSeeds_[0], seeds, size_t(32) * B_);
        VELA_CUDA(cudaEventRecord(ev0_, st_));
        launch(0);
        VELA_CUDA(cudaEventRecord(ev1_, st_));
        VELA_CUDA(cudaEventSynchronize(ev1_));
        VELA_CUDA(cudaGetLastError());
        float ms = 0; VELA_CUDA(cudaEventElapsedTime(&ms, ev0_, ev1_)); last_ms = ms;
        check_step(0);
        std::memcpy(x0, hOut_[0], size_t(32768) * B_);
    }
    // ---- pipelined form: two batches in flight, each with its own I/O buffers and graph (src/engine.cu:610-649)
    void submit(const uint8_t* seeds) {
        VELA_REQUIRE(have_prompt_, "submit: no prompt set");
        VELA_REQUIRE(inflight_ < 2, "submit: two batches already in flight");
        VELA_CUDA(cudaSetDevice(m_.device));
        const int slot = sub_slot_;
        ensure_slot(slot);
        std::memcpy(hSeeds_[slot], seeds, size_t(32) * B_);
        launch(slot);
        VELA_CUDA(cudaEventRecord(done_[slot], st_));
        sub_slot_ ^= 1; ++inflight_;
    }
    void collect(uint8_t* x0) {
        VELA_REQUIRE(inflight_ > 0, "collect: nothing in flight");
        const int slot = col_slot_;
        VELA_CUDA(cudaEventSynchronize(done_[slot]));
        VELA_CUDA(cudaGetLastError());
        col_slot_ ^= 1; --inflight_;
        check_step(slot);
        std::memcpy(x0, hOut_[slot], size_t(32768) * B_);
    }
    // ---- device-resident form: seeds and x0 in device memory, enqueued on st_ without waiting (slot 0's buffers)
    void launch_device(const uint8_t* dseeds, uint8_t* dx0) {
        VELA_REQUIRE(have_prompt_, "launch_device: no prompt set");
        VELA_REQUIRE(inflight_ == 0, "launch_device: batches in flight (collect them first)");
        VELA_CUDA(cudaSetDevice(m_.device));
        if (graph_ && !gexec_dev_) gexec_dev_ = capture(0, false);
        VELA_CUDA(cudaMemcpyAsync(dSeeds_[0], dseeds, size_t(32) * B_, cudaMemcpyDeviceToDevice, st_));
        if (graph_) VELA_CUDA(cudaGraphLaunch(gexec_dev_, st_));
        else forward(0, false);
        VELA_CUDA(cudaMemcpyAsync(dx0, dOut_[0], size_t(32768) * B_, cudaMemcpyDeviceToDevice, st_));
    }
    int graph_kernels() const { return graph_kernels_; }
    // Self-check of the attention kernel (Engine::testAttention, src/engine.cu:575-597): seeded activations of random
    // bit width 1..bits (0: all zero) for Q [B, Tq, C] and K, V [B, Tk, C], quantised by the library's quantisers, then
    // the tiled kernel against the plain-loop exact definition; returns the number of differing output words.
    long test_attention(int B, int Tq, int Tk, int heads, bool causal, int bits) {
        VELA_REQUIRE(inflight_ == 0, "test_attention: batches in flight");
        VELA_REQUIRE(B > 0 && Tq > 0 && Tk > 0 && Tk <= 4096 && heads > 0 && bits >= 0 && bits <= 31, "test_attention: bad arguments");
        VELA_CUDA(cudaSetDevice(m_.device));
        const int C = 64 * heads, G = B * heads, Tqp = int(align_up(Tq, 128)), Tkp = int(align_up(Tk, 64));
        const size_t mark = arena_.off;
        uint64_t state = 0x243F6A8885A308D3ull ^ (uint64_t(B) << 48) ^ (uint64_t(Tq) << 24) ^ uint64_t(Tk);
        auto draw = [&](int T) {
            std::vector<int32_t> h(size_t(B) * T * C);
            for (auto& v : h) {
                state += 0x9E3779B97F4A7C15ull;
                uint64_t z = (state ^ (state >> 30)) * 0xBF58476D1CE4E5B9ull; z = (z ^ (z >> 27)) * 0x94D049BB133111EBull; z ^= z >> 31;
                const int w = bits ? 1 + int((z >> 40) % uint64_t(bits)) : 0;
                v = w ? int32_t(int64_t(z & ((uint64_t(1) << w) - 1)) - (int64_t(1) << (w - 1))) : 0;
            }
            int32_t* d = static_cast<int32_t*>(arena_.alloc(h.size() * 4));
            VELA_CUDA(cudaMemcpyAsync(d, h.data(), h.size() * 4, cudaMemcpyHostToDevice, st_));
            VELA_CUDA(cudaStreamSynchronize(st_));
            return d;
        };
        const int32_t *xq = draw(Tq), *xk = draw(Tk), *xv = draw(Tk);
        HeadQ q = head_alloc(B, heads, Tq, Tqp), k = head_alloc(B, heads, Tk, Tkp);
        quant_heads(st_, xq, B, Tq, C, heads, Tqp, q.hi, q.lo, q.e, q.hs, q.ls, q.ts, 0);
        quant_heads(st_, xk, B, Tk, C, heads, Tkp, k.hi, k.lo, k.e, k.hs, k.ls, k.ts, 0);
        Tensor v; v.B = B; v.T = Tk; v.C = C; v.d = const_cast<int32_t*>(xv);
        const KV kv = kv_of(k, v, heads);
        int32_t* got = static_cast<int32_t*>(arena_.alloc(size_t(B) * Tq * C * 4));
        int32_t* ref = static_cast<int32_t*>(arena_.alloc(size_t(B) * Tq * C * 4));
        fused_attention(st_, q.hi, q.lo, q.e, q.hs, q.ls, kv.khi, kv.klo, kv.ek, kv.ksum, kv.vhi, kv.vlo, kv.ev, kv.vsum,
                        B, heads, Tq, Tqp, Tk, Tkp, causal, m_.lut_exp, C, got, nullptr, lo_);
        attention_plain(st_, q.hi, q.lo, q.e, Tqp, kv.khi, kv.klo, kv.ek, kv.vhi, kv.vlo, kv.ev, B, heads, Tq, Tk, Tkp, causal, m_.lut_exp, C, ref);
        std::vector<int32_t> hg(size_t(B) * Tq * C), hr(hg.size());
        VELA_CUDA(cudaMemcpyAsync(hg.data(), got, hg.size() * 4, cudaMemcpyDeviceToHost, st_));
        VELA_CUDA(cudaMemcpyAsync(hr.data(), ref, hr.size() * 4, cudaMemcpyDeviceToHost, st_));
        VELA_CUDA(cudaStreamSynchronize(st_));
        arena_.off = mark;
        if (const unsigned v2 = device_error(true)) throw Error(VELA_ERR_TIMEOUT, "test_attention: a bounded wait gave up (device error code " + std::to_string(v2) + ")");
        long bad = 0;
        for (size_t i = 0; i < hg.size(); ++i) bad += hg[i] != hr[i];
        return bad;
    }
    // the engine's device error word (synchronises the engine's stream); clear: reset it to zero
    unsigned device_error(bool clear) {
        VELA_CUDA(cudaSetDevice(m_.device));
        VELA_CUDA(cudaStreamSynchronize(st_));
        unsigned v = 0;
        VELA_CUDA(cudaMemcpy(&v, dErr_, sizeof(v), cudaMemcpyDeviceToHost));
        if (clear && v) VELA_CUDA(cudaMemset(dErr_, 0, sizeof(unsigned)));
        return v;
    }
    // ---- one eager step with every block output handed to `tap` (parity against the reference's blocks)
    void step_taps(const uint8_t* seeds, uint8_t* x0, TapFn tap, void* user) {
        VELA_REQUIRE(have_prompt_, "step_taps: no prompt set");
        VELA_REQUIRE(inflight_ == 0, "step_taps: batches in flight");
        VELA_CUDA(cudaSetDevice(m_.device));
        std::memcpy(hSeeds_[0], seeds, size_t(32) * B_);
        tap_ = tap; tap_user_ = user;
        try { forward(0); } catch (...) { tap_ = nullptr; throw; }
        tap_ = nullptr;
        VELA_CUDA(cudaStreamSynchronize(st_));
        VELA_CUDA(cudaGetLastError());
        check_step(0);
        std::memcpy(x0, hOut_[0], size_t(32768) * B_);
    }

private:
    const Model& m_; int B_; bool graph_;
    cudaStream_t st_ = nullptr; Arena arena_; std::vector<void*> persist_;
    uint8_t *dSeeds_[2] = {nullptr, nullptr}, *dOut_[2] = {nullptr, nullptr}, *hSeeds_[2] = {nullptr, nullptr}, *hOut_[2] = {nullptr, nullptr};
    cudaGraphExec_t gexec_[2] = {nullptr, nullptr}; bool ready_[2] = {false, false};
    cudaGraphExec_t gexec_dev_ = nullptr; int graph_kernels_ = 0;
    cudaEvent_t done_[2] = {nullptr, nullptr}, ev0_ = nullptr, ev1_ = nullptr;
    int inflight_ = 0, sub_slot_ = 0, col_slot_ = 0;
    int32_t *dNoise_ = nullptr, *dX_ = nullptr, *dEps_ = nullptr, *dIds_ = nullptr, *dCtx_ = nullptr;
    unsigned* dErr_ = nullptr; unsigned* hErr_[2] = {nullptr, nullptr}; LaunchOpts lo_;
    std::vector<KV> cross_;                   // per transformer block of the plan: the prompt's cross-attention K/V
    bool have_prompt_ = false;
    TapFn tap_ = nullptr; void* tap_user_ = nullptr;
    static constexpr size_t WORKSPACE = size_t(64) << 20;    // split-K partials

    void* palloc(size_t n) { void* p = nullptr; VELA_CUDA(cudaMalloc(&p, std::max<size_t>(n, 16))); persist_.push_back(p); return p; }
    Tensor talloc(int B, int T, int C) { Tensor t; t.B = B; t.T = T; t.C = C; t.d = static_cast<int32_t*>(arena_.alloc(t.n() * 4)); return t; }
    uint32_t* rowmax_alloc(int rows) { auto* p = static_cast<uint32_t*>(arena_.alloc(size_t(rows) * 4)); VELA_CUDA(cudaMemsetAsync(p, 0, size_t(rows) * 4, st_)); return p; }
    QIn qalloc(int B, int T, int K) {
        QIn q; q.B = B; q.T = T; q.K = K; q.Kp = int(align_up(K, 16)); q.Mp = int(align_up(size_t(B) * T, 64));
        q.hi = static_cast<int8_t*>(arena_.alloc(size_t(q.Mp) * q.Kp)); q.lo = static_cast<int8_t*>(arena_.alloc(size_t(q.Mp) * q.Kp));
        q.e = static_cast<int32_t*>(arena_.alloc(size_t(q.Mp) * 4));
        return q;
    }
    HeadQ head_alloc(int B, int heads, int T, int Tp) {
        HeadQ h; h.B = B; h.T = T; h.Tp = Tp; h.heads = heads; const size_t G = size_t(B) * heads;
        h.hi = static_cast<int8_t*>(arena_.alloc(G * Tp * 64)); h.lo = static_cast<int8_t*>(arena_.alloc(G * Tp * 64));
        h.e = static_cast<int32_t*>(arena_.alloc(G * Tp * 4));
        h.hs = static_cast<i64*>(arena_.alloc(G * Tp * 8)); h.ls = static_cast<i64*>(arena_.alloc(G * Tp * 8)); h.ts = static_cast<i64*>(arena_.alloc(G * Tp * 8));
        return h;
    }
    void emit(const std::string& name, const Tensor& t) {
        if (!tap_) return;
        VELA_CUDA(cudaStreamSynchronize(st_));
        std::vector<int32_t> h(t.n());
        VELA_CUDA(cudaMemcpy(h.data(), t.d, t.n() * 4, cudaMemcpyDeviceToHost));
        tap_(tap_user_, name.c_str(), h.data(), h.size());
    }
    vela_aepi epi_plain(int32_t* Y, int ldy, const int32_t* R, uint32_t* rowmax) {
        vela_aepi E; std::memset(&E, 0, sizeof(E));
        E.epi = VELA_EPI_PLAIN; E.Y = Y; E.ldy = ldy; E.residual = R; E.rowmax = rowmax;
        E.workspace = workspace_; E.workspace_bytes = WORKSPACE;
        return E;
    }
    void* workspace_ = nullptr;

    // ---- ops
    Tensor lin_q(const QIn& q, const Lin& L, int32_t* out = nullptr, const int32_t* residual = nullptr, uint32_t* rowmax = nullptr) {
        VELA_REQUIRE(q.K == L.K && q.Kp == L.Kp, "lin_q: K mismatch");
        Tensor y; y.B = q.B; y.T = q.T; y.C = L.N; y.d = out ? out : static_cast<int32_t*>(arena_.alloc(y.n() * 4)); y.rowmax = rowmax;
        vela_asrc A; std::memset(&A, 0, sizeof(A)); A.src = VELA_SRC_I8; A.hi = q.hi; A.lo = q.lo; A.ld8 = q.Kp; A.e = q.e;
        gemm_w8a16(st_, A, q.Mp, q.rows(), L.w, L.Kp, L.Np, L.N, L.Kp, L.cst, epi_plain(y.d, L.N, residual, rowmax), lo_);
        return y;
    }
    // int32 input quantised on load (Engine::linX, src/engine.cu:162-175); the row max comes from the producer or a pixmax pass
    Tensor lin_x(const Tensor& x, const Lin& L, int32_t* out = nullptr, const int32_t* residual = nullptr, bool wantRowmax = false) {
        VELA_REQUIRE(x.C == L.K, "lin_x: K mismatch");
        const int rows = x.B * x.T;
        const uint32_t* rm = x.rowmax;
        if (!rm) { uint32_t* p = static_cast<uint32_t*>(arena_.alloc(size_t(rows) * 4)); pixmax(st_, x.d, rows, x.C, p); rm = p; }
        Tensor y; y.B = x.B; y.T = x.T; y.C = L.N; y.d = out ? out : static_cast<int32_t*>(arena_.alloc(y.n() * 4));
        if (wantRowmax) y.rowmax = rowmax_alloc(rows);
        gemm_x(x.d, rows, x.C, rm, L, epi_plain(y.d, L.N, residual, y.rowmax));
        return y;
    }
    // GEMM on an int32 input with known row maxima.  Large inputs are quantised once into hi / lo planes (one read,
    // planes in the arena) and run on the planar TMA path, which spares the GEMM the per-column-tile re-quantising
    // of the quantise-on-load source; small ones quantise on load.
    void gemm_x(const int32_t* xd, int rows, int K, const uint32_t* rm, const Lin& L, const vela_aepi& E) {
        if (size_t(rows) * size_t(K) >= (size_t(1) << 21) && K % 4 == 0) {
            const int Mp = int(align_up(rows, 64));
            int8_t* hi = static_cast<int8_t*>(arena_.alloc(size_t(Mp) * L.Kp)); int8_t* lo = static_cast<int8_t*>(arena_.alloc(size_t(Mp) * L.Kp));
            int32_t* e = static_cast<int32_t*>(arena_.alloc(size_t(Mp) * 4));
            quant_rows_rm(st_, xd, rm, rows, K, K, hi, lo, e, L.Kp, Mp);
            vela_asrc A; std::memset(&A, 0, sizeof(A)); A.src = VELA_SRC_I8; A.hi = hi; A.lo = lo; A.ld8 = L.Kp; A.e = e;
            gemm_w8a16(st_, A, Mp, rows, L.w, L.Kp, L.Np, L.N, L.Kp, L.cst, E, lo_);
            return;
        }
        vela_asrc A; std::memset(&A, 0, sizeof(A)); A.src = VELA_SRC_X32; A.x = xd; A.ldx = K; A.rowmax = rm; A.K = L.K;
        gemm_w8a16(st_, A, int(align_up(rows, 64)), rows, L.w, L.Kp, L.Np, L.N, L.Kp, L.cst, E, lo_);
    }
    // Which 3x3 convolutions run as explicit im2col + planar GEMM: at least 640 output channels on at most 32 x 32
    // pixels, where the implicit form would re-quantise each window for four or more column tiles.  At 64 x 64 with
    // 320 channels (two column tiles) the implicit conv is faster.
    static bool explicit_im2col(const Lin& L, int out_pixels) { return L.N >= 640 && out_pixels <= 1024; }
    // 3x3 pad-1 convolution (Engine::conv3, src/engine.cu:254-280): implicit GEMM on the int32 image
    Tensor conv3(const Tensor& x, int H, int W, const Lin& L, int stride, int32_t* out = nullptr, const int32_t* residual = nullptr, const uint32_t* pmIn = nullptr) {
        VELA_REQUIRE(L.conv3 && x.C * 9 == L.K, "conv3: shape mismatch");
        const int Ho = (H - 1) / stride + 1, Wo = (W - 1) / stride + 1, rows = x.B * Ho * Wo;
        Tensor y; y.B = x.B; y.T = Ho * Wo; y.C = L.N; y.d = out ? out : static_cast<int32_t*>(arena_.alloc(y.n() * 4));
        const size_t mk = arena_.off;
        const uint32_t* pm = pmIn;
        if (!pm) { uint32_t* p = static_cast<uint32_t*>(arena_.alloc(size_t(x.B) * H * W * 4)); pixmax(st_, x.d, x.B * H * W, x.C, p); pm = p; }
        const int Mp = int(align_up(rows, 64));
        int32_t* e = static_cast<int32_t*>(arena_.alloc(size_t(Mp) * 4));
        if (explicit_im2col(L, Ho * Wo) && x.C % 4 == 0) {
            // the deep levels: every window quantised once into hi / lo planes (the reference's engine takes its
            // im2col path here too), then the planar GEMM with wide tiles
            int8_t* hi = static_cast<int8_t*>(arena_.alloc(size_t(Mp) * L.Kp)); int8_t* lo = static_cast<int8_t*>(arena_.alloc(size_t(Mp) * L.Kp));
            im2col3(st_, x.d, pm, x.B, H, W, x.C, stride, hi, lo, e, L.Kp);
            vela_asrc A; std::memset(&A, 0, sizeof(A)); A.src = VELA_SRC_I8; A.hi = hi; A.lo = lo; A.ld8 = L.Kp; A.e = e;
            gemm_w8a16(st_, A, Mp, rows, L.w, L.Kp, L.Np, L.N, L.Kp, L.cst, epi_plain(y.d, L.N, residual, nullptr), lo_);
            arena_.off = mk;
            return y;
        }
        // the other depths, the 4-channel input image included, are quantised while loaded: no im2col buffer
        conv_e(st_, pm, x.B, H, W, stride, e);
        vela_asrc A; std::memset(&A, 0, sizeof(A)); A.src = VELA_SRC_CONV32; A.img = x.d; A.H = H; A.W = W; A.C = x.C; A.stride = stride; A.Ho = Ho; A.Wo = Wo; A.K = L.K; A.e = e;
        gemm_w8a16(st_, A, Mp, rows, L.w, L.Kp, L.Np, L.N, L.Kp, L.cst, epi_plain(y.d, L.N, residual, nullptr), lo_);
        arena_.off = mk;
        return y;
    }
    vela_gnstat* gn_stats_of(const Tensor& x, const Norm& n) {
        VELA_REQUIRE(n.C == x.C, "groupnorm: C mismatch");
        vela_gnstat* gs = static_cast<vela_gnstat*>(arena_.alloc(sizeof(vela_gnstat) * x.B * 32));
        gn_stats(st_, x.d, x.B, x.T, x.C, n.den, gs);
        return gs;
    }
    // Engine::groupnormSilu (src/engine.cu:242-253)
    Tensor gn_silu(const Tensor& x, const Norm& n, uint32_t*& pm) {
        Tensor y = talloc(x.B, x.T, x.C);
        pm = static_cast<uint32_t*>(arena_.alloc(size_t(x.B) * x.T * 4));
        const size_t mk = arena_.off;
        vela_gnstat* gs = gn_stats_of(x, n);
        gn_apply(st_, x.d, x.B, x.T, x.C, gs, n.g, n.beta, m_.lut_sig, y.d, pm, nullptr, nullptr, nullptr, 0);
        arena_.off = mk;
        return y;
    }
    // Engine::groupnormQ (src/engine.cu:231-241)
    QIn gn_q(const Tensor& x, const Norm& n) {
        QIn q = qalloc(x.B, x.T, x.C);
        const size_t mk = arena_.off;
        vela_gnstat* gs = gn_stats_of(x, n);
        gn_apply(st_, x.d, x.B, x.T, x.C, gs, n.g, n.beta, nullptr, nullptr, nullptr, q.hi, q.lo, q.e, q.Kp);
        arena_.off = mk;
        return q;
    }
    // Engine::layernormQ (src/engine.cu:225-230)
    QIn ln_q(const Tensor& x, const Norm& n) {
        VELA_REQUIRE(n.C == x.C, "layernorm: C mismatch");
        QIn q = qalloc(x.B, x.T, x.C);
        lnorm_q(st_, x.d, x.B * x.T, x.C, n.g, n.beta, n.den, q.hi, q.lo, q.e, q.Kp);
        return q;
    }
    // merged q|k|v GEMM with head quantisation in the epilogue (Engine::linQ3H, src/engine.cu:318-331)
    void qkv(const QIn& n, const Lin& L, int C, int heads, int T, HeadQ& q, HeadQ& k, Tensor& v) {
        VELA_REQUIRE(n.K == L.K && L.N == 3 * C && C == heads * 64, "qkv: shape mismatch");
        const int TpQ = int(align_up(T, 128)), TpK = int(align_up(T, 64));
        q = head_alloc(n.B, heads, T, TpQ); k = head_alloc(n.B, heads, T, TpK); v = talloc(n.B, T, C);
        vela_aepi E; std::memset(&E, 0, sizeof(E));
        E.epi = VELA_EPI_QKV; E.Y2 = v.d; E.heads = heads; E.T = T; E.TpQ = TpQ; E.TpK = TpK; E.C = C;
        E.qhi = q.hi; E.qlo = q.lo; E.qe = q.e; E.qhs = q.hs; E.qls = q.ls; E.qts = q.ts;
        E.khi = k.hi; E.klo = k.lo; E.ke = k.e; E.khs = k.hs; E.kls = k.ls; E.kts = k.ts;
        vela_asrc A; std::memset(&A, 0, sizeof(A)); A.src = VELA_SRC_I8; A.hi = n.hi; A.lo = n.lo; A.ld8 = n.Kp; A.e = n.e;
        gemm_w8a16(st_, A, n.Mp, n.rows(), L.w, L.Kp, L.Np, L.N, L.Kp, L.cst, E, lo_);
        if (TpQ > T) quant_heads(st_, nullptr, n.B, T, C, heads, TpQ, q.hi, q.lo, q.e, q.hs, q.ls, q.ts, T);
        if (TpK > T) quant_heads(st_, nullptr, n.B, T, C, heads, TpK, k.hi, k.lo, k.e, k.hs, k.ls, k.ts, T);
    }
    // query of the cross attention: GEMM with the head quantisation fused (k_quant_heads of src/engine.cu:358-360)
    HeadQ q_only(const QIn& n, const Lin& L, int C, int heads, int T) {
        VELA_REQUIRE(n.K == L.K && L.N == C && C == heads * 64, "q projection: shape mismatch");
        const int TpQ = int(align_up(T, 128));
        HeadQ q = head_alloc(n.B, heads, T, TpQ);
        vela_aepi E; std::memset(&E, 0, sizeof(E));
        E.epi = VELA_EPI_QKV; E.heads = heads; E.T = T; E.TpQ = TpQ; E.TpK = TpQ; E.C = C;
        E.qhi = q.hi; E.qlo = q.lo; E.qe = q.e; E.qhs = q.hs; E.qls = q.ls; E.qts = q.ts;
        vela_asrc A; std::memset(&A, 0, sizeof(A)); A.src = VELA_SRC_I8; A.hi = n.hi; A.lo = n.lo; A.ld8 = n.Kp; A.e = n.e;
        gemm_w8a16(st_, A, n.Mp, n.rows(), L.w, L.Kp, L.Np, L.N, L.Kp, L.cst, E, lo_);
        if (TpQ > T) quant_heads(st_, nullptr, n.B, T, C, heads, TpQ, q.hi, q.lo, q.e, q.hs, q.ls, q.ts, T);
        return q;
    }
    // V columns of a self attention (Engine::quantKVH, src/engine.cu:332-340)
    KV kv_of(const HeadQ& k, const Tensor& v, int heads) {
        KV kv; kv.Tk = k.T; kv.Tkp = k.Tp; kv.khi = k.hi; kv.klo = k.lo; kv.ek = k.e; kv.ksum = k.ts;
        const size_t G = size_t(v.B) * heads;
        kv.vhi = static_cast<int8_t*>(arena_.alloc(G * 64 * kv.Tkp)); kv.vlo = static_cast<int8_t*>(arena_.alloc(G * 64 * kv.Tkp));
        kv.ev = static_cast<int32_t*>(arena_.alloc(G * 64 * 4)); kv.vsum = static_cast<i64*>(arena_.alloc(G * 64 * 8));
        uint32_t* colmax = static_cast<uint32_t*>(arena_.alloc(G * 64 * 4));
        quant_v(st_, v.d, v.B, k.T, v.C, heads, kv.Tkp, kv.vhi, kv.vlo, kv.ev, kv.vsum, colmax);
        return kv;
    }
    Tensor attention(const HeadQ& q, const KV& kv, int heads, bool causal, int Tq, int C) {
        Tensor out = talloc(q.B, Tq, C);
        out.rowmax = rowmax_alloc(q.B * Tq);
        fused_attention(st_, q.hi, q.lo, q.e, q.hs, q.ls, kv.khi, kv.klo, kv.ek, kv.ksum, kv.vhi, kv.vlo, kv.ev, kv.vsum,
                        q.B, heads, Tq, q.Tp, kv.Tk, kv.Tkp, causal, m_.lut_exp, C, out.d, out.rowmax, lo_);
        return out;
    }
    // GroupNorm + SiLU of x, then a 3x3 convolution of the result (stride 1) into `out` (+ residual): the resnet's two
    // halves and the output head; the normalised tensor's pixel maxima feed the convolution's window exponents
    Tensor norm_act_conv(const Tensor& x, int side, const Norm& norm, const Lin& conv, int32_t* out = nullptr, const int32_t* residual = nullptr) {
        Tensor y; y.B = x.B; y.T = x.T; y.C = conv.N;
        y.d = out ? out : static_cast<int32_t*>(arena_.alloc(y.n() * 4));
        const size_t scope = arena_.off;
        uint32_t* pix = nullptr;
        const Tensor act = gn_silu(x, norm, pix);
        conv3(act, side, side, conv, 1, y.d, residual, pix);
        arena_.off = scope;
        return y;
    }
    // resnet block (src/engine.cu:389-405 computes the same): two norm-act-conv halves, the second one adding the
    // shortcut -- the input itself, or its 1x1 projection when the width changes
    Tensor res_block(const Tensor& x, int side, const std::string& p) {
        const Lin& second = m_.lin(p + ".conv2");
        Tensor y = talloc(x.B, x.T, second.N);
        const size_t scope = arena_.off;
        const Tensor mid = norm_act_conv(x, side, m_.norm(p + ".norm1"), m_.lin(p + ".conv1"));
        const int32_t* shortcut = m_.has_lin(p + ".conv_shortcut") ? lin_x(x, m_.lin(p + ".conv_shortcut")).d : x.d;
        norm_act_conv(mid, side, m_.norm(p + ".norm2"), second, y.d, shortcut);
        arena_.off = scope;
        return y;
    }
    // the three residual sub-layers of a transformer block, each adding into the running rows h (rows of x, width C)
    void self_attention_into(Tensor& h, const std::string& b, int heads) {
        const QIn n = ln_q(h, m_.norm(b + ".norm1"));
        HeadQ q, k; Tensor v;
        qkv(n, m_.lin(b + ".attn1.to_qkv"), h.C, heads, h.T, q, k, v);
        const Tensor o = attention(q, kv_of(k, v, heads), heads, false, h.T, h.C);
        lin_x(o, m_.lin(b + ".attn1.to_out.0"), h.d, h.d);
    }
    void cross_attention_into(Tensor& h, const std::string& b, int heads, const KV& prompt) {
        const QIn n = ln_q(h, m_.norm(b + ".norm2"));
        const Tensor o = attention(q_only(n, m_.lin(b + ".attn2.to_q"), h.C, heads, h.T), prompt, heads, false, h.T, h.C);
        lin_x(o, m_.lin(b + ".attn2.to_out.0"), h.d, h.d);
    }
    // GEGLU feed-forward; its second GEMM also leaves the row maxima of h for proj_out's quantise-on-load
    void feed_forward_into(Tensor& h, const std::string& b) {
        const QIn n = ln_q(h, m_.norm(b + ".norm3"));
        const Lin& up = m_.lin(b + ".ff.net.0.proj.agi");
        Tensor g; g.B = h.B; g.T = h.T; g.C = up.N / 2;
        g.d = static_cast<int32_t*>(arena_.alloc(g.n() * 4)); g.rowmax = rowmax_alloc(h.B * h.T);
        vela_asrc A; std::memset(&A, 0, sizeof(A)); A.src = VELA_SRC_I8; A.hi = n.hi; A.lo = n.lo; A.ld8 = n.Kp; A.e = n.e;
        vela_aepi E; std::memset(&E, 0, sizeof(E)); E.epi = VELA_EPI_GEGLU; E.Y = g.d; E.ldy = g.C; E.Lphi = m_.lut_phi; E.rowmax = g.rowmax;
        gemm_w8a16(st_, A, n.Mp, n.rows(), up.w, up.Kp, up.Np, up.N, up.Kp, up.cst, E, lo_);
        const Lin& down = m_.lin(b + ".ff.net.2");
        VELA_REQUIRE(down.K == g.C, "ff.net.2: input width differs from the GEGLU output");
        gemm_x(g.d, h.B * h.T, g.C, g.rowmax, down, epi_plain(h.d, h.C, h.d, h.rowmax));
    }
    // transformer block (src/engine.cu:406-454 computes the same): GroupNorm -> proj_in -> the three sub-layers on
    // the rows h -> proj_out + the block input
    Tensor transformer(const Tensor& x, const UNetBlock& blk) {
        Tensor y = talloc(x.B, x.T, x.C);
        const size_t scope = arena_.off;
        Tensor h = talloc(x.B, x.T, x.C);
        h.rowmax = rowmax_alloc(x.B * x.T);
        const std::string b = inner_block(blk);
        auto sublayer = [&](auto&& body) { const size_t m = arena_.off; body(); arena_.off = m; };
        sublayer([&] { lin_q(gn_q(x, m_.norm(blk.name + ".norm")), m_.lin(blk.name + ".proj_in"), h.d); });
        sublayer([&] { self_attention_into(h, b, blk.heads); });
        sublayer([&] { cross_attention_into(h, b, blk.heads, cross_.at(size_t(blk.xattn))); });
        sublayer([&] { feed_forward_into(h, b); });
        lin_x(h, m_.lin(blk.name + ".proj_out"), y.d, x.d);
        arena_.off = scope;
        return y;
    }
    // the UNet (src/engine.cu:455-490): the block table walked in order; kept results live until their resnet on the
    // way up consumes them
    void unet(const Tensor& x, Tensor& eps) {
        int side = 64;
        Tensor h = x;
        std::vector<Tensor> kept;
        for (const UNetBlock& blk : unet_plan()) {
            switch (blk.kind) {
                case BlockKind::ConvIn: h = conv3(h, side, side, m_.lin(blk.name), 1); break;
                case BlockKind::Res:
                    if (blk.pop) {
                        VELA_REQUIRE(!kept.empty(), "unet: no kept tensor for " + blk.name);
                        const Tensor s = kept.back(); kept.pop_back();
                        Tensor cat = talloc(h.B, h.T, h.C + s.C);
                        concat(st_, h.d, h.C, s.d, s.C, h.B * h.T, cat.d);
                        h = cat;
                    }
                    h = res_block(h, side, blk.name);
                    break;
                case BlockKind::Xfmr: h = transformer(h, blk); break;
                case BlockKind::Down: h = conv3(h, side, side, m_.lin(blk.name), 2); side /= 2; break;
                case BlockKind::Up: {
                    Tensor up = talloc(h.B, h.T * 4, h.C);
                    upsample2(st_, h.d, h.B, side, side, h.C, up.d);
                    side *= 2;
                    h = conv3(up, side, side, m_.lin(blk.name), 1);
                    break;
                }
                case BlockKind::Out:
                    h = norm_act_conv(h, side, m_.norm("unet.conv_norm_out"), m_.lin(blk.name), eps.d);
                    break;
            }
            if (blk.push) kept.push_back(h);
            emit(blk.tap, h);
        }
    }
    // Engine::textEncoder (src/engine.cu:491-527), the 77 real rows
    void text_encoder(const std::vector<int32_t>& ids) {
        const int T = 77, D = m_.te_dim;
        VELA_CUDA(cudaMemcpyAsync(dIds_, ids.data(), T * 4, cudaMemcpyHostToDevice, st_));
        Tensor x = talloc(1, T, D);
        text_embed(st_, dIds_, T, T, m_.tok_w, m_.tok_m, m_.tok_s, m_.te_pos, D, x.d);
        for (int l = 0; l < 23; ++l) {
            const std::string p = "te.layers." + std::to_string(l);
            size_t mk = arena_.off;
            QIn n = ln_q(x, m_.norm(p + ".layer_norm1"));
            HeadQ qh, kh; Tensor v;
            qkv(n, m_.lin(p + ".self_attn.qkv"), D, 16, T, qh, kh, v);
            KV kv = kv_of(kh, v, 16);
            Tensor a = attention(qh, kv, 16, true, T, D);
            lin_x(a, m_.lin(p + ".self_attn.out_proj"), x.d, x.d);
            arena_.off = mk;
            QIn n2 = ln_q(x, m_.norm(p + ".layer_norm2"));
            const Lin& L1 = m_.lin(p + ".mlp.fc1");
            Tensor f; f.B = 1; f.T = T; f.C = L1.N; f.d = static_cast<int32_t*>(arena_.alloc(f.n() * 4)); f.rowmax = rowmax_alloc(T);
            vela_asrc A; std::memset(&A, 0, sizeof(A)); A.src = VELA_SRC_I8; A.hi = n2.hi; A.lo = n2.lo; A.ld8 = n2.Kp; A.e = n2.e;
            vela_aepi E = epi_plain(f.d, L1.N, nullptr, f.rowmax); E.epi = VELA_EPI_GELU; E.Lphi = m_.lut_phi;
            gemm_w8a16(st_, A, n2.Mp, T, L1.w, L1.Kp, L1.Np, L1.N, L1.Kp, L1.cst, E, lo_);
            lin_x(f, m_.lin(p + ".mlp.fc2"), x.d, x.d);
            arena_.off = mk;
        }
        const Norm& fn = m_.norm("te.final_layer_norm");
        lnorm(st_, x.d, T, D, fn.g64, fn.beta64, fn.den, dCtx_);
    }
    // Engine::forwardIO (src/engine.cu:599-609)
    // io = false: the step reads dSeeds_[slot] and leaves x0 in dOut_[slot] (device-resident form, launch_device)
    void forward(int slot, bool io = true) {
        if (io) VELA_CUDA(cudaMemcpyAsync(dSeeds_[slot], hSeeds_[slot], size_t(32) * B_, cudaMemcpyHostToDevice, st_));
        arena_.off = 0;
        workspace_ = arena_.alloc(WORKSPACE);
        noise(st_, dSeeds_[slot], B_, nullptr, m_.lut_gauss, m_.c_cin, dNoise_, dX_);
        Tensor x; x.d = dX_; x.B = B_; x.T = 4096; x.C = 4;
        emit("x", x);
        Tensor eps; eps.d = dEps_; eps.B = B_; eps.T = 4096; eps.C = 4;
        unet(x, eps);
        finalize(st_, dNoise_, dEps_, B_, m_.c_sig, dOut_[slot]);
        if (io) {
            VELA_CUDA(cudaMemcpyAsync(hOut_[slot], dOut_[slot], size_t(32768) * B_, cudaMemcpyDeviceToHost, st_));
            VELA_CUDA(cudaMemcpyAsync(hErr_[slot], dErr_, sizeof(unsigned), cudaMemcpyDeviceToHost, st_));
        }
    }
    // a finished step of `slot` whose kernels reported a timed-out wait: reset the word and fail (x0 is not valid)
    void check_step(int slot) {
        const unsigned v = *hErr_[slot];
        if (!v) return;
        *hErr_[slot] = 0;
        VELA_CUDA(cudaMemsetAsync(dErr_, 0, sizeof(unsigned), st_));
        VELA_CUDA(cudaStreamSynchronize(st_));
        throw Error(VELA_ERR_TIMEOUT, "a kernel of the step gave up a bounded wait (device error code " + std::to_string(v) + ")");
    }
    cudaGraphExec_t capture(int slot, bool io) {
        forward(slot, io);
        VELA_CUDA(cudaStreamSynchronize(st_));
        VELA_CUDA(cudaGetLastError());
        cudaGraph_t g = nullptr;
        VELA_CUDA(cudaStreamBeginCapture(st_, cudaStreamCaptureModeThreadLocal));
        try { forward(slot, io); } catch (...) { cudaStreamEndCapture(st_, &g); if (g) cudaGraphDestroy(g); throw; }
        VELA_CUDA(cudaStreamEndCapture(st_, &g));
        size_t n = 0;
        VELA_CUDA(cudaGraphGetNodes(g, nullptr, &n));
        std::vector<cudaGraphNode_t> nodes(n);
        VELA_CUDA(cudaGraphGetNodes(g, nodes.data(), &n));
        int kernels = 0;
        for (size_t i = 0; i < n; ++i) { cudaGraphNodeType t; VELA_CUDA(cudaGraphNodeGetType(nodes[i], &t)); kernels += t == cudaGraphNodeTypeKernel; }
        graph_kernels_ = kernels;
        cudaGraphExec_t ex = nullptr;
        const cudaError_t rc = cudaGraphInstantiate(&ex, g, 0);
        cudaGraphDestroy(g);
        VELA_CUDA(rc);
        return ex;
    }
    // graph per slot: one eager warm-up run, then capture (src/engine.cu:610-631)
    void ensure_slot(int slot) {
        if (ready_[slot]) return;
        if (graph_) gexec_[slot] = capture(slot, true);
        ready_[slot] = true;
    }
    void launch(int slot) {
        if (graph_) VELA_CUDA(cudaGraphLaunch(gexec_[slot], st_));
        else forward(slot);
    }
};
}  // namespace vela

// ------------------------------------------------------------------ C ABI (engine)
using namespace vela;
struct vela_model { Model m; };
struct vela_engine { std::unique_ptr<Engine> e; };

extern "C" vela_model* vela_model_load(int device, const char* path) {
    vela_model* out = nullptr;
    const int rc = guarded("vela_model_load", [&] {
        VELA_REQUIRE(path != nullptr, "null path");
        std::unique_ptr<vela_model> m(new vela_model());
        m->m.load(device, path);
        out = m.release();
    });
    return rc == VELA_OK ? out : nullptr;
}
extern "C" vela_model* vela_model_load_memory(int device, const uint8_t* image, size_t bytes) {
    vela_model* out = nullptr;
    const int rc = guarded("vela_model_load_memory", [&] {
        Poisd f; f.view(image, bytes);
        std::unique_ptr<vela_model> m(new vela_model());
        m->m.load(device, f);
        out = m.release();
    });
    return rc == VELA_OK ? out : nullptr;
}
extern "C" void vela_model_free(vela_model* m) { delete m; }
extern "C" size_t vela_model_bytes(const vela_model* m) { return m ? m->m.bytes : 0; }
extern "C" vela_engine* vela_engine_create(const vela_model* m, const vela_engine_config* cfg) {
    vela_engine* out = nullptr;
    const int rc = guarded("vela_engine_create", [&] {
        VELA_REQUIRE(m && cfg && cfg->batch > 0, "engine_create: model and batch > 0 required");
        std::unique_ptr<vela_engine> e(new vela_engine());
        e->e.reset(new Engine(m->m, cfg->batch, cfg->graph != 0, cfg->arena_bytes));
        out = e.release();
    });
    return rc == VELA_OK ? out : nullptr;
}
extern "C" void vela_engine_destroy(vela_engine* e) { delete e; }
extern "C" int vela_engine_set_prompt(vela_engine* e, const int32_t* tokens, int n) {
    return guarded("vela_engine_set_prompt", [&] { VELA_REQUIRE(e && (tokens || n == 0) && n >= 0, "bad arguments"); e->e->set_prompt(std::vector<int>(tokens, tokens + n)); });
}
extern "C" int vela_engine_context(vela_engine* e, int32_t* ctx) { return guarded("vela_engine_context", [&] { VELA_REQUIRE(e && ctx, "bad arguments"); e->e->context(ctx); }); }
extern "C" int vela_engine_run(vela_engine* e, const uint8_t* seeds, uint8_t* x0) {
    return guarded("vela_engine_run", [&] { VELA_REQUIRE(e && seeds && x0, "bad arguments"); e->e->run(seeds, x0); });
}
extern "C" int vela_engine_submit(vela_engine* e, const uint8_t* seeds) {
    return guarded("vela_engine_submit", [&] { VELA_REQUIRE(e && seeds, "bad arguments"); e->e->submit(seeds); });
}
extern "C" int vela_engine_collect(vela_engine* e, uint8_t* x0) {
    return guarded("vela_engine_collect", [&] { VELA_REQUIRE(e && x0, "bad arguments"); e->e->collect(x0); });
}
extern "C" int vela_engine_step_taps(vela_engine* e, const uint8_t* seeds, uint8_t* x0, vela_tap_fn tap, void* user) {
    return guarded("vela_engine_step_taps", [&] { VELA_REQUIRE(e && seeds && x0, "bad arguments"); e->e->step_taps(seeds, x0, tap, user); });
}
extern "C" int vela_engine_launch_device(vela_engine* e, const uint8_t* d_seeds, uint8_t* d_x0) {
    return guarded("vela_engine_launch_device", [&] { VELA_REQUIRE(e && d_seeds && d_x0, "bad arguments"); e->e->launch_device(d_seeds, d_x0); });
}
extern "C" int vela_engine_graph_kernels(const vela_engine* e) { return e ? e->e->graph_kernels() : 0; }
extern "C" unsigned vela_engine_device_error(vela_engine* e, int clear) {
    if (!e) return 0;
    try { return e->e->device_error(clear != 0); } catch (...) { return 0xFFFFFFFFu; }
}
extern "C" long long vela_engine_test_attention(vela_engine* e, int B, int Tq, int Tk, int heads, int causal, int bits) {
    long long bad = -1;
    const int rc = guarded("vela_engine_test_attention", [&] {
        VELA_REQUIRE(e, "null engine");
        bad = e->e->test_attention(B, Tq, Tk, heads, causal != 0, bits);
    });
    return rc == VELA_OK ? bad : -1;
}
extern "C" int vela_engine_in_flight(const vela_engine* e) { return e ? e->e->in_flight() : 0; }
extern "C" int vela_engine_batch(const vela_engine* e) { return e ? e->e->batch() : 0; }
extern "C" size_t vela_engine_arena_peak(const vela_engine* e) { return e ? e->e->arena_peak() : 0; }
extern "C" void* vela_engine_stream(const vela_engine* e) { return e ? static_cast<void*>(e->e->stream()) : nullptr; }
extern "C" double vela_engine_last_ms(const vela_engine* e) { return e ? e->e->last_ms : 0.0; }
