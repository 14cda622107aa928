// Seeded random-init model in the POISDv1 container format.
//
// The reference engine loads one POISD file (format: src/poisd.cpp:17-33 --
// "POISDv1\0", u32 count, then per entry u16 name length, name, u8 dtype
// {0 i8, 1 i16, 2 i32, 3 u8}, u8 ndims, u32 dims[], little-endian data).
// The real sd-turbo-int weights are not available, so bench and parity runs
// use this file: every tensor the reference loader and engine touch
// (src/poisd.cpp:34, src/engine.cu:11-101,389-527) with the SD-2.1 UNet and
// 23-layer text-encoder shapes, int8 weights uniform in [-127, 127] and
// per-channel int32 {m, s, b} whose shift keeps activations near Q16 unity.
// LUTs are synthesised from their definitions (Q16 sigmoid / normal CDF on
// [-16, 16) in 1/64 steps, exp(-z/2^16)*2^30 for z = i*1024, Q16 inverse
// normal CDF for the 65536 noise codes).
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

namespace vela {
namespace {

struct Rng {   // splitmix64, one stream per tensor (name-hashed), so content is order independent
    uint64_t s;
    explicit Rng(uint64_t seed) : s(seed) {}
    uint64_t next() { uint64_t z = (s += 0x9E3779B97F4A7C15ull); z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull; z = (z ^ (z >> 27)) * 0x94D049BB133111EBull; return z ^ (z >> 31); }
    int64_t range(int64_t lo, int64_t hi) { return lo + int64_t(next() % uint64_t(hi - lo + 1)); }   // inclusive
};
uint64_t hashName(const std::string& n, uint64_t seed) {
    uint64_t h = 1469598103934665603ull ^ seed;
    for (unsigned char c : n) { h ^= c; h *= 1099511628211ull; }
    return h;
}

class Writer {
public:
    explicit Writer(FILE* f) : f_(f) {}
    void tensor(const std::string& name, uint8_t dtype, std::vector<uint32_t> dims, const void* data, size_t bytes) {
        uint16_t nl = uint16_t(name.size());
        put(&nl, 2); put(name.data(), nl);
        uint8_t hdr[2] = {dtype, uint8_t(dims.size())}; put(hdr, 2);
        for (uint32_t d : dims) put(&d, 4);
        put(data, bytes);
        ++count_;
    }
    uint32_t count() const { return count_; }
    bool ok() const { return ok_; }
private:
    void put(const void* p, size_t n) { if (n && std::fwrite(p, 1, n, f_) != n) ok_ = false; }
    FILE* f_; uint32_t count_ = 0; bool ok_ = true;
};

struct Gen {
    Writer& w; uint64_t seed;
    void i32(const std::string& name, std::vector<uint32_t> dims, const std::vector<int32_t>& v) { w.tensor(name, 2, dims, v.data(), v.size() * 4); }
    void lin(const std::string& base, int N, int K) {
        Rng r(hashName(base, seed));
        std::vector<int8_t> wt(size_t(N) * K);
        for (size_t i = 0; i < wt.size(); i += 8) {
            uint64_t x = r.next();
            for (int j = 0; j < 8 && i + j < wt.size(); ++j) wt[i + j] = int8_t(int((x >> (8 * j)) & 255) % 255 - 127);
        }
        w.tensor(base + ".w", 0, {uint32_t(N), uint32_t(K)}, wt.data(), wt.size());
        // gain ~1 per layer: y ~ acc * m / 2^(s - e) with acc ~ 2^18.2 sqrt(K) 2^-12 |x| 2^e
        const int sbase = 21 + int(std::floor(0.5 * std::log2(double(K))));
        std::vector<int32_t> m(N), s(N), b(N);
        for (int n = 0; n < N; ++n) { m[n] = int32_t(r.range(16384, 32767)); s[n] = int32_t(sbase + r.range(0, 1)); b[n] = int32_t(r.range(-50000, 50000)); }
        i32(base + ".m", {uint32_t(N)}, m); i32(base + ".s", {uint32_t(N)}, s); i32(base + ".b", {uint32_t(N)}, b);
    }
    void conv(const std::string& base, int N, int C) { lin(base, N, 9 * C); }
    void norm(const std::string& base, int C) {
        Rng r(hashName(base, seed));
        std::vector<int32_t> g(C), beta(C);
        for (int c = 0; c < C; ++c) { g[c] = int32_t(r.range(65536 - 16384, 65536 + 16384)); beta[c] = int32_t(r.range(-8192, 8192)); }
        i32(base + ".g", {uint32_t(C)}, g); i32(base + ".beta", {uint32_t(C)}, beta);
        i32(base + ".eps", {1}, {100000});
    }
    void resnet(const std::string& p, int cin, int cout) {
        norm(p + ".norm1", cin); conv(p + ".conv1", cout, cin); norm(p + ".norm2", cout); conv(p + ".conv2", cout, cout);
        if (cin != cout) lin(p + ".conv_shortcut", cout, cin);
    }
    void transformer(const std::string& p, int C) {
        norm(p + ".norm", C); lin(p + ".proj_in", C, C); lin(p + ".proj_out", C, C);
        const std::string b = p + ".transformer_blocks.0";
        norm(b + ".norm1", C); norm(b + ".norm2", C); norm(b + ".norm3", C);
        lin(b + ".attn1.to_q", C, C); lin(b + ".attn1.to_k", C, C); lin(b + ".attn1.to_v", C, C); lin(b + ".attn1.to_out.0", C, C);
        lin(b + ".attn2.to_q", C, C); lin(b + ".attn2.to_k", C, 1024); lin(b + ".attn2.to_v", C, 1024); lin(b + ".attn2.to_out.0", C, C);
        lin(b + ".ff.net.0.proj.a", 4 * C, C); lin(b + ".ff.net.0.proj.g", 4 * C, C); lin(b + ".ff.net.2", C, 4 * C);
    }
};

double normCdf(double x) { return 0.5 * std::erfc(-x / std::sqrt(2.0)); }
double normInv(double p) {   // bisection on the CDF: deterministic, accurate to the last bit needed for Q16
    double lo = -40, hi = 40;
    for (int i = 0; i < 200; ++i) { double mid = 0.5 * (lo + hi); if (normCdf(mid) < p) lo = mid; else hi = mid; }
    return 0.5 * (lo + hi);
}

}  // namespace

int synthModelWrite(const char* path, uint64_t seed) {
    FILE* f = std::fopen(path, "wb+");
    if (!f) return -1;
    static const char MAGIC[8] = {'P', 'O', 'I', 'S', 'D', 'v', '1', 0};
    uint32_t zero = 0;
    std::fwrite(MAGIC, 1, 8, f); std::fwrite(&zero, 4, 1, f);   // count patched below
    Writer w(f); Gen g{w, seed};
    // ---- UNet (src/engine.cu:455-490) ----
    const int CH[4] = {320, 640, 1280, 1280};
    g.conv("unet.conv_in", 320, 4);
    std::vector<int> skips = {320};
    int h = 320;
    for (int i = 0; i < 4; ++i) {
        for (int j = 0; j < 2; ++j) {
            const std::string p = "unet.down_blocks." + std::to_string(i);
            g.resnet(p + ".resnets." + std::to_string(j), h, CH[i]); h = CH[i];
            if (i < 3) g.transformer(p + ".attentions." + std::to_string(j), CH[i]);
            skips.push_back(h);
        }
        if (i < 3) { g.conv("unet.down_blocks." + std::to_string(i) + ".downsamplers.0.conv", CH[i], CH[i]); skips.push_back(h); }
    }
    g.resnet("unet.mid_block.resnets.0", 1280, 1280); g.transformer("unet.mid_block.attentions.0", 1280); g.resnet("unet.mid_block.resnets.1", 1280, 1280);
    const int UCH[4] = {1280, 1280, 640, 320};
    for (int i = 0; i < 4; ++i) {
        const std::string p = "unet.up_blocks." + std::to_string(i);
        for (int j = 0; j < 3; ++j) {
            const int s = skips.back(); skips.pop_back();
            g.resnet(p + ".resnets." + std::to_string(j), h + s, UCH[i]); h = UCH[i];
            if (i > 0) g.transformer(p + ".attentions." + std::to_string(j), UCH[i]);
        }
        if (i < 3) g.conv(p + ".upsamplers.0.conv", UCH[i], UCH[i]);
    }
    g.norm("unet.conv_norm_out", 320); g.conv("unet.conv_out", 4, 320);
    // ---- text encoder (src/engine.cu:491-527) ----
    {
        const int V = 49408, D = 1024;
        Rng r(hashName("te.tok", seed));
        std::vector<int8_t> tw(size_t(V) * D);
        for (size_t i = 0; i < tw.size(); ++i) tw[i] = int8_t(r.range(-127, 127));
        w.tensor("te.tok.w", 0, {uint32_t(V), uint32_t(D)}, tw.data(), tw.size());
        std::vector<int32_t> tm(V), ts(V), pos(size_t(77) * D);
        for (int v = 0; v < V; ++v) { tm[v] = int32_t(r.range(16384, 32767)); ts[v] = 22; }
        for (auto& p : pos) p = int32_t(r.range(-16384, 16384));
        g.i32("te.tok.m", {uint32_t(V)}, tm); g.i32("te.tok.s", {uint32_t(V)}, ts); g.i32("te.pos", {77, uint32_t(D)}, pos);
        for (int l = 0; l < 23; ++l) {
            const std::string p = "te.layers." + std::to_string(l);
            g.norm(p + ".layer_norm1", D); g.norm(p + ".layer_norm2", D);
            g.lin(p + ".self_attn.q_proj", D, D); g.lin(p + ".self_attn.k_proj", D, D); g.lin(p + ".self_attn.v_proj", D, D); g.lin(p + ".self_attn.out_proj", D, D);
            g.lin(p + ".mlp.fc1", 4 * D, D); g.lin(p + ".mlp.fc2", D, 4 * D);
        }
        g.norm("te.final_layer_norm", D);
    }
    // ---- LUTs and constants (src/poisd.cpp:34, src/intops.cuh:43-57, src/attn.cu:131, src/kernels.cu:585) ----
    {
        std::vector<int32_t> sig(2049), phi(2049), ex(1025), gauss(65536);
        for (int i = 0; i <= 2048; ++i) { const double x = (i - 1024) / 64.0; sig[i] = int32_t(std::lround(65536.0 / (1.0 + std::exp(-x)))); phi[i] = int32_t(std::lround(65536.0 * normCdf(x))); }
        for (int i = 0; i <= 1024; ++i) ex[i] = int32_t(std::lround(1073741824.0 * std::exp(-i / 64.0)));
        for (int u = 0; u < 65536; ++u) gauss[u] = int32_t(std::lround(65536.0 * normInv((u + 0.5) / 65536.0)));
        g.i32("lut.sigmoid", {2049}, sig); g.i32("lut.phi", {2049}, phi); g.i32("lut.exp", {1025}, ex); g.i32("lut.gauss", {65536}, gauss);
        g.i32("c.sig", {1}, {957800});       // sigma_max ~ 14.61 in Q16
        g.i32("c.cin", {1}, {73343000});     // 1/sqrt(sigma^2 + 1) in Q30
        const char vocab[] = "vela-b200 synthetic vocabulary";
        const char merges[] = "vela-b200 synthetic merges";
        w.tensor("tok.vocab", 3, {uint32_t(sizeof vocab - 1)}, vocab, sizeof vocab - 1);
        w.tensor("tok.merges", 3, {uint32_t(sizeof merges - 1)}, merges, sizeof merges - 1);
    }
    const uint32_t cnt = w.count();
    bool ok = w.ok();
    ok = ok && std::fseek(f, 8, SEEK_SET) == 0 && std::fwrite(&cnt, 4, 1, f) == 1;
    ok = (std::fclose(f) == 0) && ok;
    return ok ? 0 : -2;
}
}  // namespace vela
