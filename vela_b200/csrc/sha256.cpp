// Host share hashing of the reference's mining / verify path (src/main.cpp:79,139,262-264; src/sha256.h:84-91):
//   poi_out(seed, x0)  = SHA-256(SHA-256("POI/out") || SHA-256("POI/out") || seed[32] || x0[32768])   (tagged hash)
//   share(header, poi) = SHA-256(SHA-256(header[80] || poi[32]))                                       (sha256d)
// SHA-256 itself is FIPS 180-4.  The round constants and the initial state are derived here from their definition
// (the first 32 fraction bits of the cube roots of the first 64 primes and of the square roots of the first 8),
// with exact integer roots, once at start-up.
//
// This stays on the host: at B200 rates one GPU produces about 232 x 32 KiB = 7.6 MB of x0 per second, a few
// percent of one core for a portable SHA-256; vela_poi_out_batch spreads a batch over threads.
#include "status.h"
#include "vela_b200.h"

#include <algorithm>

#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace vela {
namespace {

typedef unsigned __int128 u128;

uint64_t icbrt(u128 v) {            // floor(cbrt(v)) for v < 2^120
    uint64_t lo = 0, hi = uint64_t(1) << 40;
    while (lo < hi) {
        const uint64_t mid = lo + (hi - lo + 1) / 2;
        if (u128(mid) * mid * mid <= v) lo = mid; else hi = mid - 1;
    }
    return lo;
}
uint64_t isqrt128(u128 v) {         // floor(sqrt(v)) for v < 2^120
    uint64_t lo = 0, hi = uint64_t(1) << 60;
    while (lo < hi) {
        const uint64_t mid = lo + (hi - lo + 1) / 2;
        if (u128(mid) * mid <= v) lo = mid; else hi = mid - 1;
    }
    return lo;
}

struct Tables {
    uint32_t k[64], h0[8];
    Tables() {
        int primes[64], n = 0;
        for (int c = 2; n < 64; ++c) {
            bool p = true;
            for (int d = 2; d * d <= c; ++d) if (c % d == 0) { p = false; break; }
            if (p) primes[n++] = c;
        }
        for (int i = 0; i < 64; ++i) k[i] = uint32_t(icbrt(u128(primes[i]) << 96));      // frac(cbrt p) * 2^32
        for (int i = 0; i < 8; ++i) h0[i] = uint32_t(isqrt128(u128(primes[i]) << 64));    // frac(sqrt p) * 2^32
    }
};
const Tables& tables() { static const Tables t; return t; }

inline uint32_t rotr(uint32_t x, int r) { return (x >> r) | (x << (32 - r)); }

class Sha256 {
public:
    Sha256() { std::memcpy(h_, tables().h0, sizeof(h_)); }
    void update(const uint8_t* p, size_t n) {
        bytes_ += n;
        if (fill_) {
            const size_t t = std::min(n, size_t(64) - fill_);
            std::memcpy(buf_ + fill_, p, t); fill_ += t; p += t; n -= t;
            if (fill_ == 64) { block(buf_); fill_ = 0; }
        }
        for (; n >= 64; p += 64, n -= 64) block(p);
        if (n) { std::memcpy(buf_, p, n); fill_ = n; }
    }
    void digest(uint8_t out[32]) {
        const uint64_t bits = bytes_ * 8;
        const uint8_t pad = 0x80;
        update(&pad, 1);
        const uint8_t zero[64] = {0};
        update(zero, fill_ <= 56 ? 56 - fill_ : 120 - fill_);
        uint8_t len[8];
        for (int i = 0; i < 8; ++i) len[i] = uint8_t(bits >> (56 - 8 * i));
        update(len, 8);
        for (int i = 0; i < 8; ++i) for (int j = 0; j < 4; ++j) out[4 * i + j] = uint8_t(h_[i] >> (24 - 8 * j));
    }

private:
    void block(const uint8_t* p) {
        const uint32_t* K = tables().k;
        uint32_t w[64];
        for (int i = 0; i < 16; ++i) w[i] = uint32_t(p[4 * i]) << 24 | uint32_t(p[4 * i + 1]) << 16 | uint32_t(p[4 * i + 2]) << 8 | p[4 * i + 3];
        for (int i = 16; i < 64; ++i) {
            const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
            const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
            w[i] = w[i - 16] + s0 + w[i - 7] + s1;
        }
        uint32_t a = h_[0], b = h_[1], c = h_[2], d = h_[3], e = h_[4], f = h_[5], g = h_[6], h = h_[7];
        for (int i = 0; i < 64; ++i) {
            const uint32_t t1 = h + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + K[i] + w[i];
            const uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
            h = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
        }
        h_[0] += a; h_[1] += b; h_[2] += c; h_[3] += d; h_[4] += e; h_[5] += f; h_[6] += g; h_[7] += h;
    }
    uint32_t h_[8];
    uint8_t buf_[64];
    size_t fill_ = 0;
    uint64_t bytes_ = 0;
};

void sha256(const uint8_t* p, size_t n, uint8_t out[32]) { Sha256 s; s.update(p, n); s.digest(out); }

void poi_out(const uint8_t* seed, const uint8_t* x0, uint8_t out[32]) {
    static const char tag[] = "POI/out";
    uint8_t t[32];
    sha256(reinterpret_cast<const uint8_t*>(tag), sizeof(tag) - 1, t);
    Sha256 s;
    s.update(t, 32); s.update(t, 32); s.update(seed, 32); s.update(x0, 32768);
    s.digest(out);
}

}  // namespace
}  // namespace vela

using namespace vela;

extern "C" int vela_sha256d(const uint8_t* data, size_t n, uint8_t* out32) {
    return guarded_host("vela_sha256d", [&] {
        VELA_REQUIRE(out32 && (data || n == 0), "sha256d: null pointer");
        uint8_t h[32];
        sha256(data, n, h);
        sha256(h, 32, out32);
    });
}

extern "C" int vela_poi_out(const uint8_t* seed32, const uint8_t* x0, uint8_t* out32) {
    return guarded_host("vela_poi_out", [&] {
        VELA_REQUIRE(seed32 && x0 && out32, "poi_out: null pointer");
        poi_out(seed32, x0, out32);
    });
}

extern "C" int vela_poi_out_batch(const uint8_t* seeds, const uint8_t* x0, int batch, int threads, uint8_t* out) {
    return guarded_host("vela_poi_out_batch", [&] {
        VELA_REQUIRE(seeds && x0 && out && batch > 0, "poi_out_batch: bad arguments");
        const int nt = std::max(1, std::min(threads, batch));
        if (nt == 1) {
            for (int b = 0; b < batch; ++b) poi_out(seeds + 32 * size_t(b), x0 + 32768 * size_t(b), out + 32 * size_t(b));
            return;
        }
        std::vector<std::thread> pool;
        for (int t = 0; t < nt; ++t)
            pool.emplace_back([=] {
                for (int b = t; b < batch; b += nt) poi_out(seeds + 32 * size_t(b), x0 + 32768 * size_t(b), out + 32 * size_t(b));
            });
        for (auto& th : pool) th.join();
    });
}

extern "C" int vela_share_hash(const uint8_t* header80, const uint8_t* poi32, uint8_t* out32) {
    return guarded_host("vela_share_hash", [&] {
        VELA_REQUIRE(header80 && poi32 && out32, "share_hash: null pointer");
        uint8_t m[112], h[32];
        std::memcpy(m, header80, 80); std::memcpy(m + 80, poi32, 32);
        sha256(m, 112, h);
        sha256(h, 32, out32);
    });
}
