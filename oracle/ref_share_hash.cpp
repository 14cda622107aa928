// Test infrastructure (not product): the reference's own host hashing (src/sha256.h, included from the reference
// checkout by oracle/Makefile) applied to the inputs in argv[1]; writes the digests to argv[2].
//   input:  batch (u32) | seeds [batch][32] | x0 [batch][32768] | headers [batch][80]
//   output: poiOut [batch][32] (src/main.cpp:79) | sha256d(header || poiOut) [batch][32] (src/main.cpp:263-264)
#include "sha256.h"

#include <cstdio>
#include <cstring>
#include <vector>

using namespace meow;

int main(int argc, char** argv) {
    if (argc != 3) return 2;
    FILE* f = std::fopen(argv[1], "rb");
    if (!f) return 3;
    unsigned batch = 0;
    if (std::fread(&batch, 4, 1, f) != 1 || batch == 0 || batch > 1024) return 4;
    std::vector<uint8_t> seeds(size_t(batch) * 32), x0(size_t(batch) * 32768), hdr(size_t(batch) * 80);
    if (std::fread(seeds.data(), 1, seeds.size(), f) != seeds.size() || std::fread(x0.data(), 1, x0.size(), f) != x0.size() ||
        std::fread(hdr.data(), 1, hdr.size(), f) != hdr.size()) return 5;
    std::fclose(f);
    std::vector<uint8_t> out(size_t(batch) * 64);
    for (unsigned b = 0; b < batch; ++b) {
        TaggedHasher h("POI/out");
        h.update(&seeds[b * 32], 32);
        h.update(&x0[size_t(b) * 32768], 32768);
        const auto poi = h.digest();
        uint8_t m[112];
        std::memcpy(m, &hdr[b * 80], 80);
        std::memcpy(m + 80, poi.data(), 32);
        const auto share = sha256d(m, 112);
        std::memcpy(&out[b * 32], poi.data(), 32);
        std::memcpy(&out[(size_t(batch) + b) * 32], share.data(), 32);
    }
    FILE* g = std::fopen(argv[2], "wb");
    if (!g) return 6;
    std::fwrite(out.data(), 1, out.size(), g);
    std::fclose(g);
    return 0;
}
