// Compile-and-link check of include/vela_b200_engine.hpp against libvela_b200.so (run by tests/test_engine_shim_cpu.py),
// in the forms the reference's host uses (src/main.cpp): EngineConfig with every field set, DevModel::load from a
// parsed model and from a path, the public bytes / device fields.  Without a usable model DevModel::load must throw,
// as the reference's loader does.
#include "vela_b200_engine.hpp"

#include <cstdio>
#include <vector>

namespace {
// the shape of the reference's meow::Poisd as DevModel::load uses it: data() is the file image
struct ParsedModel {
    std::vector<uint8_t> image;
    const std::vector<uint8_t>& data() const { return image; }
};
}  // namespace

int main(int argc, char** argv) {
    const char* path = argc > 1 ? argv[1] : "/nonexistent/model.poisd";
    meow::EngineConfig cfg;
    cfg.batch = 8; cfg.graph = true; cfg.fusedAttention = true; cfg.customGemmMaxK = 1536; cfg.fusedLoader = true; cfg.gnFuse = false;
    cfg.scoreBytes = size_t(256) << 20; cfg.arenaBytes = 0; cfg.gemmWorkspace = 32 << 20;
    meow::DevModel dm;
    ParsedModel empty;
    empty.image = {'P', 'O', 'I', 'S', 'D', 'v', '1', 0, 0, 0, 0, 0};     // a valid header holding no tensors
    try {
        dm.load(0, empty);
        return 3;
    } catch (const std::runtime_error& ex) {
        std::printf("image load refused: %s\n", ex.what());
    }
    try {
        dm.load(0, path);
    } catch (const std::runtime_error& ex) {
        std::printf("load refused: %s (bytes %zu, device %d)\n", ex.what(), dm.bytes, dm.device);
        try {
            meow::Engine e(dm, cfg);
        } catch (const std::runtime_error& ex2) {
            std::printf("engine refused: %s\n", ex2.what());
            return 0;
        }
        return 2;
    }
    return 1;
}
