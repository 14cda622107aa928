// Compile-and-link check of include/vela_b200_engine.hpp against libvela_b200.so (run by tests/test_engine_shim_cpu.py).
// Without a usable model (here: a path that does not exist) DevModel::load must throw, as the reference's loader does.
#include "vela_b200_engine.hpp"

#include <cstdio>

int main(int argc, char** argv) {
    const char* path = argc > 1 ? argv[1] : "/nonexistent/model.poisd";
    meow::DevModel dm;
    try {
        dm.load(0, path);
    } catch (const std::runtime_error& ex) {
        std::printf("load refused: %s\n", ex.what());
        try {
            meow::EngineConfig cfg;
            cfg.batch = 8;
            meow::Engine e(dm, cfg);
        } catch (const std::runtime_error& ex2) {
            std::printf("engine refused: %s\n", ex2.what());
            return 0;
        }
        return 2;
    }
    return 1;
}
