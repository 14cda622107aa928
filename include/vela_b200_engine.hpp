// C++ engine API over the vela_b200 C ABI, shaped like the reference's engine classes (src/engine.h) so that a
// reference host -- src/main.cpp's runSingle, runBench, mineLane and runVerifyServer -- builds against vela_b200
// unchanged: put include/reference_host/ (whose engine.h includes this header) ahead of the reference's own
// engine.h on the include path and link libvela_b200.so (INTEGRATION.md gives the recipe).  Header-only; it adds no
// behaviour of its own.
//
//   meow::EngineConfig  <- EngineConfig (src/engine.h:55): every field; batch, graph and arenaBytes take effect, the
//                          reference's tuning switches (fusedAttention, customGemmMaxK, fusedLoader, gnFuse,
//                          scoreBytes, gemmWorkspace) are accepted and have no effect here (one kernel per op)
//   meow::DevModel      <- DevModel (src/engine.h:16-37): load(device, parsed POISD) as the reference's hosts call
//                          it (any type with data() returning the file bytes, e.g. meow::Poisd), load(device, path),
//                          the public `bytes` and `device` fields
//   meow::Engine        <- Engine (src/engine.h:57-124): setPrompt, run, submit, collect, inFlight, batch, arenaPeak,
//                          stream, lastMs, testAttention
//
// Errors: the C ABI returns status codes; this layer throws std::runtime_error with vela_last_error(), as the
// reference's engine throws on CUDA and argument errors.
#pragma once
#include "vela_b200.h"

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

namespace meow {

inline void vela_check(int rc) {
    if (rc != VELA_OK) throw std::runtime_error(vela_last_error());
}

struct EngineConfig {
    int batch = 4;
    bool fusedAttention = true;          // accepted, no effect
    int customGemmMaxK = 1536;           // accepted, no effect
    bool fusedLoader = true;             // accepted, no effect
    bool gnFuse = false;                 // accepted, no effect
    size_t arenaBytes = 0;               // 0: 1 GiB + 512 MiB per inference
    size_t scoreBytes = 256u << 20;      // accepted, no effect (no score buffers)
    int gemmWorkspace = 32 << 20;        // accepted, no effect (the split-K workspace lives in the arena)
    bool graph = true;
};

class DevModel {
public:
    DevModel() = default;
    DevModel(const DevModel&) = delete;
    DevModel& operator=(const DevModel&) = delete;
    ~DevModel() { if (m_) vela_model_free(m_); }
    // the reference's form: a POISD model the host has already read (meow::Poisd::data() is the file image)
    template <class ParsedModel>
    auto load(int dev, const ParsedModel& model) -> decltype(model.data().data(), void()) {
        adopt(dev, vela_model_load_memory(dev, reinterpret_cast<const uint8_t*>(model.data().data()), model.data().size()));
    }
    void load(int dev, const std::string& path) { adopt(dev, vela_model_load(dev, path.c_str())); }
    const vela_model* handle() const { return m_; }
    size_t bytes = 0;                    // device bytes of the prepared weights
    int device = 0;

private:
    void adopt(int dev, vela_model* m) {
        if (!m) throw std::runtime_error(vela_last_error());
        if (m_) vela_model_free(m_);
        m_ = m;
        device = dev;
        bytes = vela_model_bytes(m);
    }
    vela_model* m_ = nullptr;
};

class Engine {
public:
    Engine(const DevModel& dm, const EngineConfig& cfg) {
        if (!dm.handle()) throw std::runtime_error("meow::Engine: the model is not loaded");
        vela_engine_config c{cfg.batch, cfg.graph ? 1 : 0, cfg.arenaBytes};
        e_ = vela_engine_create(dm.handle(), &c);
        if (!e_) throw std::runtime_error(vela_last_error());
    }
    Engine(const Engine&) = delete;
    Engine& operator=(const Engine&) = delete;
    ~Engine() { if (e_) vela_engine_destroy(e_); }

    void setPrompt(const std::vector<int>& tokens) {
        std::vector<int32_t> t(tokens.begin(), tokens.end());
        vela_check(vela_engine_set_prompt(e_, t.data(), int(t.size())));
    }
    // seeds: batch x 32 bytes; x0: batch x 32768 bytes (int16 little-endian)
    void run(const uint8_t* seeds, uint8_t* x0) { vela_check(vela_engine_run(e_, seeds, x0)); lastMs = vela_engine_last_ms(e_); }
    void submit(const uint8_t* seeds) { vela_check(vela_engine_submit(e_, seeds)); }
    void collect(uint8_t* x0) { vela_check(vela_engine_collect(e_, x0)); }
    int inFlight() const { return vela_engine_in_flight(e_); }
    int batch() const { return vela_engine_batch(e_); }
    size_t arenaPeak() const { return vela_engine_arena_peak(e_); }
    void* stream() const { return vela_engine_stream(e_); }   // a cudaStream_t
    // mismatching output words of the attention kernel against the exact definition on seeded random data
    long testAttention(int B, int Tq, int Tk, int heads, bool causal, int scaleBits) {
        const long long bad = vela_engine_test_attention(e_, B, Tq, Tk, heads, causal ? 1 : 0, scaleBits);
        if (bad < 0) throw std::runtime_error(vela_last_error());
        return long(bad);
    }
    double lastMs = 0;

private:
    vela_engine* e_ = nullptr;
};

}  // namespace meow
