// C++ engine API over the vela_b200 C ABI, shaped like the reference's engine classes so a reference host
// (src/main.cpp) can switch to vela_b200 by including this header in place of src/engine.h and linking
// libvela_b200.so.  Header-only; it adds no behaviour of its own.
//
//   meow::EngineConfig  <- EngineConfig (src/engine.h): batch, graph, arenaBytes (its other fields have no effect here)
//   meow::DevModel      <- DevModel (src/engine.h:16-40); load() takes the POISD file path instead of a parsed Poisd
//   meow::Engine        <- Engine (src/engine.h:42-124): setPrompt, run, submit, collect, inFlight, batch,
//                          arenaPeak, stream, lastMs
//
// Errors: the C ABI returns status codes; this layer throws std::runtime_error with vela_last_error(), as the
// reference's engine throws on CUDA and argument errors.
#pragma once
#include "vela_b200.h"

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
    bool graph = true;
    size_t arenaBytes = 0;      // 0: 1 GiB + 512 MiB per inference
};

class DevModel {
public:
    DevModel() = default;
    DevModel(const DevModel&) = delete;
    DevModel& operator=(const DevModel&) = delete;
    ~DevModel() { if (m_) vela_model_free(m_); }
    void load(int device, const std::string& path) {
        vela_model* m = vela_model_load(device, path.c_str());
        if (!m) throw std::runtime_error(vela_last_error());
        if (m_) vela_model_free(m_);
        m_ = m;
        device_ = device;
    }
    const vela_model* handle() const { return m_; }
    size_t bytes() const { return m_ ? vela_model_bytes(m_) : 0; }
    int device() const { return device_; }

private:
    vela_model* m_ = nullptr;
    int device_ = 0;
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

    void setPrompt(const std::vector<int32_t>& tokens) { vela_check(vela_engine_set_prompt(e_, tokens.data(), int(tokens.size()))); }
    // seeds: batch x 32 bytes; x0: batch x 32768 bytes (int16 little-endian)
    void run(const uint8_t* seeds, uint8_t* x0) { vela_check(vela_engine_run(e_, seeds, x0)); lastMs = vela_engine_last_ms(e_); }
    void submit(const uint8_t* seeds) { vela_check(vela_engine_submit(e_, seeds)); }
    void collect(uint8_t* x0) { vela_check(vela_engine_collect(e_, x0)); }
    int inFlight() const { return vela_engine_in_flight(e_); }
    int batch() const { return vela_engine_batch(e_); }
    size_t arenaPeak() const { return vela_engine_arena_peak(e_); }
    void* stream() const { return vela_engine_stream(e_); }   // a cudaStream_t
    double lastMs = 0;

private:
    vela_engine* e_ = nullptr;
};

}  // namespace meow
