// Host-side pieces of the C ABI: error reporting, version, model tooling.
#include "vela_b200.h"
#include "status.h"
#include <string>

namespace vela {
int synthModelWrite(const char* path, uint64_t seed);
static thread_local std::string g_lastError;
void setError(const std::string& msg) { g_lastError = msg; }
}  // namespace vela

extern "C" const char* vela_last_error(void) { return vela::g_lastError.c_str(); }
extern "C" const char* vela_version(void) { return "vela_b200 0.1 (sm_100a)"; }

extern "C" int vela_synth_model_write(const char* path, uint64_t seed) {
    if (!path) return vela::fail(VELA_ERR_ARG, "synth_model_write: null path");
    const int rc = vela::synthModelWrite(path, seed);
    if (rc == -1) return vela::fail(VELA_ERR_IO, std::string("synth_model_write: cannot open ") + path);
    if (rc != 0) return vela::fail(VELA_ERR_IO, std::string("synth_model_write: write failed for ") + path);
    return VELA_OK;
}
