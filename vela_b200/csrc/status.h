// Status-code plumbing shared by every C-ABI entry point.
#pragma once
#include "vela_b200.h"
#include <cuda_runtime.h>
#include <stdexcept>
#include <string>

namespace vela {
void setError(const std::string& msg);
inline int fail(int code, const std::string& msg) { setError(msg); return code; }

// Exception carrying a C-ABI status; thrown inside the library, turned into a return code at the boundary.
struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};
#define VELA_CUDA(x) do { cudaError_t _e = (x); if (_e != cudaSuccess) \
    throw ::vela::Error(VELA_ERR_CUDA, std::string("CUDA error ") + cudaGetErrorString(_e) + " at " #x " (" __FILE__ ":" + std::to_string(__LINE__) + ")"); } while (0)
#define VELA_REQUIRE(cond, msg) do { if (!(cond)) throw ::vela::Error(VELA_ERR_ARG, std::string(msg)); } while (0)

// Run `body` and map exceptions to status codes; a kernel-launch error is checked (without synchronising).
template <class F> int guarded(const char* what, F&& body) {
    try {
        body();
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return fail(VELA_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
        return VELA_OK;
    } catch (const Error& ex) {
        return fail(ex.code, std::string(what) + ": " + ex.what());
    } catch (const std::exception& ex) {
        return fail(VELA_ERR_ARG, std::string(what) + ": " + ex.what());
    }
}
// The same for host-only entries (no CUDA state is touched or queried).
template <class F> int guarded_host(const char* what, F&& body) {
    try {
        body();
        return VELA_OK;
    } catch (const Error& ex) {
        return fail(ex.code, std::string(what) + ": " + ex.what());
    } catch (const std::exception& ex) {
        return fail(VELA_ERR_ARG, std::string(what) + ": " + ex.what());
    }
}
}  // namespace vela
