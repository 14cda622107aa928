// vela_quant_v_static: the V-operand quantiser with its column-maximum scratch held in a fixed device array,
// so that the call allocates nothing.
//
// Who needs it: a caller that must not allocate device memory at the moment it quantises V -- a host process
// whose device memory is already committed to its engines' arenas and model copies (the miner and verify-server
// hosts size these to the card), or a caller on a latency-critical path where cudaFree would wait for the whole
// device to go idle and stall the other lanes' steps in flight.  vela_quant_v asks such a caller for a
// u32[G*64] scratch buffer; this entry point uses the library's own instead.
//
// The scratch is one file-scope __device__ array of VELA_QUANT_V_STATIC_MAX_COLS words (256 KiB), which every
// GPU that loads the library holds until the process exits.  In host code its name is only a stand-in for the
// device symbol, never a device address: the first call on each device resolves the address with
// cudaGetSymbolAddress while that device is current, and later calls reuse it.  Every call on a device shares
// the same array and it keeps the last call's contents, so each call clears the G*64 words it uses before the
// column-max kernel runs, and two calls whose work overlaps on the GPU (different streams, or different host
// threads on one device) race on it: such callers must order their calls on one stream.  The resolved address
// belongs to the device's primary context as it was at the first call: a process that resets a device
// (cudaDeviceReset) must not call this entry point on that device again.
#include "ops.h"
#include "status.h"
#include "host_util.h"
#include <mutex>

namespace vela {
namespace {
constexpr int MAX_COLS = VELA_QUANT_V_STATIC_MAX_COLS;
constexpr int MAX_DEVICES = 64;

static __device__ __align__(256) uint32_t g_quant_v_colmax[MAX_COLS];

std::mutex g_setup_mu;
uint32_t* g_colmax_addr[MAX_DEVICES] = {nullptr};

// device address of g_quant_v_colmax on the current device (resolved once per device)
uint32_t* colmax_scratch() {
    const int dev = current_device();
    VELA_REQUIRE(dev >= 0 && dev < MAX_DEVICES, "quant_v_static: device ordinal out of range");
    std::lock_guard<std::mutex> lk(g_setup_mu);
    if (!g_colmax_addr[dev]) {
        uint32_t* p = nullptr;
        VELA_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_quant_v_colmax));
        VELA_REQUIRE(p != nullptr, "quant_v_static: no device address for the scratch array");
        g_colmax_addr[dev] = p;
    }
    return g_colmax_addr[dev];
}
}  // namespace
}  // namespace vela

using namespace vela;

extern "C" int vela_quant_v_static(void* stream, const int32_t* X, int B, int Tk, int C, int heads, int Tkp,
                                   int8_t* vt_hi, int8_t* vt_lo, int32_t* ev, int64_t* vsum) {
    return guarded("vela_quant_v_static", [&] {
        VELA_REQUIRE(B > 0 && heads > 0, "quant_v_static: B and heads must be positive");
        const long long cols = static_cast<long long>(B) * heads * 64;
        if (cols > MAX_COLS)
            throw Error(VELA_ERR_ARG, "quant_v_static: B*heads*64 = " + std::to_string(cols) + " columns exceed the static scratch of " +
                                          std::to_string(MAX_COLS) + " (use vela_quant_v with a caller-provided scratch)");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        // quant_v clears the first B*heads*64 words before its column-max kernel accumulates into them
        quant_v(st, X, B, Tk, C, heads, Tkp, vt_hi, vt_lo, ev, vsum, colmax_scratch());
    });
}
