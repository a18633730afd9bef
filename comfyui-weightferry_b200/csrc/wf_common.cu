// Library-wide entry points (version, status strings) and the per-device facts the launchers size grids with.
#include "wf_common.cuh"

#include <cstdlib>

#include <atomic>

namespace wf {

namespace {
constexpr int kMaxDevices = 64;
std::atomic<int> g_sm[kMaxDevices];   // 0 = not queried yet
std::atomic<int> g_ok[kMaxDevices];   // 0 = not checked, 1 = usable, -1 = not an sm_100 part
}  // namespace

int env_digit(const char *name, int dflt) {
    const char *v = getenv(name);
    return (v != nullptr && v[0] >= '0' && v[0] <= '9') ? v[0] - '0' : dflt;
}

int device_sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
    int n = g_sm[dev].load(std::memory_order_relaxed);
    if (n == 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        g_sm[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

int check_device() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return WF_ERR_DEVICE;
    }
    int ok = g_ok[dev].load(std::memory_order_relaxed);
    if (ok == 0) {
        int major = 0;
        if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) {
            cudaGetLastError();
            return WF_ERR_DEVICE;
        }
        ok = (major == 10) ? 1 : -1;  // the fatbinary holds sm_100a code only
        g_ok[dev].store(ok, std::memory_order_relaxed);
    }
    return ok == 1 ? WF_OK : WF_ERR_DEVICE;
}

}  // namespace wf

extern "C" WF_API int wf_version(void) { return 1 * 10000 + 0 * 100 + 0; }

extern "C" WF_API const char *wf_status_string(int status) {
    switch (status) {
        case WF_OK: return "ok";
        case WF_ERR_ARG: return "invalid argument (size, pointer or dtype outside the contract)";
        case WF_ERR_UNSUPPORTED: return "unsupported type or mode";
        case WF_ERR_SHAPE: return "byte count and value count disagree for this format";
        case WF_ERR_DEVICE: return "no usable sm_100 device is current";
        case WF_ERR_TOO_LARGE: return "problem larger than the library's fixed buffer (no-allocation entry point)";
        default: break;
    }
    if (status > 0) return cudaGetErrorString(static_cast<cudaError_t>(status));
    return "unknown status";
}
