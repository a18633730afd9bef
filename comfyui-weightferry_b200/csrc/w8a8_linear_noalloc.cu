// W8A8 linear with no device allocation: per-token int8 quantisation of bf16 activations followed by the int8 GEMM,
// with the intermediate int8 activations and their scales kept in a fixed buffer that lives inside this library.
//
// Who needs it: some callers cannot allocate device memory at the moment they run a layer -- for example a plugin
// hosted by an application whose own allocator has already reserved the GPU's memory, or a latency-sensitive path
// where a cudaMalloc (which can synchronise the device) is not acceptable. The regular path (wf_quant_rows into
// caller-allocated x_q / x_s, then wf_w8a8_gemm) needs that scratch from the caller; this entry point does not.
//
// The scratch is one file-scope __device__ array of kScratchActs int8 activations plus kScratchRows float32 scales
// (about 16.3 MB). Every GPU that loads this library holds it until the process exits. Its device address is looked
// up with cudaGetSymbolAddress once per device, on the first call made while that device is current (so make that
// first call before any stream capture). All calls share the one buffer and it keeps the last call's contents;
// nothing in it has to start at zero, because the quantiser writes every byte the GEMM then reads. Calls whose
// work overlaps on the GPU (different streams, or different host threads without ordering) race on the buffer.
// The address is kept per device index for the life of the process, so a device reset (cudaDeviceReset) while the
// library is loaded is not supported.

#include "wf_common.cuh"

#include <atomic>
#include <mutex>

namespace {

constexpr int64_t kScratchActs = int64_t(1) << 24;  // int8 activations: m * k <= 16,777,216 (8192 x 2048 fits)
constexpr int64_t kScratchRows = int64_t(1) << 16;  // float32 scales: m <= 65,536 tokens
constexpr int64_t kMaxRowWidth = 51200;             // the quantiser's widest row (k), as wf_quant_rows checks

// [0, kScratchActs): x_q; [kScratchActs, + 4 * kScratchRows): x_s. 256-byte aligned (TMA needs 16).
static __device__ __align__(256) uint8_t g_noalloc_scratch[kScratchActs + 4 * kScratchRows];

constexpr int kMaxDevices = 64;
std::atomic<uintptr_t> g_scratch_addr[kMaxDevices];
std::mutex g_setup_mutex;

// The device address of the scratch on the current device (host code cannot use the symbol itself: its name on the
// host is only a stand-in). Returns WF_OK or an error status.
int scratch_on_current_device(uint8_t **out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return static_cast<int>(e);
    if (dev < 0 || dev >= kMaxDevices) return WF_ERR_DEVICE;
    uintptr_t a = g_scratch_addr[dev].load(std::memory_order_acquire);
    if (a == 0) {
        std::lock_guard<std::mutex> lock(g_setup_mutex);
        a = g_scratch_addr[dev].load(std::memory_order_relaxed);
        if (a == 0) {
            void *p = nullptr;
            e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
            if (e != cudaSuccess || p == nullptr) return e != cudaSuccess ? static_cast<int>(e) : WF_ERR_DEVICE;
            a = reinterpret_cast<uintptr_t>(p);
            g_scratch_addr[dev].store(a, std::memory_order_release);
        }
    }
    *out = reinterpret_cast<uint8_t *>(a);
    return WF_OK;
}

}  // namespace

extern "C" WF_API int wf_w8a8_linear_noalloc(const void *x, const int8_t *wq, const float *ws, void *y, int64_t m,
                                            int64_t n, int64_t k, wf_stream_t stream) {
    if (m < 0 || n < 0 || k <= 0) return WF_ERR_ARG;
    if (m == 0 || n == 0) return WF_OK;
    if (m > kScratchRows || k > kScratchActs / m) return WF_ERR_TOO_LARGE;  // m * k <= kScratchActs, no overflow
    if (k > kMaxRowWidth) return WF_ERR_UNSUPPORTED;  // refused before any launch, as the quantiser would
    if (k % 16 != 0 || n % 8 != 0) return WF_ERR_ARG;  // the GEMM's operand rules, checked before any launch
    int rc = wf::check_device();
    if (rc != WF_OK) return rc;
    uint8_t *scratch = nullptr;
    rc = scratch_on_current_device(&scratch);
    if (rc != WF_OK) return rc;
    int8_t *xq = reinterpret_cast<int8_t *>(scratch);
    float *xs = reinterpret_cast<float *>(scratch + kScratchActs);
    // plain per-token absmax quantisation (no pending operation, no rotation), then the GEMM and its rescale
    rc = wf_quant_rows(x, nullptr, nullptr, nullptr, xq, xs, m, k, 1, 0.0f, 0, 0, stream);
    if (rc != WF_OK) return rc;
    return wf_w8a8_gemm(xq, wq, xs, ws, y, nullptr, m, n, k, stream);
}
