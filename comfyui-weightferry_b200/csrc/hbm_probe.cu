// Measurement helper for the benchmark: the HBM rate a plain streaming kernel reaches for a given read : write byte
// mix. The dequantisation reads packed blocks and writes about 3.6 times as many bytes; the measured copy bandwidth
// (read = write) overstates what HBM sustains for such write-heavy traffic, so the benchmark times this probe over
// the same buffers and byte counts and reports it beside the copy-based roofline.
//
// out[j] = in[floor(j * r)] ^ j for every 16-byte unit j of the output, r = n_in / n_out rounded down to a 32.32
// fixed-point number (so the input index never reaches n_in). The structure of the dequantisation without its
// arithmetic: a CTA takes 2048 output units at a time, stages the input units they need (each read from DRAM once,
// coalesced) in shared memory, and writes the 2048 units with coalesced 16-byte stores; CTAs of 256 threads, about
// four tiles each.

#include "wf_common.cuh"

#include <algorithm>

namespace wf {
namespace {

constexpr int kTileOut = 2048;  // output units per tile; its input range has at most kTileOut + 1 units (r <= 1)

__global__ void __launch_bounds__(256) hbm_probe_kernel(const uint4 *__restrict__ in, int64_t n_in,
                                                        uint64_t ratio_fp, uint4 *__restrict__ out, int64_t n_out) {
    __shared__ uint4 tile[kTileOut + 1];
    const int64_t n_tiles = (n_out + kTileOut - 1) / kTileOut;
    for (int64_t t = blockIdx.x; t < n_tiles; t += gridDim.x) {
        const int64_t j0 = t * kTileOut, j1 = min(j0 + kTileOut, n_out);  // output units [j0, j1)
        // j < 2^31 and ratio_fp < 2^32: the products fit 64 bits; every index is <= j * n_in / n_out < n_in
        const int64_t a = static_cast<int64_t>((static_cast<uint64_t>(j0) * ratio_fp) >> 32);
        const int64_t b = static_cast<int64_t>((static_cast<uint64_t>(j1 - 1) * ratio_fp) >> 32);  // inclusive
        for (int64_t i = a + threadIdx.x; i <= b; i += 256) tile[i - a] = __ldg(in + i);
        __syncthreads();
#pragma unroll 4
        for (int64_t j = j0 + threadIdx.x; j < j1; j += 256) {
            const uint4 v = tile[static_cast<int64_t>((static_cast<uint64_t>(j) * ratio_fp) >> 32) - a];
            out[j] = make_uint4(v.x ^ static_cast<uint32_t>(j), v.y, v.z, v.w);
        }
        __syncthreads();  // the tile is overwritten by the next one
    }
}

}  // namespace
}  // namespace wf

extern "C" WF_API int wf_hbm_probe(const void *in, int64_t in_bytes, void *out, int64_t out_bytes,
                                  wf_stream_t stream) {
    if (!in || !out || in_bytes <= 0 || out_bytes <= 0 || in_bytes % 16 || out_bytes % 16) return WF_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) % 16) return WF_ERR_ARG;
    const int64_t n_in = in_bytes / 16, n_out = out_bytes / 16;
    if (n_in >= (int64_t(1) << 31) || n_out >= (int64_t(1) << 31)) return WF_ERR_TOO_LARGE;
    int rc = wf::check_device();
    if (rc != WF_OK) return rc;
    if (n_in > n_out) return WF_ERR_ARG;  // the probe models reads at most as large as writes (ratio_fp <= 2^32)
    const uint64_t ratio_fp = (static_cast<uint64_t>(n_in) << 32) / static_cast<uint64_t>(n_out);  // n_in < 2^31
    // about four tiles per CTA, never fewer CTAs than fit at once (the dequantisation kernels' grid rule: the HBM
    // sustains more of a write-heavy mix with many short-lived CTAs than with one persistent wave)
    const int64_t n_tiles = (n_out + wf::kTileOut - 1) / wf::kTileOut;
    const int64_t resident = wf::wave_ctas<wf::hbm_probe_kernel>(256, 0);
    const int grid = static_cast<int>(std::min<int64_t>(n_tiles, std::max<int64_t>(resident, (n_tiles + 3) / 4)));
    wf::hbm_probe_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4 *>(in), n_in, ratio_fp, static_cast<uint4 *>(out), n_out);
    return static_cast<int>(cudaGetLastError());
}
