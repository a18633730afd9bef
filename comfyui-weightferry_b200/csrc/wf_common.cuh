// Shared device helpers of the WeightFerry B200 kernels: the reference's exact rounding steps, half-precision
// loads, cp.async staging and per-device launch geometry.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <atomic>

#include "weightferry_b200.h"

namespace wf {

// ---------------------------------------------------------------------------------------------------- rounding
// rnd<D>(x): float32 -> the nearest value of dtype D, returned as float32 (enhancers/gguf_dequant.py:72-83 _round).
//   float16  : cvt.rn.f16.f32 then back (RNE, subnormals and overflow to inf as the hardware conversion does);
//   bfloat16 : round to nearest even on the bits, (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000 -- the reference's
//              integer form, kept as is so that non-finite inputs give the same bits too;
//   float32  : identity.
template <int D>
__device__ __forceinline__ float rnd(float x);

template <>
__device__ __forceinline__ float rnd<WF_F16>(float x) {
    return __half2float(__float2half_rn(x));
}

template <>
__device__ __forceinline__ float rnd<WF_BF16>(float x) {
    uint32_t u = __float_as_uint(x);
    u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
    return __uint_as_float(u);
}

template <>
__device__ __forceinline__ float rnd<WF_F32>(float x) {
    return x;
}

// bf16 rounding of the fused-block kernels (_r16, enhancers/fused_kernels.py:44-49): the same integer form.
__device__ __forceinline__ float r16(float x) { return rnd<WF_BF16>(x); }

// The float16 stored in the low 16 bits of `bits`, as float32 (exact).
__device__ __forceinline__ float f16_bits_to_f32(uint32_t bits) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits & 0xFFFFu)));
}

// Small non-negative integer (< 2^23) to float32 without the conversion pipe: place it in the mantissa of 2^23
// and subtract 2^23 (exact).
__device__ __forceinline__ float small_u2f(uint32_t v) {
    return __fsub_rn(__uint_as_float(0x4B000000u | v), 8388608.0f);
}

// Signed int8 held in the low byte of `b` (two's complement) to float32, exact: 2^23 + 128 + q, minus the bias.
__device__ __forceinline__ float s8_to_f32(uint32_t b) {
    return __fsub_rn(__uint_as_float(0x4B000000u | ((b ^ 0x80u) & 0xFFu)), 8388736.0f);
}

// ---------------------------------------------------------------------------------------------------- smem reads
// The 8 bytes at an arbitrary shared-memory address p (p 1-aligned), as two little-endian 32-bit words. Reads the
// three aligned words that cover them; the buffer must extend at least 8 bytes past p + 8.
__device__ __forceinline__ uint2 lds8_any(const uint8_t *p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~static_cast<uintptr_t>(3));
    const uint32_t sh = static_cast<uint32_t>(a & 3u) * 8u;
    const uint32_t w0 = w[0], w1 = w[1], w2 = w[2];
    uint2 r;
    r.x = __funnelshift_r(w0, w1, sh);
    r.y = __funnelshift_r(w1, w2, sh);
    return r;
}

// The 16-bit little-endian word at a 2-aligned shared-memory address.
__device__ __forceinline__ uint32_t lds16(const uint8_t *p) {
    return *reinterpret_cast<const uint16_t *>(p);
}

// ---------------------------------------------------------------------------------------------------- cp.async
__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gmem_src) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------------------------------------------- stores
// Eight float32 values already rounded to dtype OUT, written as OUT (16 B for the 2-byte types, 32 B for float32).
// bfloat16 / float16 use the hardware RNE conversion (exact on these values; NaN becomes the canonical NaN, as the
// reference's final `.to(dtype)` does).
template <int OUT, bool VEC>
__device__ __forceinline__ void store8(void *dst, const float x[8]) {
    if constexpr (OUT == WF_BF16) {
        __nv_bfloat162 h[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
        if constexpr (VEC) {
            *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(h);
        } else {
            __nv_bfloat162 *d = reinterpret_cast<__nv_bfloat162 *>(dst);
            const __nv_bfloat16 *hs = reinterpret_cast<const __nv_bfloat16 *>(h);
            __nv_bfloat16 *ds = reinterpret_cast<__nv_bfloat16 *>(d);
#pragma unroll
            for (int i = 0; i < 8; ++i) ds[i] = hs[i];
        }
    } else if constexpr (OUT == WF_F16) {
        __half2 h[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
        if constexpr (VEC) {
            *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(h);
        } else {
            const __half *hs = reinterpret_cast<const __half *>(h);
            __half *ds = reinterpret_cast<__half *>(dst);
#pragma unroll
            for (int i = 0; i < 8; ++i) ds[i] = hs[i];
        }
    } else {
        if constexpr (VEC) {
            float4 *d = reinterpret_cast<float4 *>(dst);
            d[0] = make_float4(x[0], x[1], x[2], x[3]);
            d[1] = make_float4(x[4], x[5], x[6], x[7]);
        } else {
            float *d = reinterpret_cast<float *>(dst);
#pragma unroll
            for (int i = 0; i < 8; ++i) d[i] = x[i];
        }
    }
}

__host__ __device__ constexpr int dtype_size(int d) { return d == WF_F32 ? 4 : 2; }

// ---------------------------------------------------------------------------------------------------- host side
// Streaming multiprocessors of the current device (cached per device).
int device_sm_count();
// Returns WF_OK when the current device is usable (a compute capability 10.x part), else WF_ERR_DEVICE.
int check_device();
// The first character of environment variable `name` as a digit 0-9, else `dflt` (unset, empty or not a digit). The
// kernels' tuning switches are read once per process through this.
int env_digit(const char *name, int dflt);

// Resident CTAs of KERN (threads per CTA, dynamic shared memory) on the whole current device: CTAs per SM times the
// SMs. One cache per kernel (KERN is a template parameter) and device, read and written atomically, since several
// host threads launch (the compute thread and the SSD uploader's); 1 per SM when the query fails.
template <auto KERN>
int wave_ctas(int threads, size_t smem) {
    static std::atomic<int> occ[64];
    int dev = 0;
    cudaGetDevice(&dev);
    int o = (dev >= 0 && dev < 64) ? occ[dev].load(std::memory_order_relaxed) : 0;
    if (o == 0) {
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, KERN, threads, smem) != cudaSuccess || o < 1) o = 1;
        if (dev >= 0 && dev < 64) occ[dev].store(o, std::memory_order_relaxed);
    }
    return o * device_sm_count();
}

}  // namespace wf
