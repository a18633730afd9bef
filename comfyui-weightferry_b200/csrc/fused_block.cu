// Fused Cosmos / Anima block prologue kernels for sm_100a: modulate, LayerNorm + modulate (kernel A), RMSNorm-128,
// RMSNorm-128 + split-half 3D RoPE (kernel B), and the per-token int8 row quantiser of the W8A8 linear.
//
// Arithmetic follows the reference's Triton kernels operation by operation (enhancers/fused_kernels.py,
// enhancers/sage_fused.py): every bf16 rounding where the reference rounds (_r16), the same summation orders (the
// Welford order of PyTorch's vectorized layer norm, the lane trees of the RMS sums), fused multiply-adds exactly
// where the reference writes them, and the same hardware approximations (rsqrt.approx.f32, and the approximate
// float32 division Triton emits for `/`). All memory-bound: one read of the activations, one write.
//
// Data layout: rows of bf16, contiguous. A row of the layer-norm / quantiser kernels is one CTA of 128 threads,
// thread t holding the 4-value vectors t, t + 128, ... of the row (PyTorch's layout, which fixes the Welford order);
// the RMS kernels put one row of 128 on one warp.

#include "wf_common.cuh"

#include <atomic>

#include <algorithm>
#include <cstdlib>

namespace wf {
namespace {

// ------------------------------------------------------------------------------------------------- helpers
// The quantisers feed the int8 GEMM, which is launched as a programmatic dependent: signalling at the start of every
// CTA lets the GEMM's CTAs be launched (and do their set-up) as soon as all quantiser CTAs are running; the GEMM waits
// for this grid's completion and memory before it reads anything (griddepcontrol.wait). No effect on other launches.
__device__ __forceinline__ void allow_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float rsqrt_approx(float v) {
    float r;
    asm("rsqrt.approx.f32 %0, %1;" : "=f"(r) : "f"(v));
    return r;
}

// Triton's float32 `/` (the reference's quantiser divides with it): the full-range approximate division.
__device__ __forceinline__ float div_full(float a, float b) {
    float r;
    asm("div.full.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// Two float32 lanes in one 64-bit register and Blackwell's packed float32 arithmetic on them: each lane is rounded
// exactly as the scalar instruction rounds it (IEEE round to nearest), so a pair of scalar operations and one packed
// one give the same bits -- in half the instructions.
__device__ __forceinline__ uint64_t f2pack(float lo, float hi) {
    return (static_cast<uint64_t>(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ float f2lo(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float f2hi(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v >> 32)); }
__device__ __forceinline__ uint64_t bf_pair(uint32_t w) {  // the two bf16 of a word as float32 lanes (exact)
    return (static_cast<uint64_t>(w & 0xFFFF0000u) << 32) | (w << 16);
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// packed bf16 pairs: absolute value, maximum and minimum of each lane (exact; max / min return the other operand
// when one is NaN, as fmaxf / fminf do)
__device__ __forceinline__ uint32_t bf2_abs(uint32_t a) {
    uint32_t d;
    asm("abs.bf16x2 %0, %1;" : "=r"(d) : "r"(a));
    return d;
}
__device__ __forceinline__ uint32_t bf2_max(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t bf2_min(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("min.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// four bf16 (8 bytes) -> float
__device__ __forceinline__ void unpack4(uint2 w, float v[4]) {
    v[0] = bf_lo(w.x);
    v[1] = bf_hi(w.x);
    v[2] = bf_lo(w.y);
    v[3] = bf_hi(w.y);
}

// two floats -> packed bf16 pair (RNE; equal to the reference's bit-level rounding on every non-NaN value)
__device__ __forceinline__ uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}

__device__ __forceinline__ float load_w(const void *w, int wdt, int i) {
    if (wdt == WF_BF16) return __bfloat162float(static_cast<const __nv_bfloat16 *>(w)[i]);
    if (wdt == WF_F16) return __half2float(static_cast<const __half *>(w)[i]);
    return static_cast<const float *>(w)[i];
}

// bf16(bf16(n * s) + h) for bf16 pairs: the product of two bf16 values is exact in float32, so one bf16 rounding of it
// (mul.rn.bf16x2) is the reference's float product rounded to bf16; float32 holds at least 2 * 8 + 2 bits, so the
// float sum of two bf16 values rounded to bf16 is the correctly rounded bf16 sum (add.rn.bf16x2). The _rn forms keep
// the compiler from contracting the two into one fma, which would round once instead of twice.
__device__ __forceinline__ uint32_t mod_bf16x2(uint32_t n, uint32_t s, uint32_t h) {
    const __nv_bfloat162 t = __hmul2_rn(*reinterpret_cast<const __nv_bfloat162 *>(&n),
                                        *reinterpret_cast<const __nv_bfloat162 *>(&s));
    const __nv_bfloat162 o = __hadd2_rn(t, *reinterpret_cast<const __nv_bfloat162 *>(&h));
    return *reinterpret_cast<const uint32_t *>(&o);
}

// ------------------------------------------------------------------------------------------------- modulate
// out = R16(R16(x * s1) + shift) (fused_kernels.py:51-62 _mod), 8 values per thread, grid-stride. d % 8 == 0.
__global__ void __launch_bounds__(256) modulate_kernel(const uint4 *__restrict__ x, const __nv_bfloat16 *__restrict__ s1,
                                                       const __nv_bfloat16 *__restrict__ sh, uint4 *__restrict__ out,
                                                       int64_t n_vec, int64_t d, int64_t rows_per_group) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n_vec; i += stride) {
        const int64_t e = i * 8;
        const int64_t row = e / d, col = e - row * d;
        const int64_t goff = (row / rows_per_group) * d + col;
        const uint4 xv = __ldg(x + i);
        const uint4 sv = __ldg(reinterpret_cast<const uint4 *>(s1 + goff));
        const uint4 hv = __ldg(reinterpret_cast<const uint4 *>(sh + goff));
        out[i] = make_uint4(mod_bf16x2(xv.x, sv.x, hv.x), mod_bf16x2(xv.y, sv.y, hv.y), mod_bf16x2(xv.z, sv.z, hv.z),
                            mod_bf16x2(xv.w, sv.w, hv.w));
    }
}

// ------------------------------------------------------------------------------------------------- gated residual
// out = bf16_rn(x + f32(gate * o)) -- PyTorch's bf16 addcmul(x, gate, o) (one float32 product, one float32 sum, one
// rounding), the block's residual update (fused_block.py:527-532 _add_residual). gate row (row / rows_per_group),
// 8 values per thread, grid-stride; out may be x. d % 8 == 0.
__global__ void __launch_bounds__(256) gated_residual_kernel(const uint4 *__restrict__ x,
                                                             const __nv_bfloat16 *__restrict__ gate,
                                                             const uint4 *__restrict__ o, uint4 *out, int64_t n_vec,
                                                             int64_t d, int64_t rows_per_group) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n_vec; i += stride) {
        const int64_t e = i * 8;
        const int64_t row = e / d, col = e - row * d;
        const uint4 xv = x[i];  // plain load: out may alias x
        const uint4 ov = __ldg(o + i);
        const uint4 gv = __ldg(reinterpret_cast<const uint4 *>(gate + (row / rows_per_group) * d + col));
        const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w}, os[4] = {ov.x, ov.y, ov.z, ov.w},
                       gs[4] = {gv.x, gv.y, gv.z, gv.w};
        uint32_t r[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
            r[k] = pack2(__fadd_rn(bf_lo(xs[k]), __fmul_rn(bf_lo(gs[k]), bf_lo(os[k]))),
                         __fadd_rn(bf_hi(xs[k]), __fmul_rn(bf_hi(gs[k]), bf_hi(os[k]))));
        out[i] = make_uint4(r[0], r[1], r[2], r[3]);
    }
}

// ------------------------------------------------------------------------------------------------- Welford
struct Welford {
    float m, s, c;
};

// _wcombine (fused_kernels.py:84-93): own = the lower lane / warp, oth = the one merged into it
__device__ __forceinline__ Welford wcombine(Welford own, Welford oth) {
    const float delta = __fsub_rn(own.m, oth.m);
    const float count = __fadd_rn(oth.c, own.c);
    const float coef = __fdiv_rn(1.0f, count);
    const float n_a = __fmul_rn(oth.c, coef);
    const float n_b = __fmul_rn(own.c, coef);
    Welford r;
    r.m = __fmaf_rn(n_a, oth.m, __fmul_rn(n_b, own.m));
    r.s = __fmaf_rn(__fmul_rn(__fmul_rn(delta, delta), oth.c), n_b, __fadd_rn(oth.s, own.s));
    r.c = count;
    return r;
}

// PyTorch's vectorized layer-norm statistics of one row, as _ln_stats reproduces them (fused_kernels.py:106-135):
// each thread's Welford state over its values (in its vector order), then shuffle-down merges 16 .. 1, then warps
// 2, 3 into 0, 1 and 1 into 0 (ln_merge_n below); (mean, sigma2 / K) to every thread of the 128.
//
// One Welford update (fused_kernels.py:118-121: delta = v - m, c += 1, m = fma(delta, 1 / c, m),
// s = fma(delta, v - m, s)) when this is the thread's i-th value (i = 0, 1, ...): the count is i + 1 for every
// thread, so the correctly rounded 1 / count comes from a table (the host's IEEE division of 1 by i + 1: the same
// bits as div.rn).
struct RcpTable {
    float v[64];
};
constexpr RcpTable make_rcp() {
    RcpTable t{};
    for (int i = 0; i < 64; ++i) t.v[i] = 1.0f / static_cast<float>(i + 1);
    return t;
}
__constant__ RcpTable c_rcp = make_rcp();

__device__ __forceinline__ void welford_step_i(Welford &w, float v, int i) {
    const float delta = __fsub_rn(v, w.m);
    w.c = static_cast<float>(i + 1);
    w.m = __fmaf_rn(delta, c_rcp.v[i], w.m);
    w.s = __fmaf_rn(delta, __fsub_rn(v, w.m), w.s);
}

// bf16 rounding of a pair through the packed RNE conversion (the same value as the bit-level rounding on every
// non-NaN input)
__device__ __forceinline__ float2 r16x2(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    const uint32_t u = *reinterpret_cast<const uint32_t *>(&h);
    return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xFFFF0000u));
}

__device__ __forceinline__ void ln_merge(Welford w, int64_t K, float &mu, float &var, float *red);


// wcombine of two states that each hold C values: the count C + C and its correctly rounded reciprocal are
// compile-time constants (C is the same in every lane), so the division of the merge becomes a product
template <int C>
__device__ __forceinline__ Welford wcombine_n(Welford own, Welford oth) {
    constexpr float count = static_cast<float>(2 * C);
    constexpr float coef = 1.0f / count;  // evaluated at compile time in IEEE arithmetic: div.rn's value
    constexpr float c_one = static_cast<float>(C);  // both states hold C values
    constexpr float nab = c_one * coef;              // each side's weight, in IEEE arithmetic as at run time
    const float delta = __fsub_rn(own.m, oth.m);
    Welford r;
    r.m = __fmaf_rn(nab, oth.m, __fmul_rn(nab, own.m));
    r.s = __fmaf_rn(__fmul_rn(__fmul_rn(delta, delta), c_one), nab, __fadd_rn(oth.s, own.s));
    r.c = count;
    return r;
}

template <int N>  // values per thread (4 * K / 512)
__device__ __forceinline__ void ln_merge_n(Welford w, int64_t K, float &mu, float &var, float *red) {
#define WF_SHFL_MERGE(OFF, C)                                   \
    {                                                           \
        Welford o;                                              \
        o.m = __shfl_down_sync(0xFFFFFFFFu, w.m, OFF);          \
        o.s = __shfl_down_sync(0xFFFFFFFFu, w.s, OFF);          \
        o.c = static_cast<float>(C);  /* the same in every lane */ \
        w = wcombine_n<C>(w, o);                                \
    }
    WF_SHFL_MERGE(16, N) WF_SHFL_MERGE(8, 2 * N) WF_SHFL_MERGE(4, 4 * N) WF_SHFL_MERGE(2, 8 * N)
    WF_SHFL_MERGE(1, 16 * N)
#undef WF_SHFL_MERGE
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        red[warp * 3 + 0] = w.m;
        red[warp * 3 + 1] = w.s;
        red[warp * 3 + 2] = w.c;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        Welford w0{red[0], red[1], red[2]}, w1{red[3], red[4], red[5]}, w2{red[6], red[7], red[8]},
            w3{red[9], red[10], red[11]};
        w0 = wcombine_n<32 * N>(w0, w2);
        w1 = wcombine_n<32 * N>(w1, w3);
        w0 = wcombine_n<64 * N>(w0, w1);
        red[12] = w0.m;
        red[13] = __fdiv_rn(w0.s, static_cast<float>(K));
    }
    __syncthreads();
    mu = red[12];
    var = red[13];
}

template <int N>
__device__ __forceinline__ void ln_stats_n(const float *v, int64_t K, float &mu, float &var, float *red) {
    Welford w{0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < N; ++i) welford_step_i(w, v[i], i);
    ln_merge_n<N>(w, K, mu, var, red);
}

__device__ __forceinline__ void ln_stats(const float *v, int nv, int64_t K, float &mu, float &var, float *red) {
    Welford w{0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < nv; ++i) welford_step_i(w, v[i], i);
    ln_merge(w, K, mu, var, red);
}

// the same statistics with this thread's nvec vectors of 4 in shared memory at p, p + 512, ... (floats)
__device__ __forceinline__ void ln_stats_strided(const float *p, int nvec, int64_t K, float &mu, float &var,
                                                 float *red) {
    Welford w{0.f, 0.f, 0.f};
    for (int j = 0; j < nvec; ++j) {
        const float4 v = *reinterpret_cast<const float4 *>(p + 512 * j);
        welford_step_i(w, v.x, 4 * j);
        welford_step_i(w, v.y, 4 * j + 1);
        welford_step_i(w, v.z, 4 * j + 2);
        welford_step_i(w, v.w, 4 * j + 3);
    }
    ln_merge(w, K, mu, var, red);
}

__device__ __forceinline__ void ln_merge(Welford w, int64_t K, float &mu, float &var, float *red) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        Welford o;
        o.m = __shfl_down_sync(0xFFFFFFFFu, w.m, off);
        o.s = __shfl_down_sync(0xFFFFFFFFu, w.s, off);
        o.c = __shfl_down_sync(0xFFFFFFFFu, w.c, off);
        w = wcombine(w, o);  // meaningful for lanes < off; lane 0 ends with the warp's state
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        red[warp * 3 + 0] = w.m;
        red[warp * 3 + 1] = w.s;
        red[warp * 3 + 2] = w.c;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        Welford w0{red[0], red[1], red[2]}, w1{red[3], red[4], red[5]}, w2{red[6], red[7], red[8]},
            w3{red[9], red[10], red[11]};
        w0 = wcombine(w0, w2);
        w1 = wcombine(w1, w3);
        w0 = wcombine(w0, w1);
        red[12] = w0.m;
        red[13] = __fdiv_rn(w0.s, static_cast<float>(K));
    }
    __syncthreads();
    mu = red[12];
    var = red[13];
}

// ------------------------------------------------------------------------------------------------- kernel A
// LayerNorm (no affine) + modulate, one row at a time per CTA of 128 threads (fused_kernels.py:219-232 _lnmod):
// x = R16((x - mu) * rsqrt.approx(var + eps)); out = R16(R16(x * s1) + shift). K % 512 == 0, NV = K / 512.
// Persistent: CTA b handles rows b, b + gridDim.x, ...; the next row's x is loaded into registers while the current
// row is reduced and written, so every thread keeps a row's loads in flight.
template <int NV>
__global__ void __launch_bounds__(128) ln_modulate_kernel(const __nv_bfloat16 *__restrict__ x,
                                                          const __nv_bfloat16 *__restrict__ s1,
                                                          const __nv_bfloat16 *__restrict__ sh,
                                                          __nv_bfloat16 *__restrict__ out, int64_t rows, int64_t K,
                                                          int64_t rows_per_group, float eps, int pf) {
    __shared__ float red[2][16];  // two buffers: row i + 1's statistics never overwrite what row i still reads
    const int t = threadIdx.x;
    int64_t row = blockIdx.x;
    if (row >= rows) return;
    asm volatile("griddepcontrol.wait;" ::: "memory");  // launched as a programmatic dependent: x is ready here
    allow_dependents();
    uint2 raw[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) raw[j] = __ldg(reinterpret_cast<const uint2 *>(x + row * K) + t + 128 * j);
    uint2 sraw[NV], hraw[NV];
    int64_t cached_group = -1;
    int parity = 0;
    for (; row < rows; row += gridDim.x, parity ^= 1) {
        float v[NV * 4];
#pragma unroll
        for (int j = 0; j < NV; ++j) unpack4(raw[j], v + 4 * j);
        const int64_t nrow = row + gridDim.x;
        if (nrow < rows) {
#pragma unroll
            for (int j = 0; j < NV; ++j) raw[j] = __ldg(reinterpret_cast<const uint2 *>(x + nrow * K) + t + 128 * j);
        }
        // past the register prefetch of the next row, pull row nrow + pf into L2 (K x 2 bytes, 16-byte aligned)
        if (pf > 0 && t == 0 && nrow + pf < rows)
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(x + (nrow + pf) * K),
                         "r"(static_cast<uint32_t>(K * 2)) : "memory");
        // the modulation rows of this row's group (kept while consecutive rows stay in one group)
        const int64_t group = static_cast<int64_t>(static_cast<uint32_t>(row) / static_cast<uint32_t>(rows_per_group));
        if (group != cached_group) {
            cached_group = group;
#pragma unroll
            for (int j = 0; j < NV; ++j) {
                sraw[j] = __ldg(reinterpret_cast<const uint2 *>(s1 + group * K) + t + 128 * j);
                hraw[j] = __ldg(reinterpret_cast<const uint2 *>(sh + group * K) + t + 128 * j);
            }
        }
        float mu, var;
        ln_stats_n<NV * 4>(v, K, mu, var, red[parity]);  // its two barriers are the row's only ones
        const float rstd = rsqrt_approx(__fadd_rn(var, eps));
        const uint64_t neg_mu = f2pack(-mu, -mu), rstd2 = f2pack(rstd, rstd);  // x - mu == x + (-mu), exactly
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int64_t c = static_cast<int64_t>(t + 128 * j) * 4;
            const uint64_t a = mul2(add2(f2pack(v[4 * j], v[4 * j + 1]), neg_mu), rstd2);
            const uint64_t b = mul2(add2(f2pack(v[4 * j + 2], v[4 * j + 3]), neg_mu), rstd2);
            const uint32_t n01 = pack2(f2lo(a), f2hi(a));
            const uint32_t n23 = pack2(f2lo(b), f2hi(b));
            *reinterpret_cast<uint2 *>(out + row * K + c) =
                make_uint2(mod_bf16x2(n01, sraw[j].x, hraw[j].x), mod_bf16x2(n23, sraw[j].y, hraw[j].y));
        }
    }
}

// resident CTAs per SM of a kernel (cached per kernel and device) times the SMs: a persistent grid's width
template <auto KERN>
int persistent_grid(int threads, size_t smem, int64_t items) {
    const int64_t g = std::min<int64_t>(items, wave_ctas<KERN>(threads, smem));
    return static_cast<int>(std::max<int64_t>(g, 1));
}

// A launch as a programmatic dependent of the previous kernel in the stream: its CTAs may be scheduled while that
// kernel finishes; the kernel executes griddepcontrol.wait before its first global access.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), int grid, int threads, cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
    cfg.blockDim = dim3(static_cast<unsigned>(threads), 1, 1);
    cfg.stream = stream;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// ------------------------------------------------------------------------------------------------- RMSNorm-128
// One row of 128 per warp (fused_kernels.py:189-217 _rms128): lane t squares values 4t .. 4t+3 and adds them as
// ((a + b) + c) + d, a pairwise tree over the lanes (lane t + lane t + 16, ...), rstd = rsqrt.approx(sum / 128 +
// eps), y = R16((x * rstd) * w). 8 warps per CTA, rows grid-strided.
__global__ void __launch_bounds__(256) rms128_kernel(const __nv_bfloat16 *__restrict__ x, const void *__restrict__ w,
                                                     int wdt, __nv_bfloat16 *__restrict__ out, int64_t n_rows,
                                                     float eps) {
    const int lane = threadIdx.x & 31;
    float wv[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) wv[k] = load_w(w, wdt, 4 * lane + k);
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < n_rows;
         r += warps) {
        float v[4];
        unpack4(__ldg(reinterpret_cast<const uint2 *>(x + r * 128) + lane), v);
        float s = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(v[0], v[0]), __fmul_rn(v[1], v[1])), __fmul_rn(v[2], v[2])),
                            __fmul_rn(v[3], v[3]));
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) s = __fadd_rn(s, __shfl_down_sync(0xFFFFFFFFu, s, off));
        s = __shfl_sync(0xFFFFFFFFu, s, 0);
        const float rstd = rsqrt_approx(__fadd_rn(__fmul_rn(s, 0.0078125f), eps));
        float o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) o[k] = __fmul_rn(__fmul_rn(v[k], rstd), wv[k]);
        *reinterpret_cast<uint2 *>(out + r * 128 + 4 * lane) = make_uint2(pack2(o[0], o[1]), pack2(o[2], o[3]));
    }
}

// ------------------------------------------------------------------------------------------------- kernel B
// RMSNorm-128 + split-half RoPE of contiguous (B, L, H, 128) rows (sage_fused.py:246-272 _rms_rope128, the
// reproduction of comfy_kitchen's rope kernel): lane t owns values t, t+32, t+64, t+96; squares summed by fma from
// 0 in that order, pairwise lane tree, rr = rsqrt.approx(sum / 128 + eps), n = R16((x * rr) * w); then the pairs
// (d, d + 64) rotate: y0 = R16(fma(f00, lo, f01 * hi)), y1 = R16(fma(f10, lo, f11 * hi)). Rotations f[token, d] are
// float32 2x2 with element strides (s_tok, s_d, s_i, s_j).
// One (batch, token) per warp: its rotations are read once for all its heads; the heads' rows are loaded four at a
// time before any of them is reduced, so each warp keeps several loads in flight.
template <bool F4>
__device__ __forceinline__ void load_rot(const float *fd, int64_t s_i, int64_t s_j, float r[4]) {
    if constexpr (F4) {
        const float4 q = __ldg(reinterpret_cast<const float4 *>(fd));
        r[0] = q.x; r[1] = q.y; r[2] = q.z; r[3] = q.w;
    } else {
        r[0] = __ldg(fd); r[1] = __ldg(fd + s_j); r[2] = __ldg(fd + s_i); r[3] = __ldg(fd + s_i + s_j);
    }
}

constexpr int kRopeHeads = 16;  // head rows staged per warp at a time (4 KB)
constexpr int kRopeWarps = 4;   // warps per CTA (two 4 KB buffers each: 32 KB of shared memory)

// Staging layout of a row block: 16-byte chunk c of row R at chunk (c ^ 2 (R & 1)) of the row, so that the two
// half-warps (rows of opposite parity, 256 bytes apart: the same banks) read and write disjoint banks.
__device__ __forceinline__ int rope_swz(int q) { return q ^ (((q >> 4) & 1) << 1); }

// The tensors of one launch: q alone, or q and k (same shape, rotations and weight dtype).
struct RopeTensors {
    const __nv_bfloat16 *x[2];
    const void *w[2];
    __nv_bfloat16 *out[2];
};

template <bool F4>
__global__ void __launch_bounds__(kRopeWarps * 32) rms_rope_kernel(const __grid_constant__ RopeTensors t, int n_tensors,
                                                                   const float *__restrict__ f, int wdt,
                                                                   int64_t n_tok, int64_t heads, int64_t tokens,
                                                                   float eps, int64_t s_tok, int64_t s_d, int64_t s_i,
                                                                   int64_t s_j) {
    // Work item = (tensor, batch, token, group of up to 16 heads). A warp walks its items with two shared-memory
    // buffers: the next item's rows (4 KB) are copied in by 16-byte cp.async while the current one is computed. Each
    // half-warp reduces rows (layout below) reading the values its sums need from shared memory, two rows at a time
    // so their shuffle chains overlap; the results go back in place and leave with 16-byte stores; the token's
    // rotations are read once for all heads of the item. q and k in one launch give each warp twice the items (one
    // ramp and one tail instead of two).
    __shared__ __align__(16) __nv_bfloat16 stage[kRopeWarps][2][kRopeHeads * 128];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t n_hc = (heads + kRopeHeads - 1) / kRopeHeads;
    const int64_t per_tensor = n_tok * n_hc;
    const int64_t items = per_tensor * n_tensors;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * kRopeWarps;
    int64_t it = static_cast<int64_t>(blockIdx.x) * kRopeWarps + wid;
    if (it >= items) return;  // whole warps only; nothing below synchronises the CTA
    // Half-warp layout: half hf (= lane / 16) of the warp takes rows hh + hf, hh + 2 + hf of each group of four;
    // its lane L holds values L + 16 k (k = 0..7) of the row, i.e. the partial sums of lanes L (k even) and L + 16
    // (k odd) of the reference's 32-lane layout. The first level of the reference's shuffle-down tree (t + 16) is
    // then a local add and the other four levels an xor butterfly inside the half: every lane ends with the bits of
    // the reference's lane 0, each node being the same two operands (IEEE addition is commutative).
    const int hf = lane >> 4, L = lane & 15;
    // item -> (tensor ti, row block bt, first head h0); returns the item's head count
    auto rows_of = [&](int64_t item, int &ti, int64_t &bt, int64_t &h0) -> int {
        ti = item >= per_tensor ? 1 : 0;
        const int64_t local = item - ti * per_tensor;
        bt = local / n_hc;
        h0 = (local - bt * n_hc) * kRopeHeads;
        return static_cast<int>(heads - h0 < kRopeHeads ? heads - h0 : kRopeHeads);
    };
    auto issue = [&](int64_t item, __nv_bfloat16 *dst) {
        int ti;
        int64_t bt, h0;
        const int chunks = rows_of(item, ti, bt, h0) * 16;  // 16-byte chunks of the item's rows
        const uint4 *src = reinterpret_cast<const uint4 *>(t.x[ti] + (bt * heads + h0) * 128);
#pragma unroll
        for (int i = 0; i < kRopeHeads / 2; ++i) {
            const int q = lane + 32 * i;
            if (q < chunks) cp_async16(reinterpret_cast<uint4 *>(dst) + rope_swz(q), src + q);
        }
        cp_async_commit();
    };
    issue(it, stage[wid][0]);
    for (int p = 0; it < items; it += warps, p ^= 1) {
        if (it + warps < items) issue(it + warps, stage[wid][p ^ 1]);
        else cp_async_commit();  // an empty group: wait_group<1> below then still means "this item's copies"
        int ti;
        int64_t bt, h0;
        const int nh = rows_of(it, ti, bt, h0);
        const int64_t tok = bt % tokens;
        float rot[4][4];  // frequencies d = L + 16 k, k = 0..3 (pairs (d, d + 64))
#pragma unroll
        for (int k = 0; k < 4; ++k) load_rot<F4>(f + tok * s_tok + (L + 16 * k) * s_d, s_i, s_j, rot[k]);
        float w[8];  // the tensor's weights at this lane's values (L1 hits after the first item)
#pragma unroll
        for (int k = 0; k < 8; ++k) w[k] = load_w(t.w[ti], wdt, L + 16 * k);
        cp_async_wait<1>();
        __syncwarp();
        __nv_bfloat16 *buf = stage[wid][p];
        for (int hh = 0; hh < nh; hh += 4) {  // rows hh + hf and hh + 2 + hf (those >= nh computed, not written)
            float v[2][8], sum[2];
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                // value L + 16 k of row R sits at element 16 (k ^ (R & 1)) + L of the row (R & 1 == hf)
                const __nv_bfloat16 *ev = buf + (hh + 2 * r + hf) * 128 + L + 16 * hf;  // k even
                const __nv_bfloat16 *od = ev - 32 * hf;                                  // k odd
#pragma unroll
                for (int k = 0; k < 8; ++k) v[r][k] = __bfloat162float((k & 1) ? od[16 * k] : ev[16 * k]);
                float a0 = __fmul_rn(v[r][0], v[r][0]), a1 = __fmul_rn(v[r][1], v[r][1]);
                a0 = __fmaf_rn(v[r][2], v[r][2], a0);
                a1 = __fmaf_rn(v[r][3], v[r][3], a1);
                a0 = __fmaf_rn(v[r][4], v[r][4], a0);
                a1 = __fmaf_rn(v[r][5], v[r][5], a1);
                a0 = __fmaf_rn(v[r][6], v[r][6], a0);
                a1 = __fmaf_rn(v[r][7], v[r][7], a1);
                sum[r] = __fadd_rn(a0, a1);
            }
#pragma unroll
            for (int off = 8; off >= 1; off >>= 1) {
#pragma unroll
                for (int r = 0; r < 2; ++r) sum[r] = __fadd_rn(sum[r], __shfl_xor_sync(0xFFFFFFFFu, sum[r], off));
            }
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const int row = hh + 2 * r + hf;
                const float rr = rsqrt_approx(__fadd_rn(__fmul_rn(sum[r], 0.0078125f), eps));
                float n[8];
#pragma unroll
                for (int k = 0; k < 8; k += 2) {
                    const float2 nn = r16x2(__fmul_rn(__fmul_rn(v[r][k], rr), w[k]),
                                            __fmul_rn(__fmul_rn(v[r][k + 1], rr), w[k + 1]));
                    n[k] = nn.x;
                    n[k + 1] = nn.y;
                }
                if (row < nh) {  // the other half's row may be valid: no warp-wide operation below
                    __nv_bfloat16 *ev = buf + row * 128 + L + 16 * hf;
                    __nv_bfloat16 *od = ev - 32 * hf;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {  // pair (d, d + 64), d = L + 16 k (k and k + 4 of one parity)
                        const float lo = n[k], hi = n[k + 4];
                        __nv_bfloat16 *e = (k & 1) ? od : ev;
                        e[16 * k] = __float2bfloat16_rn(__fmaf_rn(rot[k][0], lo, __fmul_rn(rot[k][1], hi)));
                        e[16 * k + 64] = __float2bfloat16_rn(__fmaf_rn(rot[k][2], lo, __fmul_rn(rot[k][3], hi)));
                    }
                }
            }
        }
        __syncwarp();
        const int chunks = nh * 16;
        uint4 *dst = reinterpret_cast<uint4 *>(t.out[ti] + (bt * heads + h0) * 128);
#pragma unroll
        for (int i = 0; i < kRopeHeads / 2; ++i) {
            const int q = lane + 32 * i;
            if (q < chunks) dst[q] = reinterpret_cast<const uint4 *>(buf)[rope_swz(q)];
        }
        __syncwarp();  // every lane has read this buffer before it is refilled (the next iteration's issue)
    }
    cp_async_wait<0>();
}

// ------------------------------------------------------------------------------------------------- kernel B (v2)
// The same arithmetic as rms_rope_kernel, laid out for fewer instructions per value: one (tensor, batch-token) item
// per warp (its rotations and weights read once for all its heads), one row per half-warp at a time, and lane p of a
// half holding the reference's lanes 2p and 2p + 1 -- values 2p + 32 j and 2p + 1 + 32 j (j = 0..3), i.e. the 32-bit
// words p + 16 j of the row, read and written with coalesced 4-byte accesses straight from / to global memory. The
// reference's reduction tree maps onto xor shuffles with the same two operands at every node: level t + 16 is lane
// p + 8 (xor 8) for the even and the odd lane sums, t + 8 xor 4, t + 4 xor 2, t + 2 xor 1, and the last level t + 1
// is the lane's own even + odd sum. The RoPE pairs (d, d + 64) are words j and j + 2 of the lane: no exchange.
// Launched as a programmatic dependent (griddepcontrol.wait before the first load).
template <int WDT>
__device__ __forceinline__ float2 load_w2(const void *w, int i) {  // weights i, i + 1 (i even)
    if constexpr (WDT == WF_BF16) {
        const uint32_t u = __ldg(reinterpret_cast<const uint32_t *>(static_cast<const __nv_bfloat16 *>(w) + i));
        return make_float2(bf_lo(u), bf_hi(u));
    } else if constexpr (WDT == WF_F16) {
        const __half2 h = __ldg(reinterpret_cast<const __half2 *>(static_cast<const __half *>(w) + i));
        return __half22float2(h);
    } else {
        return __ldg(reinterpret_cast<const float2 *>(static_cast<const float *>(w) + i));
    }
}

constexpr int kRope2Warps = 8;  // warps (items) per CTA

// Up to 4 rows in flight the kernel fits in 85 registers, which leaves 3 CTAs of 256 threads per SM (the bound is
// explicit: left to itself ptxas took 89 registers, 2 CTAs per SM, and the launch 15 % longer); 8 rows need more.
template <int WDT, bool F4, int R>
__global__ void __launch_bounds__(kRope2Warps * 32, R <= 4 ? 3 : 1) rms_rope_v2_kernel(const __grid_constant__ RopeTensors t,
                                                                       int n_items, int n_tok, int heads, int tokens,
                                                                       const float *__restrict__ f, float eps,
                                                                       int64_t s_tok, int64_t s_d, int64_t s_i,
                                                                       int64_t s_j, int pf) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    allow_dependents();
    const int lane = threadIdx.x & 31, hf = lane >> 4, p = lane & 15;
    const int item = blockIdx.x * kRope2Warps + (threadIdx.x >> 5);
    if (item >= n_items) return;  // whole warps: the shuffles below involve both halves of a warp that runs
    if (pf > 0 && lane == 0 && item + pf < n_items) {
        // pull into L2 the rows of the item that the warp in this position one wave of CTAs later handles: more
        // bytes in flight than the registers of the resident warps hold, at no register or shared-memory cost
        // (a token's heads x 256 bytes, 16-byte aligned like the tensor)
        const int nx = item + pf, tn = nx >= n_tok ? 1 : 0;
        const __nv_bfloat16 *src = t.x[tn] + static_cast<size_t>(nx - tn * n_tok) * heads * 128;
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(heads * 256) : "memory");
    }
    const int ti = item >= n_tok ? 1 : 0;
    const int bt = item - ti * n_tok;
    const int tok = bt % tokens;
    // rotations of d = 2p + 32 m2 + e (m = 2 m2 + e: d = 2p, 2p + 1, 2p + 32, 2p + 33), as f00, f01, f10, f11
    float rot[4][4];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const float *fd = f + tok * s_tok + (2 * p + 32 * (m >> 1) + (m & 1)) * s_d;
        if constexpr (F4) {
            const float4 q = __ldg(reinterpret_cast<const float4 *>(fd));
            rot[m][0] = q.x; rot[m][1] = q.y; rot[m][2] = q.z; rot[m][3] = q.w;
        } else {
            rot[m][0] = __ldg(fd); rot[m][1] = __ldg(fd + s_j); rot[m][2] = __ldg(fd + s_i);
            rot[m][3] = __ldg(fd + s_i + s_j);
        }
    }
    uint64_t w[4];  // weights at 2p + 32 j (low lane), 2p + 1 + 32 j (high lane)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float2 wj = load_w2<WDT>(t.w[ti], 2 * p + 32 * j);
        w[j] = f2pack(wj.x, wj.y);
    }
    // the rotations of the pairs (d, d + 64) with d = 2p + 32 j (low lane) and 2p + 1 + 32 j (high lane)
    uint64_t r00[2], r01[2], r10[2], r11[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        r00[j] = f2pack(rot[2 * j][0], rot[2 * j + 1][0]);
        r01[j] = f2pack(rot[2 * j][1], rot[2 * j + 1][1]);
        r10[j] = f2pack(rot[2 * j][2], rot[2 * j + 1][2]);
        r11[j] = f2pack(rot[2 * j][3], rot[2 * j + 1][3]);
    }
    const uint32_t *x = reinterpret_cast<const uint32_t *>(t.x[ti]) + static_cast<size_t>(bt) * heads * 64 + p;
    uint32_t *out = reinterpret_cast<uint32_t *>(t.out[ti]) + static_cast<size_t>(bt) * heads * 64 + p;
    // both halves run the same iterations (full-warp shuffles); a half whose row is past the last head computes on
    // the last row again and does not store
    for (int h0 = 0; h0 < heads; h0 += 2 * R) {
        uint32_t u[R][4];
        int row[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            row[r] = h0 + 2 * r + hf;  // rows h0 .. h0 + 2R - 1, the halves interleaved
            const int rr = row[r] < heads ? row[r] : heads - 1;
#pragma unroll
            for (int j = 0; j < 4; ++j) u[r][j] = __ldg(x + rr * 64 + 16 * j);
        }
        uint64_t acc[R];  // the reference's lanes 2p (low) and 2p + 1 (high): fma of squares from 0
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const uint64_t v0 = bf_pair(u[r][0]);
            acc[r] = mul2(v0, v0);
#pragma unroll
            for (int j = 1; j < 4; ++j) {
                const uint64_t vj = bf_pair(u[r][j]);
                acc[r] = fma2(vj, vj, acc[r]);
            }
        }
#pragma unroll
        for (int off = 8; off >= 1; off >>= 1) {
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const float e = __shfl_xor_sync(0xFFFFFFFFu, f2lo(acc[r]), off);
                const float o = __shfl_xor_sync(0xFFFFFFFFu, f2hi(acc[r]), off);
                acc[r] = add2(acc[r], f2pack(e, o));
            }
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const float rs = rsqrt_approx(__fadd_rn(__fmul_rn(__fadd_rn(f2lo(acc[r]), f2hi(acc[r])), 0.0078125f), eps));
            const uint64_t rs2 = f2pack(rs, rs);
            uint64_t n[4];  // R16((x * rs) * w) at 2p + 32 j, 2p + 1 + 32 j
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint64_t m = mul2(mul2(bf_pair(u[r][j]), rs2), w[j]);
                const float2 nn = r16x2(f2lo(m), f2hi(m));
                n[j] = f2pack(nn.x, nn.y);
            }
            if (row[r] < heads) {
#pragma unroll
                for (int j = 0; j < 2; ++j) {  // pairs (d, d + 64): words j and j + 2
                    const uint64_t y0 = fma2(r00[j], n[j], mul2(r01[j], n[j + 2]));
                    const uint64_t y1 = fma2(r10[j], n[j], mul2(r11[j], n[j + 2]));
                    out[row[r] * 64 + 16 * j] = pack2(f2lo(y0), f2hi(y0));
                    out[row[r] * 64 + 16 * (j + 2)] = pack2(f2lo(y1), f2hi(y1));
                }
            }
        }
    }
}

// ------------------------------------------------------------------------------------------------- quantiser
// Per-token int8 quantisation of a row (fused_kernels.py:137-174 _quant_row), one row per CTA of 128 threads:
//   PRE 0 none | 1 GELU of the bf16 value from a 65536-entry bf16 table | 2 modulate | 3 LayerNorm + modulate;
//   ROT: the ConvRot Hadamard of every 256 values (four radix-4 stages of stride 1, 4, 16, 64, each 4-tuple
//        (a, b, c, d) -> (a+b+c-d, a+b-c+d, a-b+c+d, -a+b+c+d) summed left to right, then x 1/16) -- off for the
//        plain per-token absmax quantiser;
//   amax = min(max |x|, 3.38953139e38), scale = max(amax / 127, 1e-30) (stored),
//   q = rint(R16(R16(x) / R16(scale))) clamped to [-128, 127].
// The row (after PRE) is staged in shared memory as float32 (K * 4 bytes, dynamic).
template <int PRE, bool ROT>
__global__ void __launch_bounds__(128) quant_rows_kernel(const __nv_bfloat16 *__restrict__ x,
                                                         const __nv_bfloat16 *__restrict__ s1,
                                                         const __nv_bfloat16 *__restrict__ sh,
                                                         const __nv_bfloat16 *__restrict__ gelu,
                                                         int8_t *__restrict__ q, float *__restrict__ scale_out,
                                                         int64_t K, int64_t rows_per_group, float eps) {
    extern __shared__ __align__(16) float srow[];
    __shared__ float red[16];
    allow_dependents();
    const int64_t row = blockIdx.x;
    const int t = threadIdx.x;
    const __nv_bfloat16 *xr = x + row * K;
    const int nvec = static_cast<int>(K / 512);  // vectors of 4 per thread (K % 512 == 0) ...
    const int64_t goff = (row / rows_per_group) * K;
    if constexpr (PRE == 3) {
        // the row goes to shared memory first; this thread's Welford pass reads its own vectors back in order
        for (int j = 0; j < nvec; ++j) {
            float v[4];
            unpack4(__ldg(reinterpret_cast<const uint2 *>(xr) + t + 128 * j), v);
            *reinterpret_cast<float4 *>(srow + (t + 128 * j) * 4) = make_float4(v[0], v[1], v[2], v[3]);
        }
        float mu, var;
        ln_stats_strided(srow + 4 * t, nvec, K, mu, var, red);
        const float rstd = rsqrt_approx(__fadd_rn(var, eps));
        for (int j = 0; j < nvec; ++j) {
            const int64_t c = static_cast<int64_t>(t + 128 * j) * 4;
            float s[4], h[4];
            unpack4(__ldg(reinterpret_cast<const uint2 *>(s1 + goff + c)), s);
            unpack4(__ldg(reinterpret_cast<const uint2 *>(sh + goff + c)), h);
            const float4 v4 = *reinterpret_cast<const float4 *>(srow + c);
            const float v[4] = {v4.x, v4.y, v4.z, v4.w};
            float o[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float n = r16(__fmul_rn(__fsub_rn(v[k], mu), rstd));
                o[k] = r16(__fadd_rn(r16(__fmul_rn(n, s[k])), h[k]));
            }
            *reinterpret_cast<float4 *>(srow + c) = make_float4(o[0], o[1], o[2], o[3]);
        }
    } else {
        // ... or, without the layer norm, any K % 4 == 0: vectors t, t + 128, ...
        for (int64_t vi = t; vi < K / 4; vi += 128) {
            const int64_t c = vi * 4;
            float v[4];
            unpack4(__ldg(reinterpret_cast<const uint2 *>(xr + c)), v);
            if constexpr (PRE == 1) {
                const uint2 raw = __ldg(reinterpret_cast<const uint2 *>(xr + c));
                const uint32_t b[4] = {raw.x & 0xFFFFu, raw.x >> 16, raw.y & 0xFFFFu, raw.y >> 16};
#pragma unroll
                for (int k = 0; k < 4; ++k) v[k] = __bfloat162float(gelu[b[k]]);
            } else if constexpr (PRE == 2) {
                float s[4], h[4];
                unpack4(__ldg(reinterpret_cast<const uint2 *>(s1 + goff + c)), s);
                unpack4(__ldg(reinterpret_cast<const uint2 *>(sh + goff + c)), h);
#pragma unroll
                for (int k = 0; k < 4; ++k) v[k] = r16(__fadd_rn(r16(__fmul_rn(v[k], s[k])), h[k]));
            }
            *reinterpret_cast<float4 *>(srow + c) = make_float4(v[0], v[1], v[2], v[3]);
        }
    }
    __syncthreads();
    if constexpr (ROT) {
        for (int S = 1; S <= 64; S *= 4) {
            for (int64_t u = t; u < K / 4; u += 128) {
                const int64_t grp = u / 64, uu = u - grp * 64;           // 64 tuples per 256-group
                const int64_t base = grp * 256 + (uu / S) * 4 * S + (uu % S);
                const float a = srow[base], b = srow[base + S], c = srow[base + 2 * S], d = srow[base + 3 * S];
                const float y0 = __fsub_rn(__fadd_rn(__fadd_rn(a, b), c), d);
                const float y1 = __fadd_rn(__fsub_rn(__fadd_rn(a, b), c), d);
                const float y2 = __fadd_rn(__fadd_rn(__fsub_rn(a, b), c), d);
                const float y3 = __fadd_rn(__fadd_rn(__fadd_rn(-a, b), c), d);
                srow[base] = y0;
                srow[base + S] = y1;
                srow[base + 2 * S] = y2;
                srow[base + 3 * S] = y3;
            }
            __syncthreads();
        }
    }
    // amax of the row (after the 1/16 scaling when rotated)
    float amax = 0.f;
    for (int64_t c = 4 * t; c < K; c += 512) {
        float4 f4 = *reinterpret_cast<const float4 *>(srow + c);
        if constexpr (ROT) {
            f4.x = __fmul_rn(f4.x, 0.0625f); f4.y = __fmul_rn(f4.y, 0.0625f);
            f4.z = __fmul_rn(f4.z, 0.0625f); f4.w = __fmul_rn(f4.w, 0.0625f);
            *reinterpret_cast<float4 *>(srow + c) = f4;
        }
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(f4.x), fabsf(f4.y)), fmaxf(fabsf(f4.z), fabsf(f4.w))));
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, off));
    if ((t & 31) == 0) red[t >> 5] = amax;
    __syncthreads();
    amax = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    amax = fminf(amax, 3.38953139e38f);
    const float scale = fmaxf(div_full(amax, 127.0f), 1.0e-30f);
    if (t == 0) scale_out[row] = scale;
    const float sb = r16(scale);
    for (int64_t c = 4 * t; c < K; c += 512) {
        const float4 f4 = *reinterpret_cast<const float4 *>(srow + c);
        const float fv[4] = {f4.x, f4.y, f4.z, f4.w};
        uint32_t packed = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            float y = rintf(r16(div_full(r16(fv[k]), sb)));
            y = fminf(fmaxf(y, -128.0f), 127.0f);
            packed |= (static_cast<uint32_t>(static_cast<int>(y)) & 0xFFu) << (8 * k);
        }
        *reinterpret_cast<uint32_t *>(q + row * K + c) = packed;
    }
}

// v = the pending operation of the chunk (pre 1: the GELU table, pre 2: bf16(bf16(v * s1) + shift)), v bf16 in and out
template <int PRE, int NCH>
__device__ __forceinline__ void quant_pre(uint4 (&v)[NCH], const __nv_bfloat16 *__restrict__ s1,
                                          const __nv_bfloat16 *__restrict__ sh, const __nv_bfloat16 *__restrict__ gelu,
                                          int64_t goff, int lane) {
    if constexpr (PRE == 2) {
        const uint4 *sr = reinterpret_cast<const uint4 *>(s1 + goff);
        const uint4 *hr = reinterpret_cast<const uint4 *>(sh + goff);
#pragma unroll
        for (int j = 0; j < NCH; ++j) {
            const uint4 sv = __ldg(sr + 32 * j + lane), hv = __ldg(hr + 32 * j + lane);
            v[j] = make_uint4(mod_bf16x2(v[j].x, sv.x, hv.x), mod_bf16x2(v[j].y, sv.y, hv.y),
                              mod_bf16x2(v[j].z, sv.z, hv.z), mod_bf16x2(v[j].w, sv.w, hv.w));
        }
    } else if constexpr (PRE == 1) {
        const uint16_t *tab = reinterpret_cast<const uint16_t *>(gelu);
#pragma unroll
        for (int j = 0; j < NCH; ++j) {
            const uint32_t xs[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
            uint32_t o[4];
#pragma unroll
            for (int k = 0; k < 4; ++k)
                o[k] = static_cast<uint32_t>(__ldg(tab + (xs[k] & 0xFFFFu))) |
                       (static_cast<uint32_t>(__ldg(tab + (xs[k] >> 16))) << 16);
            v[j] = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
}

template <int NCH>
__device__ __forceinline__ float chunk_amax(const uint4 (&v)[NCH]) {
    uint32_t m = 0;  // the largest |value| so far in each bf16 lane (+0 to start, as fmaxf from 0)
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
        m = bf2_max(m, bf2_max(bf2_abs(v[j].x), bf2_abs(v[j].y)));
        m = bf2_max(m, bf2_max(bf2_abs(v[j].z), bf2_abs(v[j].w)));
    }
    return fmaxf(bf_lo(m), bf_hi(m));
}

// clamp(rint(bf16(v / sb)), -128, 127) of the four values of two bf16 pairs, as four bytes. The bf16 rounding of
// the quotients is one cvt.rn.bf16x2 per pair (the reference's integer rounding gives the same value for every finite
// or infinite quotient; a NaN becomes -128 either way). The bounds are integers, so clamping first gives
// rint-then-clamp's value, and the round to the nearest (even) integer is the float addition of 1.5 * 2^23, whose
// low mantissa byte is then the two's-complement int8 (exact for |y| <= 2^22).
__device__ __forceinline__ uint32_t quant_quad(uint32_t xa, uint32_t xb, float sb) {
    __nv_bfloat162 ta = __floats2bfloat162_rn(div_full(bf_lo(xa), sb), div_full(bf_hi(xa), sb));
    __nv_bfloat162 tb = __floats2bfloat162_rn(div_full(bf_lo(xb), sb), div_full(bf_hi(xb), sb));
    constexpr uint32_t kLo = 0xC300C300u, kHi = 0x42FE42FEu;  // -128 and 127 in both bf16 lanes (exact)
    const uint32_t ua = bf2_min(bf2_max(*reinterpret_cast<uint32_t *>(&ta), kLo), kHi);
    const uint32_t ub = bf2_min(bf2_max(*reinterpret_cast<uint32_t *>(&tb), kLo), kHi);
    constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
    const uint64_t M2 = f2pack(kMagic, kMagic);
    const uint64_t ra = add2(bf_pair(ua), M2), rb = add2(bf_pair(ub), M2);
    const uint32_t r0 = static_cast<uint32_t>(ra), r1 = static_cast<uint32_t>(ra >> 32);
    const uint32_t r2 = static_cast<uint32_t>(rb), r3 = static_cast<uint32_t>(rb >> 32);
    return __byte_perm(__byte_perm(r0, r1, 0x0040), __byte_perm(r2, r3, 0x0040), 0x5410);
}

template <int NCH>
__device__ __forceinline__ void quant_store(const uint4 (&v)[NCH], float sb, uint2 *qr, int lane) {
#pragma unroll
    for (int j = 0; j < NCH; ++j) qr[32 * j + lane] = make_uint2(quant_quad(v[j].x, v[j].y, sb),
                                                                  quant_quad(v[j].z, v[j].w, sb));
}

// The quantiser without rotation or layer norm (pre 0 / 1 / 2) for K = 256 * NCH * WPR: the row in registers as packed
// bf16 (WPR warps per row; lane l of the row's warp w holds the 8 values at 8 * (32 * (NCH * w + j) + l) .. +7,
// j < NCH), all of the row's 16-byte loads issued before the first is used, the absmax by shuffles (and, with
// WPR > 1, across the row's warps through shared memory), 8-byte int8 stores. With one warp per row and NCH <= 8 the
// warp walks several rows and the loads of its next row are in flight while the current one is converted. The same
// arithmetic as quant_rows_kernel above: the pending operation rounded to bf16 as there, amax = min(max |v|,
// 3.38953139e38), scale = max(amax / 127, 1e-30) (div.full), q = clamp(rint(bf16(v / bf16(scale)))) -- every v is
// already a bf16 value here, so the reference's bf16 rounding of v before the division is the identity.
// ConvRot: the 256-wide Hadamard of the quantiser (quant_rows_kernel's four radix-4 stages) on a register chunk. Element
// e = 8 * lane + i of a 256-group (i = 0..7 in the lane) has base-4 digits d0 = i & 3, d1 = 2 * (lane & 1) + (i >> 2),
// d2 = (lane >> 1) & 3, d3 = (lane >> 3) & 3; stage s combines the four elements that differ only in digit s, taken
// in digit order (a, b, c, d), into output k = their digit: ((+-a +- b) +- c) +- d with the signs of output k --
// k = 0: (+, +, +, -), 1: (+, +, -, +), 2: (+, -, +, +), 3: (-, +, +, +) -- the reference's sums, left to right.

// had4 of output k for two independent sets of four values at once (packed float32 lanes): the terms' signs as
// factors +-1 (exact), t = fma(sa, a, sb * b), then fma(sc, c, t), fma(sd, d, t) -- each fma rounds once, so every
// step is the reference's float addition of the (negated) term, in the same order
__device__ __forceinline__ uint64_t had4x2(uint64_t a, uint64_t b, uint64_t c, uint64_t d, const uint64_t (&s)[4]) {
    return fma2(s[3], d, fma2(s[2], c, fma2(s[0], a, mul2(s[1], b))));
}
// the sign factors of output k: term j is negated when j == 3 - k
__device__ __forceinline__ void had4_signs(int k, uint64_t (&s)[4]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float f = j == 3 - k ? -1.0f : 1.0f;
        s[j] = f2pack(f, f);
    }
}

// the chunk's 8 values of this lane, rotated and scaled by 1/16 (exact); all 32 lanes take part. Values i and
// i + 4 (digit 0 and 1 stages) or i and i + 1 (digit 2 and 3) share their signs and run as one packed pair.
__device__ __forceinline__ void hadamard256(float (&f)[8], int lane) {
    uint64_t s[4];
    // digit 0: inside the lane; outputs k of the two halves (values 0-3 and 4-7) as one pair
    uint64_t o[4];  // (output k of values 0-3, output k of values 4-7)
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        had4_signs(k, s);
        o[k] = had4x2(f2pack(f[0], f[4]), f2pack(f[1], f[5]), f2pack(f[2], f[6]), f2pack(f[3], f[7]), s);
    }
    // digit 1: the lane pair (lane ^ 1); this lane holds digit values 2p and 2p + 1 (its values m and 4 + m)
    const int p = lane & 1;
    uint64_t s_lo[4], s_hi[4];
    had4_signs(2 * p, s_lo);
    had4_signs(2 * p + 1, s_hi);
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const float om = f2lo(o[m]), o4m = f2hi(o[m]);
        const float q0 = __shfl_xor_sync(0xFFFFFFFFu, om, 1), q1 = __shfl_xor_sync(0xFFFFFFFFu, o4m, 1);
        const float a = p ? q0 : om, b = p ? q1 : o4m, c = p ? om : q0, d = p ? o4m : q1;
        // outputs 2p (value m, low lane) and 2p + 1 (value 4 + m, high lane): the same operands, their own signs
        uint64_t sp[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) sp[j] = (s_lo[j] & 0xFFFFFFFFull) | (s_hi[j] & 0xFFFFFFFF00000000ull);
        const uint64_t y = had4x2(f2pack(a, a), f2pack(b, b), f2pack(c, c), f2pack(d, d), sp);
        f[m] = f2lo(y);
        f[4 + m] = f2hi(y);
    }
    // digit 2: lanes that differ in bits 1-2; output d2 of this lane's quad, values i and i + 1 as a pair
    const int d2 = (lane >> 1) & 3, base2 = lane & ~6;
    had4_signs(d2, s);
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
        uint64_t v4[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
            v4[k] = f2pack(__shfl_sync(0xFFFFFFFFu, f[i], base2 | (k << 1)),
                           __shfl_sync(0xFFFFFFFFu, f[i + 1], base2 | (k << 1)));
        const uint64_t y = had4x2(v4[0], v4[1], v4[2], v4[3], s);
        f[i] = f2lo(y);
        f[i + 1] = f2hi(y);
    }
    // digit 3: lanes that differ in bits 3-4, then the exact scaling by 1/16
    const int d3 = (lane >> 3) & 3, base3 = lane & ~24;
    had4_signs(d3, s);
    const uint64_t sixteenth = f2pack(0.0625f, 0.0625f);
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
        uint64_t v4[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
            v4[k] = f2pack(__shfl_sync(0xFFFFFFFFu, f[i], base3 | (k << 3)),
                           __shfl_sync(0xFFFFFFFFu, f[i + 1], base3 | (k << 3)));
        const uint64_t y = mul2(had4x2(v4[0], v4[1], v4[2], v4[3], s), sixteenth);
        f[i] = f2lo(y);
        f[i + 1] = f2hi(y);
    }
}

// ROT: every chunk rotated in place, the row's absmax taken on the rotated float values (as the shared-memory
// kernel does), each value then held as bf16(value) -- what the quantiser divides
template <int NCH>
__device__ __forceinline__ float rotate_chunks(uint4 (&v)[NCH], int lane) {
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
        const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
        float f[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            f[2 * k] = bf_lo(w[k]);
            f[2 * k + 1] = bf_hi(w[k]);
        }
        hadamard256(f, lane);
#pragma unroll
        for (int k = 0; k < 8; ++k) amax = fmaxf(amax, fabsf(f[k]));
        v[j] = make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
    }
    return amax;
}

template <int PRE, int NCH, int WPR, bool ROT>
__device__ __forceinline__ void quant_rows_reg_body(const __nv_bfloat16 *__restrict__ x,
                                                    const __nv_bfloat16 *__restrict__ s1,
                                                    const __nv_bfloat16 *__restrict__ sh,
                                                    const __nv_bfloat16 *__restrict__ gelu, int8_t *__restrict__ q,
                                                    float *__restrict__ scale_out, int64_t rows,
                                                    int64_t rows_per_group, int64_t pf) {
    constexpr int K = 256 * NCH * WPR;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    allow_dependents();
    // launched as a programmatic dependent: the previous kernel's writes (x, and its reads of q / scale_out) are
    // complete past this point, which precedes every global access
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if constexpr (WPR == 1 && NCH <= 8) {
        // the next row waits in shared memory (cp.async), not in registers: each lane reads back and refills only
        // its own 16-byte slots, so the refill needs no synchronisation, and the kernel fits three CTAs per SM
        __shared__ __align__(16) uint4 nxt[8][NCH][32];
        const int64_t nw = static_cast<int64_t>(gridDim.x) * 8;
        int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + warp;
        uint4 v[NCH];
        if (row < rows) {
#pragma unroll
            for (int j = 0; j < NCH; ++j)
                cp_async16(&nxt[warp][j][lane], reinterpret_cast<const uint4 *>(x + row * K) + 32 * j + lane);
        }
        cp_async_commit();
        for (; row < rows; row += nw) {
            cp_async_wait<0>();
#pragma unroll
            for (int j = 0; j < NCH; ++j) v[j] = nxt[warp][j][lane];
            const int64_t nrow = row + nw;
            if (nrow < rows) {
#pragma unroll
                for (int j = 0; j < NCH; ++j)
                    cp_async16(&nxt[warp][j][lane], reinterpret_cast<const uint4 *>(x + nrow * K) + 32 * j + lane);
            }
            cp_async_commit();
            // past the staged next row, pull row nrow + pf into L2 (K x 2 bytes, 16-byte aligned)
            if (pf > 0 && lane == 0 && nrow + pf < rows)
                asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(x + (nrow + pf) * K),
                             "r"(static_cast<uint32_t>(K * 2)) : "memory");
            quant_pre<PRE, NCH>(v, s1, sh, gelu, (row / rows_per_group) * K, lane);
            float amax = ROT ? rotate_chunks<NCH>(v, lane) : chunk_amax<NCH>(v);
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, off));
            amax = fminf(amax, 3.38953139e38f);
            const float scale = fmaxf(div_full(amax, 127.0f), 1.0e-30f);
            if (lane == 0) scale_out[row] = scale;
            quant_store<NCH>(v, r16(scale), reinterpret_cast<uint2 *>(q + row * K), lane);
        }
    } else {
        constexpr int ROWS_PER_CTA = 8 / WPR;
        __shared__ float red[8];
        const int seg = warp % WPR;  // this warp's segment of its row
        const int64_t n_groups = (rows + ROWS_PER_CTA - 1) / ROWS_PER_CTA;
        for (int64_t rg = blockIdx.x; rg < n_groups; rg += gridDim.x) {
            const int64_t row = rg * ROWS_PER_CTA + warp / WPR;
            const bool live = row < rows;
            uint4 v[NCH];
            const int64_t off = static_cast<int64_t>(seg) * (K / WPR);  // element offset of the segment in the row
            float amax = 0.f;
            if (live) {
                const uint4 *xr = reinterpret_cast<const uint4 *>(x + row * K + off);
#pragma unroll
                for (int j = 0; j < NCH; ++j) v[j] = __ldg(xr + 32 * j + lane);
                quant_pre<PRE, NCH>(v, s1, sh, gelu, (row / rows_per_group) * K + off, lane);
                amax = ROT ? rotate_chunks<NCH>(v, lane) : chunk_amax<NCH>(v);
            }
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
            if constexpr (WPR > 1) {
                if (lane == 0) red[warp] = amax;
                __syncthreads();
                const int w0 = warp - seg;
#pragma unroll
                for (int w = 0; w < WPR; ++w) amax = fmaxf(amax, red[w0 + w]);
                __syncthreads();  // red is written again by the next row group
            }
            if (live) {
                amax = fminf(amax, 3.38953139e38f);
                const float scale = fmaxf(div_full(amax, 127.0f), 1.0e-30f);
                if (lane == 0 && seg == 0) scale_out[row] = scale;
                quant_store<NCH>(v, r16(scale), reinterpret_cast<uint2 *>(q + row * K + off), lane);
            }
        }
    }
}

template <int PRE, int NCH, int WPR, bool ROT = false>
__global__ void __launch_bounds__(256) quant_rows_reg_kernel(const __nv_bfloat16 *__restrict__ x,
                                                             const __nv_bfloat16 *__restrict__ s1,
                                                             const __nv_bfloat16 *__restrict__ sh,
                                                             const __nv_bfloat16 *__restrict__ gelu,
                                                             int8_t *__restrict__ q, float *__restrict__ scale_out,
                                                             int64_t rows, int64_t rows_per_group, int64_t pf) {
    quant_rows_reg_body<PRE, NCH, WPR, ROT>(x, s1, sh, gelu, q, scale_out, rows, rows_per_group, pf);
}

// The plain pipelined case (no rotation, one warp per row, K <= 2048) with three CTAs per SM: the next row waits in
// shared memory, which leaves the registers for 24 warps per SM.
template <int PRE, int NCH>
__global__ void __launch_bounds__(256, 3) quant_rows_plain_kernel(const __nv_bfloat16 *__restrict__ x,
                                                                  const __nv_bfloat16 *__restrict__ s1,
                                                                  const __nv_bfloat16 *__restrict__ sh,
                                                                  const __nv_bfloat16 *__restrict__ gelu,
                                                                  int8_t *__restrict__ q, float *__restrict__ scale_out,
                                                                  int64_t rows, int64_t rows_per_group, int64_t pf) {
    quant_rows_reg_body<PRE, NCH, 1, false>(x, s1, sh, gelu, q, scale_out, rows, rows_per_group, pf);
}

// The quantiser with the pending LayerNorm + modulate (pre 3) and no rotation, K = 512 * NV: ln_modulate_kernel's
// structure (one row per 128-thread CTA in PyTorch's vectorised layout, the same Welford order, persistent with the
// next row's loads in flight) with a quantising epilogue instead of the bf16 store: o = bf16(bf16(n * s1) + shift)
// as there, then the row's absmax over the CTA, scale = max(amax / 127, 1e-30) (div.full) and
// q = clamp(rint(bf16(o / bf16(scale)))), 4 int8 per thread-vector store.
template <int NV>
__global__ void __launch_bounds__(128) quant_lnmod_kernel(const __nv_bfloat16 *__restrict__ x,
                                                          const __nv_bfloat16 *__restrict__ s1,
                                                          const __nv_bfloat16 *__restrict__ sh,
                                                          int8_t *__restrict__ q, float *__restrict__ scale_out,
                                                          int64_t rows, int64_t K, int64_t rows_per_group, float eps,
                                                          int pf) {
    __shared__ float red[16];
    __shared__ float amax_w[2][4];
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    allow_dependents();
    int64_t row = blockIdx.x;
    if (row >= rows) return;
    asm volatile("griddepcontrol.wait;" ::: "memory");  // a programmatic dependent, as quant_rows_reg_body
    uint2 raw[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) raw[j] = __ldg(reinterpret_cast<const uint2 *>(x + row * K) + t + 128 * j);
    uint2 sraw[NV], hraw[NV];
    int64_t cached_group = -1;
    int parity = 0;
    for (; row < rows; row += gridDim.x, parity ^= 1) {
        float v[NV * 4];
#pragma unroll
        for (int j = 0; j < NV; ++j) unpack4(raw[j], v + 4 * j);
        const int64_t nrow = row + gridDim.x;
        if (nrow < rows) {
#pragma unroll
            for (int j = 0; j < NV; ++j) raw[j] = __ldg(reinterpret_cast<const uint2 *>(x + nrow * K) + t + 128 * j);
        }
        if (pf > 0 && t == 0 && nrow + pf < rows)  // as in ln_modulate_kernel
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(x + (nrow + pf) * K),
                         "r"(static_cast<uint32_t>(K * 2)) : "memory");
        const int64_t group = static_cast<int64_t>(static_cast<uint32_t>(row) / static_cast<uint32_t>(rows_per_group));
        if (group != cached_group) {
            cached_group = group;
#pragma unroll
            for (int j = 0; j < NV; ++j) {
                sraw[j] = __ldg(reinterpret_cast<const uint2 *>(s1 + group * K) + t + 128 * j);
                hraw[j] = __ldg(reinterpret_cast<const uint2 *>(sh + group * K) + t + 128 * j);
            }
        }
        float mu, var;
        ln_stats_n<NV * 4>(v, K, mu, var, red);
        const float rstd = rsqrt_approx(__fadd_rn(var, eps));
        uint32_t ob[NV * 2];  // the modulated row as bf16 pairs
        uint32_t am2 = 0;     // its largest |value| in each bf16 lane
        const uint64_t neg_mu = f2pack(-mu, -mu), rstd2 = f2pack(rstd, rstd);  // as in ln_modulate_kernel
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const uint64_t a = mul2(add2(f2pack(v[4 * j], v[4 * j + 1]), neg_mu), rstd2);
            const uint64_t b = mul2(add2(f2pack(v[4 * j + 2], v[4 * j + 3]), neg_mu), rstd2);
            ob[2 * j] = mod_bf16x2(pack2(f2lo(a), f2hi(a)), sraw[j].x, hraw[j].x);
            ob[2 * j + 1] = mod_bf16x2(pack2(f2lo(b), f2hi(b)), sraw[j].y, hraw[j].y);
            am2 = bf2_max(am2, bf2_max(bf2_abs(ob[2 * j]), bf2_abs(ob[2 * j + 1])));
        }
        float amax = fmaxf(bf_lo(am2), bf_hi(am2));
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, off));
        if (lane == 0) amax_w[parity][warp] = amax;  // two buffers: a fast warp may reach the next row first
        __syncthreads();
        amax = fmaxf(fmaxf(amax_w[parity][0], amax_w[parity][1]), fmaxf(amax_w[parity][2], amax_w[parity][3]));
        amax = fminf(amax, 3.38953139e38f);
        const float scale = fmaxf(div_full(amax, 127.0f), 1.0e-30f);
        if (t == 0) scale_out[row] = scale;
        const float sb = r16(scale);
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int64_t c = static_cast<int64_t>(t + 128 * j) * 4;
            *reinterpret_cast<uint32_t *>(q + row * K + c) = quant_quad(ob[2 * j], ob[2 * j + 1], sb);
        }
        // (red[] of the next row's statistics is written only after this row's ln_stats barriers, and amax_w
        // alternates between two buffers, so one barrier per row suffices)
    }
}

// The quantiser with the pending LayerNorm + modulate and the ConvRot rotation (pre 3, rotate), K = 512 * NV: the
// row's statistics and modulation as quant_lnmod_kernel computes them (PyTorch's vectorised layout over the 128
// threads), the modulated bf16 row then handed to the four warps through shared memory, each warp rotating whole
// 256-value groups in registers (hadamard256, 8 values per lane; groups w, w + 4, ...), the row's absmax over the
// rotated float values, each value quantised from its bf16 rounding -- bit for bit quant_rows_kernel<3, true>, whose
// four shared-memory Hadamard stages and one row per CTA this replaces.
template <int NV>
__global__ void __launch_bounds__(128) quant_lnmod_rot_kernel(const __nv_bfloat16 *__restrict__ x,
                                                              const __nv_bfloat16 *__restrict__ s1,
                                                              const __nv_bfloat16 *__restrict__ sh,
                                                              int8_t *__restrict__ q, float *__restrict__ scale_out,
                                                              int64_t rows, int64_t K, int64_t rows_per_group,
                                                              float eps, int pf) {
    constexpr int G = 2 * NV;        // 256-value groups of the row
    constexpr int NG = (G + 3) / 4;  // groups per warp (warps past the last group of a round take none)
    __shared__ __align__(16) uint32_t srow[NV * 256];  // the modulated row as bf16 pairs
    __shared__ float red[2][16];
    __shared__ float amax_w[2][4];
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    allow_dependents();
    int64_t row = blockIdx.x;
    if (row >= rows) return;
    asm volatile("griddepcontrol.wait;" ::: "memory");  // a programmatic dependent, as quant_rows_reg_body
    uint2 raw[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) raw[j] = __ldg(reinterpret_cast<const uint2 *>(x + row * K) + t + 128 * j);
    int parity = 0;
    for (; row < rows; row += gridDim.x, parity ^= 1) {
        float v[NV * 4];
#pragma unroll
        for (int j = 0; j < NV; ++j) unpack4(raw[j], v + 4 * j);
        const int64_t nrow = row + gridDim.x;
        if (nrow < rows) {
#pragma unroll
            for (int j = 0; j < NV; ++j) raw[j] = __ldg(reinterpret_cast<const uint2 *>(x + nrow * K) + t + 128 * j);
        }
        if (pf > 0 && t == 0 && nrow + pf < rows)  // as in ln_modulate_kernel
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(x + (nrow + pf) * K),
                         "r"(static_cast<uint32_t>(K * 2)) : "memory");
        const int64_t goff =
            static_cast<int64_t>(static_cast<uint32_t>(row) / static_cast<uint32_t>(rows_per_group)) * K;
        float mu, var;
        ln_stats_n<NV * 4>(v, K, mu, var, red[parity]);
        const float rstd = rsqrt_approx(__fadd_rn(var, eps));
        const uint64_t neg_mu = f2pack(-mu, -mu), rstd2 = f2pack(rstd, rstd);
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const uint2 sr = __ldg(reinterpret_cast<const uint2 *>(s1 + goff) + t + 128 * j);
            const uint2 hr = __ldg(reinterpret_cast<const uint2 *>(sh + goff) + t + 128 * j);
            const uint64_t a = mul2(add2(f2pack(v[4 * j], v[4 * j + 1]), neg_mu), rstd2);
            const uint64_t b = mul2(add2(f2pack(v[4 * j + 2], v[4 * j + 3]), neg_mu), rstd2);
            // values 4t + 512 j .. + 3 of the row: words 2t + 256 j, + 1
            *reinterpret_cast<uint2 *>(srow + 2 * t + 256 * j) =
                make_uint2(mod_bf16x2(pack2(f2lo(a), f2hi(a)), sr.x, hr.x),
                           mod_bf16x2(pack2(f2lo(b), f2hi(b)), sr.y, hr.y));
        }
        __syncthreads();  // the modulated row is in shared memory
        uint4 vv[NG];
        float amax = 0.f;
#pragma unroll
        for (int gi = 0; gi < NG; ++gi) {
            const int g = warp + 4 * gi;
            if (g < G) {  // uniform over the warp: every lane takes part in the shuffles
                vv[gi] = reinterpret_cast<const uint4 *>(srow)[32 * g + lane];  // values 256 g + 8 lane .. + 7
                const uint32_t w[4] = {vv[gi].x, vv[gi].y, vv[gi].z, vv[gi].w};
                float f[8];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    f[2 * k] = bf_lo(w[k]);
                    f[2 * k + 1] = bf_hi(w[k]);
                }
                hadamard256(f, lane);
#pragma unroll
                for (int k = 0; k < 8; ++k) amax = fmaxf(amax, fabsf(f[k]));
                vv[gi] = make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
            }
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, off));
        if (lane == 0) amax_w[parity][warp] = amax;
        __syncthreads();  // every warp's absmax; every warp is done reading this row from shared memory
        amax = fmaxf(fmaxf(amax_w[parity][0], amax_w[parity][1]), fmaxf(amax_w[parity][2], amax_w[parity][3]));
        amax = fminf(amax, 3.38953139e38f);
        const float scale = fmaxf(div_full(amax, 127.0f), 1.0e-30f);
        if (t == 0) scale_out[row] = scale;
        const float sb = r16(scale);
#pragma unroll
        for (int gi = 0; gi < NG; ++gi) {
            const int g = warp + 4 * gi;
            if (g < G)
                *reinterpret_cast<uint2 *>(q + row * K + 256 * g + 8 * lane) =
                    make_uint2(quant_quad(vv[gi].x, vv[gi].y, sb), quant_quad(vv[gi].z, vv[gi].w, sb));
        }
    }
}

// L2 prefetch distance of the row-walking quantisers past their staged next row, in quarter waves
// (WEIGHTFERRY_QUANT_PREFETCH 0 - 9, 0 = off; default 1)
int row_prefetch() {
    static const int w = env_digit("WEIGHTFERRY_QUANT_PREFETCH", 1);
    return w;
}

template <int NV, bool ROT>
constexpr auto quant_lnmod_kernel_for() {
    if constexpr (ROT) return quant_lnmod_rot_kernel<NV>;
    else return quant_lnmod_kernel<NV>;
}

template <int NV, bool ROT = false>
int launch_quant_lnmod(const void *x, const void *s1, const void *sh, int8_t *q, float *sc, int64_t rows, int64_t K,
                       int64_t rpg, float eps, cudaStream_t s) {
    constexpr auto kern = quant_lnmod_kernel_for<NV, ROT>();
    const int g = persistent_grid<kern>(128, 0, rows);
    const int pf = static_cast<int>(static_cast<int64_t>(g) * row_prefetch() / 4);
    const cudaError_t e = launch_pdl(kern, g, 128, s, static_cast<const __nv_bfloat16 *>(x),
                                     static_cast<const __nv_bfloat16 *>(s1), static_cast<const __nv_bfloat16 *>(sh),
                                     q, sc, rows, K, rpg, eps, pf);
    return static_cast<int>(e != cudaSuccess ? e : cudaGetLastError());
}

// the register quantiser's kernel for (PRE, NCH, WPR, ROT): the pipelined plain kernel where it applies
template <int PRE, int NCH, int WPR, bool ROT>
constexpr auto quant_reg_kernel() {
    if constexpr (!ROT && WPR == 1 && NCH <= 8) return quant_rows_plain_kernel<PRE, NCH>;
    else return quant_rows_reg_kernel<PRE, NCH, WPR, ROT>;
}

template <int PRE, int NCH, int WPR, bool ROT = false>
int launch_quant_reg(const void *x, const void *s1, const void *sh, const void *gelu, int8_t *q, float *sc,
                     int64_t rows, int64_t rpg, cudaStream_t s) {
    constexpr auto kern = quant_reg_kernel<PRE, NCH, WPR, ROT>();
    const int64_t groups = (rows + (8 / WPR) - 1) / (8 / WPR);
    // the pipelined variant walks about two rows per warp; the others one row group per CTA while they fit
    const int64_t want = (WPR == 1 && NCH <= 8) ? (groups + 1) / 2 : groups;
    const int grid = static_cast<int>(std::min<int64_t>(want, wave_ctas<kern>(256, 0)));
    // the pipelined kernel's L2 prefetch distance: a quarter of its warps' rows per quarter wave of row_prefetch()
    const int64_t pf = (WPR == 1 && NCH <= 8) ? static_cast<int64_t>(grid) * 8 * row_prefetch() / 4 : 0;
    const cudaError_t e = launch_pdl(kern, grid, 256, s, static_cast<const __nv_bfloat16 *>(x),
                                     static_cast<const __nv_bfloat16 *>(s1), static_cast<const __nv_bfloat16 *>(sh),
                                     static_cast<const __nv_bfloat16 *>(gelu), q, sc, rows, rpg, pf);
    return static_cast<int>(e != cudaSuccess ? e : cudaGetLastError());
}

// The rotated (ConvRot) register kernel for K = 256 * n up to 3072 (one warp per row), K = 4096 / 5120 / 6144 (four
// warps per row) or K = 2048 * n from 8192 to 32768 (eight warps per row) -- each warp's segment a whole number of
// 256-wide groups, which the rotation keeps within a warp -- or false.
template <int PRE>
bool quant_rot_dispatch(int64_t K, const void *x, const void *s1, const void *sh, const void *gelu, int8_t *q,
                        float *sc, int64_t rows, int64_t rpg, cudaStream_t s, int *rc) {
#define WF_QT(N, W) do { *rc = launch_quant_reg<PRE, N, W, true>(x, s1, sh, gelu, q, sc, rows, rpg, s); return true; } while (0)
    if (K % 256 != 0) return false;
    switch (K / 256) {
        case 1: WF_QT(1, 1); case 2: WF_QT(2, 1); case 3: WF_QT(3, 1); case 4: WF_QT(4, 1); case 5: WF_QT(5, 1);
        case 6: WF_QT(6, 1); case 8: WF_QT(8, 1); case 10: WF_QT(10, 1); case 12: WF_QT(12, 1); case 16: WF_QT(4, 4);
        case 20: WF_QT(5, 4); case 24: WF_QT(6, 4);
        default: break;
    }
    if (K % 2048 != 0) return false;
    switch (K / 2048) {
        case 4: WF_QT(4, 8); case 5: WF_QT(5, 8); case 6: WF_QT(6, 8); case 8: WF_QT(8, 8); case 10: WF_QT(10, 8);
        case 12: WF_QT(12, 8); case 16: WF_QT(16, 8);
        default: return false;
    }
#undef WF_QT
}

// The register kernel's (NCH, WPR) for K, or false: one warp per row up to K = 3072, four for K = 4096 / 5120 / 6144
// (a fifth to a fifth less time than one warp holding the whole row: fewer registers per thread, more rows in
// flight), eight from K = 8192 to 32768.
template <int PRE>
bool quant_reg_dispatch(int64_t K, const void *x, const void *s1, const void *sh, const void *gelu, int8_t *q,
                        float *sc, int64_t rows, int64_t rpg, cudaStream_t s, int *rc) {
#define WF_QR(N, W) do { *rc = launch_quant_reg<PRE, N, W>(x, s1, sh, gelu, q, sc, rows, rpg, s); return true; } while (0)
    if (K % 256 != 0) return false;
    switch (K / 256) {
        case 1: WF_QR(1, 1); case 2: WF_QR(2, 1); case 3: WF_QR(3, 1); case 4: WF_QR(4, 1); case 5: WF_QR(5, 1);
        case 6: WF_QR(6, 1); case 8: WF_QR(8, 1); case 10: WF_QR(10, 1); case 12: WF_QR(12, 1);
        case 16: WF_QR(4, 4); case 20: WF_QR(5, 4); case 24: WF_QR(6, 4);
        default: break;
    }
    if (K % 2048 != 0) return false;
    switch (K / 2048) {
        case 4: WF_QR(4, 8); case 5: WF_QR(5, 8); case 6: WF_QR(6, 8); case 8: WF_QR(8, 8); case 10: WF_QR(10, 8);
        case 12: WF_QR(12, 8); case 16: WF_QR(16, 8);
        default: return false;
    }
#undef WF_QR
}

template <int PRE, bool ROT>
int launch_quant(const void *x, const void *s1, const void *sh, const void *gelu, int8_t *q, float *sc, int64_t rows,
                 int64_t K, int64_t rpg, float eps, cudaStream_t s) {
    const size_t smem = static_cast<size_t>(K) * 4;
    auto kern = quant_rows_kernel<PRE, ROT>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return static_cast<int>(e);
    }
    kern<<<static_cast<unsigned>(rows), 128, smem, s>>>(
        static_cast<const __nv_bfloat16 *>(x), static_cast<const __nv_bfloat16 *>(s1),
        static_cast<const __nv_bfloat16 *>(sh), static_cast<const __nv_bfloat16 *>(gelu), q, sc, K, rpg, eps);
    return static_cast<int>(cudaGetLastError());
}

int grid_for(int64_t items, int per_block) {
    const int64_t want = (items + per_block - 1) / per_block;
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, static_cast<int64_t>(device_sm_count()) * 16)));
}

bool al(const void *p, int a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

}  // namespace
}  // namespace wf

using namespace wf;

extern "C" WF_API int wf_modulate(const void *x, const void *s1, const void *shift, void *out, int64_t rows,
                                 int64_t d, int64_t rows_per_group, wf_stream_t stream) {
    if (rows < 0 || d <= 0 || rows_per_group <= 0 || d % 8 != 0) return WF_ERR_ARG;
    if (rows == 0) return WF_OK;
    if (!x || !s1 || !shift || !out || !al(x, 16) || !al(s1, 16) || !al(shift, 16) || !al(out, 16)) return WF_ERR_ARG;
    int rc = check_device();
    if (rc != WF_OK) return rc;
    const int64_t n_vec = rows * d / 8;
    modulate_kernel<<<grid_for(n_vec, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4 *>(x), static_cast<const __nv_bfloat16 *>(s1),
        static_cast<const __nv_bfloat16 *>(shift), static_cast<uint4 *>(out), n_vec, d, rows_per_group);
    return static_cast<int>(cudaGetLastError());
}

extern "C" WF_API int wf_gated_residual(const void *x, const void *gate, const void *o, void *out, int64_t rows,
                                        int64_t d, int64_t rows_per_group, wf_stream_t stream) {
    if (rows < 0 || d <= 0 || rows_per_group <= 0 || d % 8 != 0) return WF_ERR_ARG;
    if (rows == 0) return WF_OK;
    if (!x || !gate || !o || !out || !al(x, 16) || !al(gate, 16) || !al(o, 16) || !al(out, 16)) return WF_ERR_ARG;
    int rc = check_device();
    if (rc != WF_OK) return rc;
    const int64_t n_vec = rows * d / 8;
    gated_residual_kernel<<<grid_for(n_vec, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4 *>(x), static_cast<const __nv_bfloat16 *>(gate), static_cast<const uint4 *>(o),
        static_cast<uint4 *>(out), n_vec, d, rows_per_group);
    return static_cast<int>(cudaGetLastError());
}

namespace wf {
namespace {
// L2 prefetch distance of ln_modulate_kernel past its register prefetch, in quarter waves of the persistent grid
// (WEIGHTFERRY_LN_PREFETCH 0 - 9, 0 = off; default 1. Measured on 8192 rows of 2048: 12.6 us at a quarter wave,
// 13.1 us without)
int ln_prefetch() {
    static const int w = env_digit("WEIGHTFERRY_LN_PREFETCH", 1);
    return w;
}
}  // namespace
}  // namespace wf

extern "C" WF_API int wf_ln_modulate(const void *x, const void *s1, const void *shift, void *out, int64_t rows,
                                    int64_t K, int64_t rows_per_group, float eps, wf_stream_t stream) {
    if (rows < 0 || rows > INT32_MAX || K <= 0 || K % 512 != 0 || K > 512 * 16 || rows_per_group <= 0)
        return WF_ERR_ARG;
    if (rows == 0) return WF_OK;
    if (!x || !s1 || !shift || !out || !al(x, 8) || !al(s1, 8) || !al(shift, 8) || !al(out, 8)) return WF_ERR_ARG;
    int rc = check_device();
    if (rc != WF_OK) return rc;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    auto X = static_cast<const __nv_bfloat16 *>(x);
    auto S = static_cast<const __nv_bfloat16 *>(s1);
    auto H = static_cast<const __nv_bfloat16 *>(shift);
    auto O = static_cast<__nv_bfloat16 *>(out);
    cudaError_t e = cudaSuccess;
#define WF_LN(NV)                                                                                        \
    case NV: {                                                                                           \
        const int g = persistent_grid<ln_modulate_kernel<NV>>(128, 0, rows);                             \
        const int pf = static_cast<int>(static_cast<int64_t>(g) * ln_prefetch() / 4);                    \
        e = launch_pdl(ln_modulate_kernel<NV>, g, 128, s, X, S, H, O, rows, K, rows_per_group, eps, pf);  \
        break;                                                                                           \
    }
    switch (K / 512) {
        WF_LN(1) WF_LN(2) WF_LN(3) WF_LN(4) WF_LN(5) WF_LN(6) WF_LN(8) WF_LN(10) WF_LN(12) WF_LN(16)
#undef WF_LN
        default: return WF_ERR_UNSUPPORTED;
    }
    return static_cast<int>(e != cudaSuccess ? e : cudaGetLastError());
}

extern "C" WF_API int wf_rms_norm_128(const void *x, const void *w, int w_dtype, void *out, int64_t n_rows, float eps,
                                     wf_stream_t stream) {
    if (n_rows < 0 || w_dtype < WF_F16 || w_dtype > WF_F32) return WF_ERR_ARG;
    if (n_rows == 0) return WF_OK;
    if (!x || !w || !out || !al(x, 8) || !al(out, 8) || !al(w, dtype_size(w_dtype))) return WF_ERR_ARG;
    int rc = check_device();
    if (rc != WF_OK) return rc;
    rms128_kernel<<<grid_for(n_rows, 8), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<const __nv_bfloat16 *>(x), w, w_dtype, static_cast<__nv_bfloat16 *>(out), n_rows, eps);
    return static_cast<int>(cudaGetLastError());
}

namespace wf {
namespace {

// WEIGHTFERRY_ROPE_V1=1 keeps the shared-memory kernel (rms_rope_kernel) for every launch
bool rope_v2() {
    static const bool v2 = env_digit("WEIGHTFERRY_ROPE_V1", 0) != 1;
    return v2;
}

// rows per half-warp in flight in rms_rope_v2_kernel (WEIGHTFERRY_ROPE_ROWS 2 / 4 / 8; measured on q and k of
// (2, 4096, 16, 128) before the L2 prefetch: 2 rows 29.0 us, 4 rows 27.4 us, 8 rows 29.0 us)
int rope_rows() {
    static const int r = [] {
        const int d = env_digit("WEIGHTFERRY_ROPE_ROWS", 4);
        return d == 2 || d == 8 ? d : 4;
    }();
    return r;
}

// L2 prefetch distance of rms_rope_v2_kernel in quarter waves of resident CTAs (WEIGHTFERRY_ROPE_PREFETCH 0 - 9,
// 0 = off; default 1. Measured on q and k of (2, 4096, 16, 128): 24.4 us at a quarter wave, 24.7 at a half, 26.0 at
// one wave, 26.6 without, 28 - 30 us at one and a half waves or more: prefetched rows that wait longer in L2 lose)
int rope_prefetch() {
    static const int w = env_digit("WEIGHTFERRY_ROPE_PREFETCH", 1);
    return w;
}

template <int WD, bool F, int R>
cudaError_t rope_v2_launch(cudaLaunchConfig_t &cfg, const RopeTensors &t, int ni, int nt, int hd, int tk,
                           const float *freqs, float eps, int64_t s_tok, int64_t s_d, int64_t s_i, int64_t s_j) {
    const int64_t pf64 = hd <= 256 ? static_cast<int64_t>(rope_prefetch()) *
                                         wave_ctas<rms_rope_v2_kernel<WD, F, R>>(kRope2Warps * 32, 0) * kRope2Warps / 4
                                   : 0;
    const int pf = static_cast<int>(std::min<int64_t>(pf64, INT32_MAX / 2));
    return cudaLaunchKernelEx(&cfg, rms_rope_v2_kernel<WD, F, R>, t, ni, nt, hd, tk, freqs, eps, s_tok, s_d, s_i, s_j,
                              pf);
}

int rope_launch(const RopeTensors &t, int n_tensors, const float *freqs, int64_t f_stride_token, int64_t f_stride_d,
                int64_t f_stride_i, int64_t f_stride_j, int w_dtype, int64_t batch, int64_t tokens, int64_t heads,
                float eps, wf_stream_t stream) {
    if (batch < 0 || tokens < 0 || heads < 0 || w_dtype < WF_F16 || w_dtype > WF_F32) return WF_ERR_ARG;
    if (batch * tokens * heads == 0) return WF_OK;
    if (!freqs || !al(freqs, 4)) return WF_ERR_ARG;
    for (int i = 0; i < n_tensors; ++i)
        if (!t.x[i] || !t.w[i] || !t.out[i] || !al(t.x[i], 16) || !al(t.out[i], 16) || !al(t.w[i], dtype_size(w_dtype)))
            return WF_ERR_ARG;
    int rc = check_device();
    if (rc != WF_OK) return rc;
    const int64_t n_tok = batch * tokens;
    const int64_t blocks =
        (n_tensors * n_tok * ((heads + kRopeHeads - 1) / kRopeHeads) + kRopeWarps - 1) / kRopeWarps;
    const bool f4 = f_stride_j == 1 && f_stride_i == 2 && f_stride_d % 4 == 0 && f_stride_token % 4 == 0 &&
                    al(freqs, 16);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int64_t n_items = n_tensors * n_tok;
    // v2 reads weight pairs as one 4-byte (bf16 / f16) or 8-byte (f32) word
    bool w_pairs = true;
    for (int i = 0; i < n_tensors; ++i) w_pairs = w_pairs && al(t.w[i], 2 * dtype_size(w_dtype));
    if (n_items <= INT32_MAX / 2 && heads <= 65536 && n_tok * heads * 64 <= INT32_MAX && tokens <= INT32_MAX &&
        w_pairs && rope_v2()) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(static_cast<unsigned>((n_items + kRope2Warps - 1) / kRope2Warps), 1, 1);
        cfg.blockDim = dim3(kRope2Warps * 32, 1, 1);
        cfg.stream = s;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr.val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        const int ni = static_cast<int>(n_items), nt = static_cast<int>(n_tok), hd = static_cast<int>(heads),
                  tk = static_cast<int>(tokens);
        cudaError_t e;
#define WF_RV2(WD, F)                                                                                          \
    e = rope_rows() == 4   ? rope_v2_launch<WD, F, 4>(cfg, t, ni, nt, hd, tk, freqs, eps, f_stride_token, f_stride_d, \
                                                      f_stride_i, f_stride_j)                                      \
        : rope_rows() == 8 ? rope_v2_launch<WD, F, 8>(cfg, t, ni, nt, hd, tk, freqs, eps, f_stride_token, f_stride_d, \
                                                      f_stride_i, f_stride_j)                                      \
                           : rope_v2_launch<WD, F, 2>(cfg, t, ni, nt, hd, tk, freqs, eps, f_stride_token, f_stride_d, \
                                                      f_stride_i, f_stride_j)
        if (w_dtype == WF_BF16) {
            if (f4) WF_RV2(WF_BF16, true); else WF_RV2(WF_BF16, false);
        } else if (w_dtype == WF_F16) {
            if (f4) WF_RV2(WF_F16, true); else WF_RV2(WF_F16, false);
        } else {
            if (f4) WF_RV2(WF_F32, true); else WF_RV2(WF_F32, false);
        }
#undef WF_RV2
        return static_cast<int>(e != cudaSuccess ? e : cudaGetLastError());
    }
    constexpr int kT = kRopeWarps * 32;
    if (f4) {
        rms_rope_kernel<true><<<persistent_grid<rms_rope_kernel<true>>(kT, 0, blocks), kT, 0, s>>>(
            t, n_tensors, freqs, w_dtype, n_tok, heads, tokens, eps, f_stride_token, f_stride_d, f_stride_i, f_stride_j);
    } else {
        rms_rope_kernel<false><<<persistent_grid<rms_rope_kernel<false>>(kT, 0, blocks), kT, 0, s>>>(
            t, n_tensors, freqs, w_dtype, n_tok, heads, tokens, eps, f_stride_token, f_stride_d, f_stride_i, f_stride_j);
    }
    return static_cast<int>(cudaGetLastError());
}

}  // namespace
}  // namespace wf

extern "C" WF_API int wf_rms_rope128(const void *x, const float *freqs, int64_t f_stride_token, int64_t f_stride_d,
                                    int64_t f_stride_i, int64_t f_stride_j, const void *w, int w_dtype, void *out,
                                    int64_t batch, int64_t tokens, int64_t heads, float eps, wf_stream_t stream) {
    wf::RopeTensors t{};
    t.x[0] = static_cast<const __nv_bfloat16 *>(x);
    t.w[0] = w;
    t.out[0] = static_cast<__nv_bfloat16 *>(out);
    return wf::rope_launch(t, 1, freqs, f_stride_token, f_stride_d, f_stride_i, f_stride_j, w_dtype, batch, tokens,
                           heads, eps, stream);
}

extern "C" WF_API int wf_rms_rope128_pair(const void *q, const void *k, const float *freqs, int64_t f_stride_token,
                                         int64_t f_stride_d, int64_t f_stride_i, int64_t f_stride_j, const void *wq,
                                         const void *wk, int w_dtype, void *q_out, void *k_out, int64_t batch,
                                         int64_t tokens, int64_t heads, float eps, wf_stream_t stream) {
    wf::RopeTensors t{};
    t.x[0] = static_cast<const __nv_bfloat16 *>(q);
    t.x[1] = static_cast<const __nv_bfloat16 *>(k);
    t.w[0] = wq;
    t.w[1] = wk;
    t.out[0] = static_cast<__nv_bfloat16 *>(q_out);
    t.out[1] = static_cast<__nv_bfloat16 *>(k_out);
    return wf::rope_launch(t, 2, freqs, f_stride_token, f_stride_d, f_stride_i, f_stride_j, w_dtype, batch, tokens,
                           heads, eps, stream);
}

extern "C" WF_API int wf_quant_rows(const void *x, const void *s1, const void *shift, const void *gelu_table,
                                   int8_t *q, float *scale, int64_t rows, int64_t K, int64_t rows_per_group,
                                   float eps, int pre, int rotate, wf_stream_t stream) {
    if (rows < 0 || K <= 0 || K % 4 != 0 || rows_per_group <= 0 || pre < 0 || pre > 3) return WF_ERR_ARG;
    if (rotate && K % 256 != 0) return WF_ERR_ARG;
    if (pre == 3 && (K % 512 != 0 || K > 8192)) return WF_ERR_ARG;
    if (static_cast<size_t>(K) * 4 > 200 * 1024) return WF_ERR_UNSUPPORTED;
    if (rows == 0) return WF_OK;
    if (!x || !q || !scale || !al(x, 8) || !al(q, 4) || !al(scale, 4)) return WF_ERR_ARG;
    if ((pre == 2 || pre == 3) && (!s1 || !shift || !al(s1, 8) || !al(shift, 8))) return WF_ERR_ARG;
    if (pre == 1 && (!gelu_table || !al(gelu_table, 2))) return WF_ERR_ARG;
    int rc = check_device();
    if (rc != WF_OK) return rc;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (!rotate && pre == 3 && rows <= INT32_MAX && al(q, 4)) {
        switch (K / 512) {  // K % 512 == 0 and K <= 8192 were checked above
#define WF_QL(NV) case NV: return launch_quant_lnmod<NV>(x, s1, shift, q, scale, rows, K, rows_per_group, eps, s);
            WF_QL(1) WF_QL(2) WF_QL(3) WF_QL(4) WF_QL(5) WF_QL(6) WF_QL(7) WF_QL(8)
            WF_QL(9) WF_QL(10) WF_QL(11) WF_QL(12) WF_QL(13) WF_QL(14) WF_QL(15) WF_QL(16)
#undef WF_QL
            default: break;
        }
    }
    if (rotate && pre == 3 && rows <= INT32_MAX && al(q, 8)) {
        switch (K / 512) {  // K % 512 == 0 and K <= 8192 were checked above
#define WF_QLR(NV) case NV: return launch_quant_lnmod<NV, true>(x, s1, shift, q, scale, rows, K, rows_per_group, eps, s);
            WF_QLR(1) WF_QLR(2) WF_QLR(3) WF_QLR(4) WF_QLR(5) WF_QLR(6) WF_QLR(7) WF_QLR(8)
            WF_QLR(9) WF_QLR(10) WF_QLR(11) WF_QLR(12) WF_QLR(13) WF_QLR(14) WF_QLR(15) WF_QLR(16)
#undef WF_QLR
            default: break;
        }
    }
    if (rotate && pre != 3 && al(x, 16) && al(q, 8) && (pre != 2 || (al(s1, 16) && al(shift, 16)))) {
        bool done = false;
        switch (pre) {
            case 0: done = quant_rot_dispatch<0>(K, x, s1, shift, gelu_table, q, scale, rows, rows_per_group, s, &rc); break;
            case 1: done = quant_rot_dispatch<1>(K, x, s1, shift, gelu_table, q, scale, rows, rows_per_group, s, &rc); break;
            default: done = quant_rot_dispatch<2>(K, x, s1, shift, gelu_table, q, scale, rows, rows_per_group, s, &rc); break;
        }
        if (done) return rc;
    }
    if (!rotate && pre != 3 && al(x, 16) && al(q, 8) && (pre != 2 || (al(s1, 16) && al(shift, 16)))) {
        bool done = false;
        switch (pre) {
            case 0: done = quant_reg_dispatch<0>(K, x, s1, shift, gelu_table, q, scale, rows, rows_per_group, s, &rc); break;
            case 1: done = quant_reg_dispatch<1>(K, x, s1, shift, gelu_table, q, scale, rows, rows_per_group, s, &rc); break;
            default: done = quant_reg_dispatch<2>(K, x, s1, shift, gelu_table, q, scale, rows, rows_per_group, s, &rc); break;
        }
        if (done) return rc;
    }
#define WF_Q(P, R) return launch_quant<P, R>(x, s1, shift, gelu_table, q, scale, rows, K, rows_per_group, eps, s)
    if (rotate) {
        switch (pre) { case 0: WF_Q(0, true); case 1: WF_Q(1, true); case 2: WF_Q(2, true); default: WF_Q(3, true); }
    } else {
        switch (pre) { case 0: WF_Q(0, false); case 1: WF_Q(1, false); case 2: WF_Q(2, false); default: WF_Q(3, false); }
    }
#undef WF_Q
}
