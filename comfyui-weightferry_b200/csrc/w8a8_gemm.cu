// W8A8 linear for sm_100a: y[m, n] = bf16( float(acc[m, n]) * x_s[m] * w_s[n] ), acc = sum_k xq[m, k] * wq[n, k]
// (int8 x int8 -> int32), the GEMM and epilogue behind the reference's int8 linear (enhancers/fused_int8.py:191-206,
// which calls comfy_kitchen's compiled CUTLASS kernel; the arithmetic here is this library's own, with the epilogue
// order written below).
//
// Blackwell-native structure, one persistent CTA per SM (320 threads):
//   warp 8      TMA producer: 128x128 tiles of xq and 256x128 tiles of wq (K-major, 128-byte swizzle) into a
//               4-stage shared-memory ring, completion counted on an mbarrier per stage;
//   warp 9      MMA issuer: one thread issues tcgen05.mma.cta_group::1.kind::i8 (M=128, N=256, K=32; 4 per stage)
//               with int32 accumulation in tensor memory; tcgen05.commit releases each stage and, per tile, hands
//               the accumulator to the epilogue. Two 256-column accumulators (all 512 TMEM columns) let tile i+1's
//               MMAs run while tile i is written out;
//   warps 0..7  epilogue: warp w reads TMEM lanes 32(w%4)..+31 (one output row per thread), columns
//               128(w/4)..+127, with tcgen05.ld (the next 32 columns in flight while the current ones are
//               converted), y = bf16_rn((float(acc) * x_s[m]) * w_s[n]) (two float32 products, each rounded to
//               nearest; w_s read with warp-uniform loads). Each 32 x 32 bf16 chunk goes to a 2 KB shared-memory
//               buffer of the warp (64-byte swizzle, two per warp) and leaves with one TMA tensor store, which
//               also clips rows >= M and columns >= N; the optional raw int32 copy is written directly.
// The residual variant (wf_w8a8_gemm_residual) adds the block's gated residual in the same epilogue:
// out = bf16_rn(float(x[m, n]) + float(gate[m / rows_per_group, n]) * float(y)) with y the bf16 value above (one
// float32 product and one float32 sum, each rounded to nearest) -- the bits of the GEMM followed by PyTorch's bf16
// addcmul(x, gate, y). Each lane bulk-prefetches its row's residual span into L2 while the tile's MMAs run; residual
// and gate then come in with plain 16-byte loads, one 32-column chunk ahead of its TMEM read. out may be x.
// Every mbarrier wait is bounded in time (about 2 s): on expiry the CTA records an error code (read with
// wf_w8a8_gemm_status), stops issuing work, waits (bounded) for its own copies and MMAs in flight, frees its tensor
// memory and returns. Every TMA load here is a plain per-CTA load of this GPU's own memory.

#include "wf_common.cuh"

#include <cuda.h>

#include <atomic>
#include <cstdlib>
#include <mutex>
#include <utility>

namespace wf {
namespace {

constexpr int BM = 128, BN = 256, BK = 128, STAGES = 4;
constexpr int A_STAGE = BM * BK;  // 16 KB
constexpr int B_STAGE = BN * BK;  // 32 KB
constexpr int STAGE_BYTES = A_STAGE + B_STAGE;
constexpr int THREADS = 320;
constexpr int EPI_THREADS = 256;
constexpr int TMEM_COLS = 512;
constexpr int OUT_BYTES = 8 * 2 * 2048;  // per epilogue warp two 32 x 32 bf16 output chunks
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + OUT_BYTES + 1024 + 256;  // ring, output chunks, slack, barriers
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// instruction descriptor of kind::i8: D int32 (bits 4-5 = 2), A and B signed int8 (bits 7-9, 10-12 = 1), both
// K-major, N >> 3 at bits 17-22, M >> 4 at bits 24-28
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((BN >> 3) << 17) | ((BM >> 4) << 24);

__device__ int g_gemm_status;  // 0 ok; 1 producer wait expired; 2 MMA wait expired; 3 epilogue wait expired
// limit of the pipeline waits (the producer's, the MMA issuer's and the epilogue's); a test shortens it so that a wait
// runs out and the abort path is exercised (wf_w8a8_gemm_set_wait_limit). The drain waits of the abort path keep
// kWaitLimitNs.
__device__ unsigned long long g_wait_limit_ns = kWaitLimitNs;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint32_t a, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t a, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(a), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_complete_tx(uint32_t a, uint32_t bytes) {  // bytes that will never arrive
    asm volatile("mbarrier.complete_tx.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(bytes) : "memory");
}
// bounded wait (kWaitLimitNs) for the phase of the given parity, for the drains of the abort path
__device__ __forceinline__ void mbar_drain_wait(uint32_t a, uint32_t parity);
__device__ __forceinline__ void mbar_arrive(uint32_t a) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(a) : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {  // an arrive on a barrier anywhere in the cluster
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t a, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ void mbar_drain_wait(uint32_t a, uint32_t parity) {
    if (mbar_try(a, parity)) return;  // the usual case; a read of the global timer costs ~0.2 us
    const uint64_t t0 = global_ns();
    while (!mbar_try(a, parity) && global_ns() - t0 < kWaitLimitNs) {
    }
}

// Wait for the phase of the given parity, at most g_wait_limit_ns; gives up early when another role aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t a, uint32_t parity, volatile int *abort_flag, int code) {
    if (mbar_try(a, parity)) return true;
    const uint64_t limit = g_wait_limit_ns;
    // try_wait suspends for a while inside each try, so 32 tries can outlast a short wait: a shortened limit (the
    // test hook) is checked after every try
    const int spins = limit < 1000000ull ? 1 : 32;
    const uint64_t t0 = global_ns();
    while (true) {
#pragma unroll 1
        for (int i = 0; i < spins; ++i)
            if (mbar_try(a, parity)) return true;
        if (*abort_flag) return false;
        if (global_ns() - t0 > limit) {
            *abort_flag = 1;
            atomicCAS(&g_gemm_status, 0, code);
            return false;
        }
    }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int c0, int c1, uint32_t mbar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(mbar)
        : "memory");
}

// shared-memory matrix descriptor: K-major, 128-byte swizzle, rows 128 B apart, 8-row groups 1024 B apart
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);        // start address
    d |= static_cast<uint64_t>(1u) << 16;                      // leading byte offset (16 B; unused when swizzled)
    d |= static_cast<uint64_t>(1024u >> 4) << 32;              // stride byte offset
    d |= static_cast<uint64_t>(1u) << 46;                      // descriptor version (Blackwell)
    d |= static_cast<uint64_t>(2u) << 61;                      // SWIZZLE_128B
    return d;
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(kIdesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t mbar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar)
                 : "memory");
}

// Programmatic dependent launch: the kernel is launched while the previous kernel of the stream (the quantiser that
// writes xq / xs) may still run, so its set-up (barriers, tensor memory, cluster sync) overlaps that kernel's tail;
// every thread waits here for the previous grid's completion and memory before it touches global memory. Without a
// programmatic launch this returns at once.
__device__ __forceinline__ void wait_prior_grid() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// tcgen05.ld of 32 consecutive columns of this thread's lane; the registers are valid only after tmem_wait32 on
// the same array (the wait names them as operands, so no use can be scheduled before it)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tmem_wait32(uint32_t (&r)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                   "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                   "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, uint32_t src, int c0, int c1) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(src)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
// every output store of this thread has finished reading its shared-memory source (the stores themselves complete
// with the grid, before any later kernel of the stream -- or a programmatic dependent past griddepcontrol.wait --
// can read the output)
__device__ __forceinline__ void bulk_wait_read_all() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Output tile `tile` -> (tile row, tile column). group_m == 0: tiles walk down the M direction first (column by
// column); group_m > 0: bands of group_m tile rows, each walked column by column, so that the tiles in flight at once
// share fewer operand rows and columns.
__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int group_m, int &mi, int &ni) {
    if (group_m <= 0) {
        mi = tile % tiles_m;
        ni = tile / tiles_m;
        return;
    }
    const int band = tile / (group_m * tiles_n);
    const int first = band * group_m;
    const int rows = min(tiles_m - first, group_m);
    const int r = tile - band * group_m * tiles_n;
    mi = first + r % rows;
    ni = r / rows;
}

// w_s of 32 output columns starting at col0 (a multiple of 32; N is a multiple of 8, so each group of 8 columns is
// wholly inside or wholly outside [0, N)); same address in every lane
struct Ws32 {
    float4 v[8];
};
__device__ __forceinline__ void load_ws32(Ws32 &w, const float *__restrict__ ws, int col0, int N) {
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        if (col0 + 8 * g < N) {
            w.v[2 * g] = __ldg(reinterpret_cast<const float4 *>(ws + col0 + 8 * g));
            w.v[2 * g + 1] = __ldg(reinterpret_cast<const float4 *>(ws + col0 + 8 * g + 4));
        } else {
            w.v[2 * g] = w.v[2 * g + 1] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
}

// the block's residual operand of the residual epilogue (resid == nullptr: the plain GEMM)
struct ResidualArgs {
    const __nv_bfloat16 *resid;  // [M, N] row-major
    const __nv_bfloat16 *gate;   // [ceil(M / rows_per_group), N] row-major
    int rows_per_group;
};

// 32 residual and gate values of this lane's row (row < M) at columns col0 .. col0 + 31 (16-byte groups past N are 0)
struct Res32 {
    uint4 r[4], g[4];
};
__device__ __forceinline__ void load_res32(Res32 &v, const ResidualArgs &res, int row, int col0, int M, int N) {
    const size_t rbase = static_cast<size_t>(row) * N, gbase = static_cast<size_t>(row / res.rows_per_group) * N;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int col = col0 + 8 * q;
        if (row < M && col < N) {
            v.r[q] = __ldg(reinterpret_cast<const uint4 *>(res.resid + rbase + col));
            v.g[q] = __ldg(reinterpret_cast<const uint4 *>(res.gate + gbase + col));
        } else {
            v.r[q] = v.g[q] = make_uint4(0u, 0u, 0u, 0u);
        }
    }
}

// bf16x2 -> two floats (exact)
__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xFFFF0000u); }

// this lane's residual span of a tile (128 columns from col0, clipped at N) into L2 ahead of its use
__device__ __forceinline__ void prefetch_res_l2(const ResidualArgs &res, int row, int col0, int M, int N) {
    if (row >= M || col0 >= N) return;
    const uint32_t bytes = static_cast<uint32_t>(min(128, N - col0)) * 2u;  // a multiple of 16 (N % 8 == 0)
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(res.resid + static_cast<size_t>(row) * N + col0),
                 "r"(bytes)
                 : "memory");
}

// 32 accumulators of this lane's row -> bf16 in the warp's chunk buffer `buf` (32 rows x 64 bytes, 64-byte swizzle:
// the 16-byte piece j of row r sits at piece j ^ ((r >> 1) & 3)), then one TMA store of the 32 x 32 chunk whose
// top-left element is (row0, col0). The buffer is reused every second chunk: lane 0 first waits until the store
// issued from it two chunks ago has read it.
template <bool RES>
__device__ __forceinline__ void emit_chunk(const uint32_t (&r)[32], const Ws32 &w, float xsr, const Res32 &rv,
                                           uint32_t buf, int lane, const CUtensorMap *tma_y, int row0, int col0) {
    uint32_t p[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const float4 wv = w.v[j >> 1];
        const float w0 = (j & 1) ? wv.z : wv.x, w1 = (j & 1) ? wv.w : wv.y;
        const float a0 = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[2 * j])), xsr), w0);
        const float a1 = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[2 * j + 1])), xsr), w1);
        __nv_bfloat162 h = __floats2bfloat162_rn(a0, a1);
        uint32_t y2 = *reinterpret_cast<uint32_t *>(&h);
        if (RES) {
            const uint4 rq = rv.r[j >> 2], gq = rv.g[j >> 2];
            const uint32_t rw = (j & 3) == 0 ? rq.x : (j & 3) == 1 ? rq.y : (j & 3) == 2 ? rq.z : rq.w;
            const uint32_t gw = (j & 3) == 0 ? gq.x : (j & 3) == 1 ? gq.y : (j & 3) == 2 ? gq.z : gq.w;
            const float o0 = __fadd_rn(bf_lo(rw), __fmul_rn(bf_lo(gw), bf_lo(y2)));
            const float o1 = __fadd_rn(bf_hi(rw), __fmul_rn(bf_hi(gw), bf_hi(y2)));
            __nv_bfloat162 o = __floats2bfloat162_rn(o0, o1);
            y2 = *reinterpret_cast<uint32_t *>(&o);
        }
        p[j] = y2;
    }
    if (lane == 0) bulk_wait_read1();
    __syncwarp();
    const uint32_t row_addr = buf + 64u * static_cast<uint32_t>(lane);
    const uint32_t sw = (static_cast<uint32_t>(lane) >> 1) & 3u;
#pragma unroll
    for (int j = 0; j < 4; ++j)
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(row_addr + 16u * (static_cast<uint32_t>(j) ^ sw)),
                     "r"(p[4 * j]), "r"(p[4 * j + 1]), "r"(p[4 * j + 2]), "r"(p[4 * j + 3])
                     : "memory");
    fence_async_smem();  // the generic-proxy writes become visible to the TMA engine
    __syncwarp();
    if (lane == 0) {
        tma_store_2d(tma_y, buf, col0, row0);
        bulk_commit();
    }
}

// the raw int32 accumulators of this lane's row (debug copy), columns >= N skipped
__device__ __forceinline__ void store_acc_chunk(const uint32_t (&r)[32], int32_t *acc_out, int row, int col0, int N) {
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        const int col = col0 + 8 * g;
        if (col >= N) break;
        int4 *dst = reinterpret_cast<int4 *>(acc_out + static_cast<size_t>(row) * N + col);
        dst[0] = make_int4(r[8 * g], r[8 * g + 1], r[8 * g + 2], r[8 * g + 3]);
        dst[1] = make_int4(r[8 * g + 4], r[8 * g + 5], r[8 * g + 6], r[8 * g + 7]);
    }
}

// One epilogue warp's share of an accumulator tile: 32 rows (TMEM lanes of taddr) x 128 columns from col0, four
// 32-column tcgen05.ld with the next one in flight while the current chunk is converted and stored. The accumulator
// is released (tcgen05 fence, then an arrive on `release`, a cluster address when PAIR) as soon as its last
// columns are in registers. `chunk` counts this warp's chunks and picks the buffer.
template <bool PAIR, bool RES>
__device__ __forceinline__ void epilogue_rows(uint32_t taddr, uint32_t release, const float *__restrict__ ws,
                                              float xsr, uint32_t out_smem, uint32_t &chunk, int lane,
                                              const CUtensorMap *tma_y, int32_t *acc_out, const ResidualArgs &res,
                                              int row0, int col0, int M, int N) {
    const int row = row0 + lane;
    const bool dbg = acc_out != nullptr && row < M;
    uint32_t ra[32], rb[32];
    Ws32 w;
    Res32 rv;
    load_ws32(w, ws, col0, N);
    if (RES) load_res32(rv, res, row, col0, M, N);
    tmem_ld32(taddr, ra);
    tmem_wait32(ra);
    tmem_ld32(taddr + 32, rb);
    emit_chunk<RES>(ra, w, xsr, rv, out_smem + 2048u * (chunk++ & 1u), lane, tma_y, row0, col0);
    if (dbg) store_acc_chunk(ra, acc_out, row, col0, N);
    load_ws32(w, ws, col0 + 32, N);
    if (RES) load_res32(rv, res, row, col0 + 32, M, N);
    tmem_wait32(rb);
    tmem_ld32(taddr + 64, ra);
    emit_chunk<RES>(rb, w, xsr, rv, out_smem + 2048u * (chunk++ & 1u), lane, tma_y, row0, col0 + 32);
    if (dbg) store_acc_chunk(rb, acc_out, row, col0 + 32, N);
    load_ws32(w, ws, col0 + 64, N);
    if (RES) load_res32(rv, res, row, col0 + 64, M, N);
    tmem_wait32(ra);
    tmem_ld32(taddr + 96, rb);
    emit_chunk<RES>(ra, w, xsr, rv, out_smem + 2048u * (chunk++ & 1u), lane, tma_y, row0, col0 + 64);
    if (dbg) store_acc_chunk(ra, acc_out, row, col0 + 64, N);
    load_ws32(w, ws, col0 + 96, N);
    if (RES) load_res32(rv, res, row, col0 + 96, M, N);
    tmem_wait32(rb);
    fence_before();
    if (PAIR)
        mbar_arrive_cluster(release);  // the accumulator may be overwritten
    else
        mbar_arrive(release);
    emit_chunk<RES>(rb, w, xsr, rv, out_smem + 2048u * (chunk++ & 1u), lane, tma_y, row0, col0 + 96);
    if (dbg) store_acc_chunk(rb, acc_out, row, col0 + 96, N);
}

template <bool RES>
__global__ void __launch_bounds__(THREADS, 1)
w8a8_gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                 const __grid_constant__ CUtensorMap tma_y, const float *__restrict__ xs,
                 const float *__restrict__ ws, int32_t *__restrict__ acc_out, ResidualArgs res, int M, int N,
                 int K, int group_m) {
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned ring (the 128-byte swizzle pattern repeats every 8 rows of 128 bytes), then the epilogue
    // warps' output chunks (4 KB per warp), then the barriers
    uint8_t *ring = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *out_chunks = ring + STAGES * STAGE_BYTES;
    uint64_t *bars = reinterpret_cast<uint64_t *>(out_chunks + OUT_BYTES);
    // bars: full[0..3], empty[0..3], tmem_full[0..1], tmem_empty[0..1], drain
    __shared__ uint32_t s_tmem_base;
    __shared__ int s_abort;
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + STAGES), tfull0 = smem_u32(bars + 2 * STAGES),
                   tempty0 = smem_u32(bars + 2 * STAGES + 2), drain = smem_u32(bars + 2 * STAGES + 4);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const int tiles_m = (M + BM - 1) / BM, tiles_n = (N + BN - 1) / BN;
    const int n_tiles = tiles_m * tiles_n;
    const int kb_count = (K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        s_abort = 0;
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(tfull0 + 8 * b, 1);
            mbar_init(tempty0 + 8 * b, EPI_THREADS);
        }
        mbar_init(drain, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 9) {  // the MMA warp owns the tensor memory
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(&s_tmem_base)), "r"(TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem_base = s_tmem_base;
    wait_prior_grid();
    volatile int *abort_flag = &s_abort;

    if (warp == 8) {
        // ------------------------------------------------------------------------------------ TMA producer
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tma_a)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tma_b)) : "memory");
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued_phase[STAGES];
            bool pending[STAGES];
            for (int s = 0; s < STAGES; ++s) pending[s] = false, issued_phase[s] = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
                int mi, ni;
                tile_coords(tile, tiles_m, tiles_n, group_m, mi, ni);
                const int m0 = mi * BM, n0 = ni * BN;
                for (int kb = 0; kb < kb_count; ++kb) {
                    if (!mbar_wait(empty0 + 8 * stage, phase ^ 1u, abort_flag, 1)) { ok = false; break; }
                    const uint32_t fb = full0 + 8 * stage;
                    mbar_expect_tx(fb, STAGE_BYTES);
                    const uint32_t a_dst = smem_u32(ring + stage * STAGE_BYTES);
                    tma_load_2d(a_dst, &tma_a, kb * BK, m0, fb);
                    tma_load_2d(a_dst + A_STAGE, &tma_b, kb * BK, n0, fb);
                    pending[stage] = true;
                    issued_phase[stage] = phase;
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
            }
            if (!ok) {
                // drain: every issued load lands before the CTA leaves (bounded)
                for (int s = 0; s < STAGES; ++s)
                    if (pending[s]) mbar_drain_wait(full0 + 8 * s, issued_phase[s]);
            }
        }
    } else if (warp == 9) {
        // ------------------------------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
                if (!mbar_wait(tempty0 + 8 * acc, acc_phase ^ 1u, abort_flag, 2)) { ok = false; break; }
                fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                for (int kb = 0; kb < kb_count; ++kb) {
                    if (!mbar_wait(full0 + 8 * stage, phase, abort_flag, 2)) { ok = false; break; }
                    fence_after();
                    const uint32_t a_addr = smem_u32(ring + stage * STAGE_BYTES);
                    const uint32_t b_addr = a_addr + A_STAGE;
#pragma unroll
                    for (int kk = 0; kk < BK / 32; ++kk)
                        mma_i8(d_tmem, smem_desc(a_addr + 32 * kk), smem_desc(b_addr + 32 * kk),
                               (kb | kk) != 0 ? 1u : 0u);
                    mma_commit(empty0 + 8 * stage);  // the stage is free once these MMAs have read it
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
                if (!ok) break;
                mma_commit(tfull0 + 8 * acc);  // the accumulator is complete
                if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
            }
            // every MMA issued by this thread has finished before the tensor memory is released
            mma_commit(drain);
            mbar_drain_wait(drain, 0);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------------------------------ epilogue (warps 0-7)
        const int quarter = warp & 3, half = warp >> 2;
        const uint32_t out_smem = smem_u32(out_chunks + warp * 4096);
        if (threadIdx.x == 0)
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tma_y)) : "memory");
        int acc = 0;
        uint32_t acc_phase = 0, chunk = 0;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
            int mi, ni;
            tile_coords(tile, tiles_m, tiles_n, group_m, mi, ni);
            const int m0 = mi * BM, n0 = ni * BN;
            const int row0 = m0 + quarter * 32;
            const float xsr = row0 + lane < M ? __ldg(xs + row0 + lane) : 0.f;
            if (RES) prefetch_res_l2(res, row0 + lane, n0 + half * 128, M, N);
            if (!mbar_wait(tfull0 + 8 * acc, acc_phase, abort_flag, 3)) break;
            fence_after();
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                   static_cast<uint32_t>(acc * BN + half * 128);
            epilogue_rows<false, RES>(taddr, tempty0 + 8 * acc, ws, xsr, out_smem, chunk, lane, &tma_y, acc_out, res,
                                      row0, n0 + half * 128, M, N);
            if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
        }
        if (lane == 0) bulk_wait_read_all();  // this warp's output stores have finished with its shared memory
        __syncwarp();
    }
    fence_before();
    __syncthreads();
    fence_after();
    if (warp == 9) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                     : "memory");
    }
}

// ---------------------------------------------------------------------------------------------- 2-SM kernel
// The same GEMM with one 256 x 256 output tile per pair of CTAs (a cluster of 2 on neighbouring SMs):
// tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 32) issued by one thread of the even CTA reads rows 0..127 of the
// A tile and columns 0..127 of the B tile from the even CTA's shared memory and the other halves from the odd CTA's
// (same offsets); each CTA's tensor memory holds its 128 accumulator rows x 256 columns. Per CTA a stage is 32 KB
// (128 rows of xq + 128 rows of wq), so 6 stages fit and each SM pulls a third less from L2 than the 1-CTA kernel.
// Each CTA's TMA loads count their bytes on the even CTA's full barrier (the .cta_group::2 form); the even CTA's
// MMA thread signals both CTAs' empty / accumulator-ready barriers with one plain commit per CTA, and both CTAs'
// epilogues release an accumulator on the even CTA's barrier.
constexpr int S2 = 6;                       // stages
constexpr int A2_STAGE = 128 * BK;          // 16 KB: this CTA's 128 rows of xq
constexpr int B2_STAGE = 128 * BK;          // 16 KB: this CTA's 128 rows of wq
constexpr int STAGE2 = A2_STAGE + B2_STAGE; // 32 KB
constexpr int SMEM2_BYTES = S2 * STAGE2 + OUT_BYTES + 1024 + 256;
constexpr uint32_t kIdesc2 = (2u << 4) | (1u << 7) | (1u << 10) | ((256u >> 3) << 17) | ((256u >> 4) << 24);
constexpr uint32_t kPeerBitMask = 0xFEFFFFFFu;  // clears the CTA-rank bit of a cluster shared address

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap *map, int c0, int c1,
                                                 uint32_t leader_mbar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(leader_mbar)
        : "memory");
}
__device__ __forceinline__ void mma_i8_pair(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(kIdesc2), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void mma_commit_pair(uint32_t cluster_mbar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_mbar)
                 : "memory");
}

template <bool RES>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
w8a8_gemm_2sm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                     const __grid_constant__ CUtensorMap tma_y, const float *__restrict__ xs,
                     const float *__restrict__ ws, int32_t *__restrict__ acc_out, ResidualArgs res, int M, int N,
                     int K, int group_m) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *ring = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *out_chunks = ring + S2 * STAGE2;
    uint64_t *bars = reinterpret_cast<uint64_t *>(out_chunks + OUT_BYTES);
    // bars: full[0..5] (used in the even CTA), empty[0..5], tmem_full[0..1], tmem_empty[0..1] (even CTA), drain
    __shared__ uint32_t s_tmem_base;
    __shared__ int s_abort;
    __shared__ int s_issued[2];  // stage loads issued by this CTA's producer; [1] in the even CTA: the odd CTA's
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + S2), tfull0 = smem_u32(bars + 2 * S2),
                   tempty0 = smem_u32(bars + 2 * S2 + 2), drain = smem_u32(bars + 2 * S2 + 4);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const uint32_t peer = rank ^ 1u;

    const int tiles_m = (M + 255) / 256, tiles_n = (N + 255) / 256;
    const int n_tiles = tiles_m * tiles_n;
    const int kb_count = (K + BK - 1) / BK;
    const int cluster_id = blockIdx.x >> 1, n_clusters = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        s_abort = 0;
        s_issued[0] = s_issued[1] = 0;
        for (int s = 0; s < S2; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(tfull0 + 8 * b, 1);
            mbar_init(tempty0 + 8 * b, 2 * EPI_THREADS);
        }
        mbar_init(drain, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 9) {  // the MMA warp of each CTA allocates (the pair's allocation: same warp, same offset)
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(&s_tmem_base)), "r"(TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    fence_before();
    cluster_sync();  // barriers initialised and tensor memory allocated in both CTAs
    fence_after();
    const uint32_t tmem_base = s_tmem_base;
    wait_prior_grid();
    volatile int *abort_flag = &s_abort;

    if (warp == 8) {
        // ------------------------------------------------------------------------------------ TMA producer
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tma_a)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tma_b)) : "memory");
            int stage = 0;
            uint32_t phase = 0;
            int issued = 0;
            bool ok = true;
            for (int tile = cluster_id; tile < n_tiles && ok; tile += n_clusters) {
                int mi, ni;
                tile_coords(tile, tiles_m, tiles_n, group_m, mi, ni);
                const int m0 = mi * 256 + static_cast<int>(rank) * 128;
                const int n0 = ni * 256 + static_cast<int>(rank) * 128;
                for (int kb = 0; kb < kb_count; ++kb) {
                    if (!mbar_wait(empty0 + 8 * stage, phase ^ 1u, abort_flag, 1)) { ok = false; break; }
                    const uint32_t leader_full = (full0 + 8 * stage) & kPeerBitMask;
                    if (rank == 0) mbar_expect_tx(full0 + 8 * stage, 2 * STAGE2);
                    const uint32_t a_dst = smem_u32(ring + stage * STAGE2);
                    tma_load_2d_pair(a_dst, &tma_a, kb * BK, m0, leader_full);
                    tma_load_2d_pair(a_dst + A2_STAGE, &tma_b, kb * BK, n0, leader_full);
                    ++issued;
                    if (++stage == S2) { stage = 0; phase ^= 1u; }
                }
            }
            // the count goes to the even CTA, whose full barriers count both CTAs' bytes: it drains after the pair
            // has stopped (below)
            if (rank == 0) {
                s_issued[0] = issued;
            } else {
                const uint32_t dst = map_to_rank(smem_u32(&s_issued[1]), 0);
                asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(dst), "r"(issued) : "memory");
            }
        }
    } else if (warp == 9) {
        // ------------------------------------------------------------------------------------ MMA issuer (even CTA)
        if (lane == 0 && rank == 0) {
            const uint32_t empty_peer = map_to_rank(empty0, peer), tfull_peer = map_to_rank(tfull0, peer);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int tile = cluster_id; tile < n_tiles && ok; tile += n_clusters) {
                if (!mbar_wait(tempty0 + 8 * acc, acc_phase ^ 1u, abort_flag, 2)) { ok = false; break; }
                fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                for (int kb = 0; kb < kb_count; ++kb) {
                    if (!mbar_wait(full0 + 8 * stage, phase, abort_flag, 2)) { ok = false; break; }
                    fence_after();
                    const uint32_t a_addr = smem_u32(ring + stage * STAGE2);
                    const uint32_t b_addr = a_addr + A2_STAGE;
#pragma unroll
                    for (int kk = 0; kk < BK / 32; ++kk)
                        mma_i8_pair(d_tmem, smem_desc(a_addr + 32 * kk), smem_desc(b_addr + 32 * kk),
                                    (kb | kk) != 0 ? 1u : 0u);
                    mma_commit_pair(empty0 + 8 * stage);       // this CTA's stage is free ...
                    mma_commit_pair(empty_peer + 8 * stage);   // ... and the other CTA's
                    if (++stage == S2) { stage = 0; phase ^= 1u; }
                }
                if (!ok) break;
                mma_commit_pair(tfull0 + 8 * acc);
                mma_commit_pair(tfull_peer + 8 * acc);
                if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
            }
            mma_commit_pair(drain);
            mbar_drain_wait(drain, 0);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------------------------------ epilogue (warps 0-7)
        const int quarter = warp & 3, half = warp >> 2;
        const uint32_t tempty_leader = map_to_rank(tempty0, 0);
        const uint32_t out_smem = smem_u32(out_chunks + warp * 4096);
        if (threadIdx.x == 0)
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tma_y)) : "memory");
        int acc = 0;
        uint32_t acc_phase = 0, chunk = 0;
        for (int tile = cluster_id; tile < n_tiles; tile += n_clusters) {
            int mi, ni;
            tile_coords(tile, tiles_m, tiles_n, group_m, mi, ni);
            const int m0 = mi * 256 + static_cast<int>(rank) * 128, n0 = ni * 256;
            const int row0 = m0 + quarter * 32;
            const float xsr = row0 + lane < M ? __ldg(xs + row0 + lane) : 0.f;
            if (RES) prefetch_res_l2(res, row0 + lane, n0 + half * 128, M, N);
            if (!mbar_wait(tfull0 + 8 * acc, acc_phase, abort_flag, 3)) break;
            fence_after();
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                   static_cast<uint32_t>(acc * BN + half * 128);
            // the pair's accumulator is released on the even CTA's barrier
            epilogue_rows<true, RES>(taddr, tempty_leader + 8 * acc, ws, xsr, out_smem, chunk, lane, &tma_y, acc_out,
                                     res, row0, n0 + half * 128, M, N);
            if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
        }
        if (lane == 0) bulk_wait_read_all();
        __syncwarp();
    }
    fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs stopped issuing; the odd CTA's load count is in the even CTA's s_issued[1]
    if (rank == 0 && warp == 8 && lane == 0) {
        // Drain: every stage load either CTA issued lands before either CTA leaves. Stage s's full barrier counts
        // both CTAs' bytes of a use; only its last issued use can be outstanding (a producer reuses a stage only
        // after the MMA consumed the previous use, which needed that use complete). A use that one CTA issued and
        // the other did not (it stopped first) gets the missing half: the arrive with the odd CTA's bytes expected,
        // or the even CTA's expectation of the odd CTA's bytes cancelled. Without an abort every use was consumed and
        // each wait returns at once.
        const int n_even = s_issued[0], n_odd = s_issued[1];
        const int last = max(n_even, n_odd);
        for (int s = 0; s < S2 && s < last; ++s) {
            const int u = s + ((last - 1 - s) / S2) * S2;
            const uint32_t bar = full0 + 8 * s;
            if (u >= n_even)
                mbar_expect_tx(bar, STAGE2);
            else if (u >= n_odd)
                mbar_complete_tx(bar, STAGE2);
            mbar_drain_wait(bar, static_cast<uint32_t>(u / S2) & 1u);
        }
    }
    cluster_sync();  // no CTA leaves (or frees tensor memory) while loads into it or the pair's MMAs may still run
    fence_after();
    if (warp == 9) {
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                     : "memory");
    }
}

// ---------------------------------------------------------------------------------------------- host
using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
    static EncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    });
    return fn;
}

// WEIGHTFERRY_PDL=0 launches the GEMM as a plain kernel instead of a programmatic dependent
bool use_pdl() {
    static const bool pdl = env_digit("WEIGHTFERRY_PDL", 1) != 0;
    return pdl;
}

// a kernel launch as a programmatic dependent of the previous one in the stream (WEIGHTFERRY_PDL=0: a plain launch)
template <typename... KArgs, typename... Args>
cudaError_t launch_dependent(void (*kern)(KArgs...), int grid, int threads, size_t smem, cudaStream_t stream,
                             Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
    cfg.blockDim = dim3(static_cast<unsigned>(threads), 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = use_pdl() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// WEIGHTFERRY_W8A8_GROUP_M: tile rows per band of the tile order (0 or unset: down M first)
int tile_group_m() {
    static const int g = [] {
        const char *v = getenv("WEIGHTFERRY_W8A8_GROUP_M");
        return v != nullptr ? std::max(0, atoi(v)) : 0;
    }();
    return g;
}

// WEIGHTFERRY_W8A8_1SM=1 keeps every problem on the one-CTA kernel (the pair kernel is used for m > 128 otherwise)
bool use_pair_kernel() {
    static const bool pair = env_digit("WEIGHTFERRY_W8A8_1SM", 0) != 1;
    return pair;
}

// a [rows, K] int8 K-major matrix as a TMA map with boxes of box_rows x 128 bytes, 128-byte swizzle, zero fill
int make_map(CUtensorMap *map, const void *base, int rows, int K, int box_rows) {
    EncodeTiled enc = encoder();
    if (enc == nullptr) return WF_ERR_DEVICE;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(K)};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(BK), static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? WF_OK : WF_ERR_ARG;
}

// y [rows, N] bf16 row-major as a TMA store map with 32 x 32 boxes and 64-byte swizzle (N % 8 == 0, base 16-aligned)
int make_out_map(CUtensorMap *map, void *base, int rows, int N) {
    EncodeTiled enc = encoder();
    if (enc == nullptr) return WF_ERR_DEVICE;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(N) * 2};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? WF_OK : WF_ERR_ARG;
}

// one launch of the pair kernel (m > 128) or the one-CTA kernel, with or without the residual epilogue
template <bool RES>
int launch(const CUtensorMap &ma, const void *wq, const CUtensorMap &my, const float *xs, const float *ws,
           int32_t *acc_out, const ResidualArgs &res, int64_t M, int64_t N, int64_t K, int dev, cudaStream_t stream) {
    int rc;
    if (M > BM && use_pair_kernel()) {
        // pairs of CTAs, 256 x 256 tiles: each CTA loads 128 rows of xq and 128 rows of wq per stage
        CUtensorMap mb2;
        if ((rc = make_map(&mb2, wq, static_cast<int>(N), static_cast<int>(K), 128)) != WF_OK) return rc;
        static std::atomic<int> clusters[64];  // any host thread may launch first
        if (clusters[dev].load(std::memory_order_acquire) == 0) {
            cudaError_t e = cudaFuncSetAttribute(w8a8_gemm_2sm_kernel<RES>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM2_BYTES);
            if (e != cudaSuccess) return static_cast<int>(e);
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(2 * device_sm_count(), 1, 1);
            cfg.blockDim = dim3(THREADS, 1, 1);
            cfg.dynamicSmemBytes = SMEM2_BYTES;
            cudaLaunchAttribute attr;
            attr.id = cudaLaunchAttributeClusterDimension;
            attr.val.clusterDim.x = 2;
            attr.val.clusterDim.y = 1;
            attr.val.clusterDim.z = 1;
            cfg.attrs = &attr;
            cfg.numAttrs = 1;
            int n = 0;
            e = cudaOccupancyMaxActiveClusters(&n, w8a8_gemm_2sm_kernel<RES>, &cfg);
            if (e != cudaSuccess) return static_cast<int>(e);
            clusters[dev].store(std::max(n, 1), std::memory_order_release);
        }
        const int64_t tiles = ((M + 255) / 256) * ((N + 255) / 256);
        const int grid =
            2 * static_cast<int>(std::min<int64_t>(tiles, clusters[dev].load(std::memory_order_acquire)));
        const cudaError_t e = launch_dependent(w8a8_gemm_2sm_kernel<RES>, grid, THREADS, SMEM2_BYTES, stream, ma, mb2,
                                               my, xs, ws, acc_out, res, static_cast<int>(M), static_cast<int>(N),
                                               static_cast<int>(K), tile_group_m());
        return static_cast<int>(e != cudaSuccess ? e : cudaGetLastError());
    }
    CUtensorMap mb;
    if ((rc = make_map(&mb, wq, static_cast<int>(N), static_cast<int>(K), BN)) != WF_OK) return rc;
    static std::atomic<bool> attr_set[64];
    if (!attr_set[dev].load(std::memory_order_acquire)) {
        cudaError_t e = cudaFuncSetAttribute(w8a8_gemm_kernel<RES>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             SMEM_BYTES);
        if (e != cudaSuccess) return static_cast<int>(e);
        attr_set[dev].store(true, std::memory_order_release);
    }
    const int64_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
    const int grid = static_cast<int>(std::min<int64_t>(tiles, device_sm_count()));
    const cudaError_t e = launch_dependent(w8a8_gemm_kernel<RES>, grid, THREADS, SMEM_BYTES, stream, ma, mb, my, xs, ws,
                                           acc_out, res, static_cast<int>(M), static_cast<int>(N), static_cast<int>(K),
                                           tile_group_m());
    return static_cast<int>(e != cudaSuccess ? e : cudaGetLastError());
}

bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

}  // namespace

int w8a8_gemm_launch(const int8_t *xq, const int8_t *wq, const float *xs, const float *ws, __nv_bfloat16 *y,
                     int32_t *acc_out, const __nv_bfloat16 *resid, const __nv_bfloat16 *gate, int64_t rows_per_group,
                     int64_t M, int64_t N, int64_t K, cudaStream_t stream) {
    if (M <= 0 || N <= 0 || K <= 0) return (M == 0 || N == 0) ? WF_OK : WF_ERR_ARG;
    if (M > (1 << 30) || N > (1 << 30) || K > (1 << 30)) return WF_ERR_ARG;
    if (K % 16 != 0 || N % 8 != 0) return WF_ERR_ARG;  // TMA row pitches of xq, wq and y
    if (!xq || !wq || !xs || !ws || !y || !aligned(xq, 16) || !aligned(wq, 16) || !aligned(ws, 16) ||
        !aligned(xs, 4) || !aligned(y, 16) || (acc_out && !aligned(acc_out, 16)))
        return WF_ERR_ARG;
    const bool res_on = resid != nullptr;
    if (res_on && (!gate || !aligned(resid, 16) || !aligned(gate, 16) || rows_per_group <= 0)) return WF_ERR_ARG;
    int rc = check_device();
    if (rc != WF_OK) return rc;
    CUtensorMap ma, my;
    if ((rc = make_map(&ma, xq, static_cast<int>(M), static_cast<int>(K), BM)) != WF_OK) return rc;
    if ((rc = make_out_map(&my, y, static_cast<int>(M), static_cast<int>(N))) != WF_OK) return rc;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return WF_ERR_DEVICE;
    ResidualArgs res{resid, gate, static_cast<int>(std::min<int64_t>(rows_per_group, 1 << 30))};
    return res_on ? launch<true>(ma, wq, my, xs, ws, acc_out, res, M, N, K, dev, stream)
                  : launch<false>(ma, wq, my, xs, ws, acc_out, res, M, N, K, dev, stream);
}

int w8a8_gemm_status(int *status) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_gemm_status, sizeof(int));
    if (e != cudaSuccess) return static_cast<int>(e);
    if (v != 0) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_gemm_status, &zero, sizeof(int));
    }
    *status = v;
    return WF_OK;
}

}  // namespace wf

extern "C" WF_API int wf_w8a8_gemm(const int8_t *xq, const int8_t *wq, const float *xs, const float *ws, void *y,
                                  int32_t *acc_dbg, int64_t m, int64_t n, int64_t k, wf_stream_t stream) {
    return wf::w8a8_gemm_launch(xq, wq, xs, ws, static_cast<__nv_bfloat16 *>(y), acc_dbg, nullptr, nullptr, 1, m, n,
                                k, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" WF_API int wf_w8a8_gemm_residual(const int8_t *xq, const int8_t *wq, const float *xs, const float *ws,
                                           const void *resid, const void *gate, int64_t rows_per_group, void *out,
                                           int64_t m, int64_t n, int64_t k, wf_stream_t stream) {
    if (resid == nullptr) return WF_ERR_ARG;
    return wf::w8a8_gemm_launch(xq, wq, xs, ws, static_cast<__nv_bfloat16 *>(out), nullptr,
                                static_cast<const __nv_bfloat16 *>(resid), static_cast<const __nv_bfloat16 *>(gate),
                                rows_per_group, m, n, k, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" WF_API int wf_w8a8_gemm_set_wait_limit(uint64_t limit_ns) {
    if (limit_ns == 0 || limit_ns > wf::kWaitLimitNs) limit_ns = wf::kWaitLimitNs;
    const unsigned long long v = limit_ns;
    return static_cast<int>(cudaMemcpyToSymbol(wf::g_wait_limit_ns, &v, sizeof(v)));
}

extern "C" WF_API int wf_w8a8_gemm_status(int *status) {
    if (status == nullptr) return WF_ERR_ARG;
    return wf::w8a8_gemm_status(status);
}
