// GGUF dequantisation (legacy Q4_0 / Q4_1 / Q5_0 / Q5_1 / Q8_0 and K-quants Q2_K .. Q6_K) for sm_100a.
//
// Arithmetic: ComfyUI-GGUF's PyTorch chain as the reference's Triton kernels restate it
// (enhancers/gguf_dequant.py:136-167 _deq, :188-256 _deq_k, :170-185 _sc / _mn): the block's float16 scale(s)
// rounded to the dequant dtype MID, every product and sum computed in float32 and rounded to MID on its own (no
// fused multiply-add: __fmul_rn / __fadd_rn / __fsub_rn), then the cast to OUT.
//
// Data movement (HBM-bound; one read of the packed bytes, one write of the values):
//   * a "chunk" is 8192 values: 256 legacy blocks or 32 super-blocks; its packed bytes are a multiple of 16 and
//     start 16-byte aligned whenever the tensor does;
//   * the grid walks the chunks, about eight per CTA (at least one full wave of resident CTAs); each CTA
//     double-buffers them in shared memory with 16-byte cp.async (the next chunk's bytes are in flight while the
//     current one is decoded);
//   * a thread decodes 8 consecutive values of one block from shared memory and writes them with one 16-byte store
//     (two for float32), so a warp writes 512 contiguous bytes per instruction;
//   * a single-tensor launch of at most two waves (one weight) also pulls the packed bytes of each CTA's chunk after
//     next into L2 (cp.async.bulk.prefetch.L2).
// The batched entry point walks the chunks of a table of tensors (checkpoint-wide sweep) with the same body.

#include "wf_common.cuh"

#include <atomic>
#include <type_traits>

#include <algorithm>

namespace wf {
namespace {

constexpr int kThreads = 256;
constexpr int kChunkValues = 8192;
constexpr int kGroupsPerThread = kChunkValues / 8 / kThreads;  // 4
constexpr int64_t kChunksPerCta = 8;                            // target chunks per CTA of a launch
constexpr int kMaxBatch = 640;  // tensors per batched launch (a 36-block checkpoint shard fits one; ~20 KB of parameters)

// ------------------------------------------------------------------------------------------------- formats
// (values per block, bytes per block) by GGML type id; _FORMATS / _KFORMATS (enhancers/gguf_dequant.py:52-56).
template <int QT> struct Fmt;
template <> struct Fmt<2>  { static constexpr int VPB = 32,  TS = 18;  };  // Q4_0
template <> struct Fmt<3>  { static constexpr int VPB = 32,  TS = 20;  };  // Q4_1
template <> struct Fmt<6>  { static constexpr int VPB = 32,  TS = 22;  };  // Q5_0
template <> struct Fmt<7>  { static constexpr int VPB = 32,  TS = 24;  };  // Q5_1
template <> struct Fmt<8>  { static constexpr int VPB = 32,  TS = 34;  };  // Q8_0
template <> struct Fmt<10> { static constexpr int VPB = 256, TS = 84;  };  // Q2_K
template <> struct Fmt<11> { static constexpr int VPB = 256, TS = 110; };  // Q3_K
template <> struct Fmt<12> { static constexpr int VPB = 256, TS = 144; };  // Q4_K
template <> struct Fmt<13> { static constexpr int VPB = 256, TS = 176; };  // Q5_K
template <> struct Fmt<14> { static constexpr int VPB = 256, TS = 210; };  // Q6_K

template <int QT>
__host__ __device__ constexpr int chunk_bytes() { return kChunkValues / Fmt<QT>::VPB * Fmt<QT>::TS; }
// one shared-memory buffer: the chunk plus 16 bytes of slack for the aligned over-reads of lds8_any
template <int QT>
__host__ __device__ constexpr int buf_stride() { return chunk_bytes<QT>() + 16; }

static_assert(chunk_bytes<2>() % 16 == 0 && chunk_bytes<3>() % 16 == 0 && chunk_bytes<6>() % 16 == 0 &&
                  chunk_bytes<7>() % 16 == 0 && chunk_bytes<8>() % 16 == 0 && chunk_bytes<10>() % 16 == 0 &&
                  chunk_bytes<11>() % 16 == 0 && chunk_bytes<12>() % 16 == 0 && chunk_bytes<13>() % 16 == 0 &&
                  chunk_bytes<14>() % 16 == 0,
              "every chunk must be a whole number of 16-byte units");

// ------------------------------------------------------------------------------------------------- decoders
// decode8<QT, MID>(blk, v0, x): values v0 .. v0 + 7 (v0 a multiple of 8) of the block at shared address blk,
// each rounded to MID exactly as the reference's kernel rounds it (before the cast to OUT).

// Legacy 32-value blocks: d at 0, m at 2 (Q4_1 / Q5_1), qh at QH (Q5_x), quants at QS (gguf_dequant.py:136-167).
template <int QT> struct Legacy;
template <> struct Legacy<2> { static constexpr bool HAS_M = false; static constexpr int QH = -1, QS = 2, SUB = 8;  };
template <> struct Legacy<3> { static constexpr bool HAS_M = true;  static constexpr int QH = -1, QS = 4, SUB = 0;  };
template <> struct Legacy<6> { static constexpr bool HAS_M = false; static constexpr int QH = 2,  QS = 6, SUB = 16; };
template <> struct Legacy<7> { static constexpr bool HAS_M = true;  static constexpr int QH = 4,  QS = 8, SUB = 0;  };

// ------------------------------------------------------------------------------------------------- float16 path
// MID = float16 (the reference's default) in packed half arithmetic. Every step of the chain is an f16 value times a
// small integer (exact in float32), or a sum / difference of two f16 values; the f16 operation rounds the exact
// result once, and the reference rounds the float32 result to f16 -- the same value, since float32 holds the
// products exactly and double rounding through float32 (24 bits) is innocuous for a sum of 11-bit values (24 >=
// 2 * 11 + 1); results in the subnormal range are multiples of 2^-24 and exact either way. __h*2_rn keep the
// compiler from contracting a product and a sum into one fma. Non-finite scales (inf * 0) give NaN payloads that
// are not reproduced bit for bit; every finite result, overflow to inf included, is.

// Two small non-negative integers (< 1024) held in bytes of `w` (chosen by the byte_perm selector `sel`, the second
// and fourth selected bytes being 0x64) become the half2 (1024 + a, 1024 + b); subtracting `bias` (1024 + offset)
// leaves (a - offset, b - offset), exactly.
__device__ __forceinline__ __half2 ints_h2(uint32_t w, uint32_t sel, __half2 bias) {
    const uint32_t bits = __byte_perm(w, 0x64646464u, sel);
    return __hsub2_rn(*reinterpret_cast<const __half2 *>(&bits), bias);
}

// 4 bytes of w -> pairs (b0, b1), (b2, b3) minus `bias`
__device__ __forceinline__ void bytes4_h2(uint32_t w, __half2 bias, __half2 &p01, __half2 &p23) {
    p01 = ints_h2(w, 0x4140u, bias);
    p23 = ints_h2(w, 0x4342u, bias);
}

__device__ __forceinline__ __half2 h2_bias(float b) { return __float2half2_rn(b); }
__device__ __forceinline__ __half h_of_bits(uint32_t bits) { return __ushort_as_half(static_cast<unsigned short>(bits)); }
__device__ __forceinline__ __half2 h2_splat_bits(uint32_t bits) { return __half2half2(h_of_bits(bits)); }
// a small integer (0 <= v < 1024) minus `off`, as an exact half
__device__ __forceinline__ __half h_int(uint32_t v, float off) {
    return __hsub_rn(h_of_bits(0x6400u | v), __float2half_rn(1024.0f + off));
}
// bit i (i = 0..3) of v moved to bit 0 of byte i
__device__ __forceinline__ uint32_t spread4(uint32_t v) { return ((v & 0xFu) * 0x00204081u) & 0x01010101u; }

// Q4_K / Q5_K: the scale and the min of sub-block `sub` (0..7) of a super-block, ds = f16(d * sc) and
// dm = f16(dmin * mn) with the 6-bit sc / mn unpacked from the 12 scale bytes (gguf_dequant.py:170-185), splatted
__device__ __forceinline__ void kq_scales(const uint8_t *blk, int sub, __half2 &ds, __half2 &dm) {
    const uint32_t dd = *reinterpret_cast<const uint32_t *>(blk);
    const uint8_t *sc_b = blk + 4;
    uint32_t sc, mn;
    if (sub < 4) {
        sc = sc_b[sub] & 63u;
        mn = sc_b[4 + sub] & 63u;
    } else {
        const int j = sub - 4;
        sc = (sc_b[8 + j] & 0xFu) | ((sc_b[j] >> 2) & 0x30u);
        mn = (sc_b[8 + j] >> 4) | ((sc_b[4 + j] >> 2) & 0x30u);
    }
    ds = __half2half2(__hmul_rn(h_of_bits(dd), h_int(sc, 0.f)));
    dm = __half2half2(__hmul_rn(h_of_bits(dd >> 16), h_int(mn, 0.f)));
}

// Q4_K / Q5_K: eight values from v0 of a super-block with their sub-block's (ds, dm): x = f16(f16(ds * q) - dm)
template <int QT>
__device__ __forceinline__ void decode8_kq(const uint8_t *blk, int v0, __half2 ds, __half2 dm, __half2 h[4]) {
    const int sub = v0 >> 5;
    constexpr int QS_OFF = (QT == 12) ? 16 : 48;
    const uint2 b = *reinterpret_cast<const uint2 *>(blk + QS_OFF + (sub >> 1) * 32 + (v0 & 31));
    const uint32_t sh = (sub & 1) * 4;
    uint32_t lo = (b.x >> sh) & 0x0F0F0F0Fu, hi = (b.y >> sh) & 0x0F0F0F0Fu;
    if constexpr (QT == 13) {
        const uint2 hb = *reinterpret_cast<const uint2 *>(blk + 16 + (v0 & 31));
        lo |= ((hb.x >> sub) & 0x01010101u) << 4;
        hi |= ((hb.y >> sub) & 0x01010101u) << 4;
    }
    const __half2 bias = h2_bias(1024.0f);
    bytes4_h2(lo, bias, h[0], h[1]);
    bytes4_h2(hi, bias, h[2], h[3]);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __hsub2_rn(__hmul2_rn(ds, h[i]), dm);
}

template <int QT>
__device__ __forceinline__ void decode8_h(const uint8_t *blk, int v0, __half2 h[4]) {
    if constexpr (QT == 8) {  // Q8_0
        const __half2 d = h2_splat_bits(lds16(blk));
        const uint2 q = lds8_any(blk + 2 + v0);
        const __half2 bias = h2_bias(1152.0f);  // (q ^ 0x80) = q + 128
        __half2 a, b, c, e;
        bytes4_h2(q.x ^ 0x80808080u, bias, a, b);
        bytes4_h2(q.y ^ 0x80808080u, bias, c, e);
        h[0] = __hmul2_rn(d, a); h[1] = __hmul2_rn(d, b); h[2] = __hmul2_rn(d, c); h[3] = __hmul2_rn(d, e);
    } else if constexpr (QT == 2 || QT == 3 || QT == 6 || QT == 7) {
        using L = Legacy<QT>;
        const __half2 d = h2_splat_bits(lds16(blk));
        const uint2 b = lds8_any(blk + L::QS + (v0 & 15));
        const uint32_t sh = (v0 >> 4) * 4;
        uint32_t lo = (b.x >> sh) & 0x0F0F0F0Fu, hi = (b.y >> sh) & 0x0F0F0F0Fu;
        if constexpr (L::QH >= 0) {
            const uint32_t hb = blk[L::QH + (v0 >> 3)];
            lo |= spread4(hb) << 4;
            hi |= spread4(hb >> 4) << 4;
        }
        const __half2 bias = h2_bias(1024.0f + L::SUB);
        bytes4_h2(lo, bias, h[0], h[1]);
        bytes4_h2(hi, bias, h[2], h[3]);
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __hmul2_rn(d, h[i]);
        if constexpr (L::HAS_M) {
            const __half2 m = h2_splat_bits(lds16(blk + 2));
#pragma unroll
            for (int i = 0; i < 4; ++i) h[i] = __hadd2_rn(h[i], m);
        }
    } else if constexpr (QT == 12 || QT == 13) {  // Q4_K / Q5_K
        __half2 ds, dm;
        kq_scales(blk, v0 >> 5, ds, dm);
        decode8_kq<QT>(blk, v0, ds, dm, h);
    } else if constexpr (QT == 14) {  // Q6_K
        const int hh = v0 >> 7, r = v0 & 127;
        const uint2 lo = lds8_any(blk + hh * 64 + (r & 63));
        const uint2 hi = lds8_any(blk + 128 + hh * 32 + (r & 31));
        const uint32_t lsh = (r >> 6) * 4, hsh = (r >> 5) * 2;
        const uint32_t q0 = ((lo.x >> lsh) & 0x0F0F0F0Fu) | (((hi.x >> hsh) & 0x03030303u) << 4);
        const uint32_t q1 = ((lo.y >> lsh) & 0x0F0F0F0Fu) | (((hi.y >> hsh) & 0x03030303u) << 4);
        const uint32_t scb = blk[192 + (v0 >> 4)];
        const __half2 d = __half2half2(__hmul_rn(h_of_bits(lds16(blk + 208)), h_int(scb ^ 0x80u, 128.f)));
        const __half2 bias = h2_bias(1056.0f);  // q - 32
        bytes4_h2(q0, bias, h[0], h[1]);
        bytes4_h2(q1, bias, h[2], h[3]);
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __hmul2_rn(d, h[i]);
    } else if constexpr (QT == 11) {  // Q3_K
        const int i16 = v0 >> 4;
        const uint32_t ls = (blk[96 + (i16 & 7)] >> ((i16 >> 3) * 4)) & 0xFu;
        const uint32_t hs = (blk[104 + (i16 & 3)] >> ((i16 >> 2) * 2)) & 3u;
        const __half2 d = __half2half2(__hmul_rn(h_of_bits(lds16(blk + 108)), h_int(ls | (hs << 4), 32.f)));
        const int r = v0 & 127;
        const uint2 ql = lds8_any(blk + 32 + (v0 >> 7) * 32 + (r & 31));
        const uint2 hm = lds8_any(blk + (v0 & 31));
        const uint32_t qsh = (r >> 5) * 2, hsh = v0 >> 5;
        // q = ql - 4 * (1 - bit) = (ql | bit << 2) - 4
        const uint32_t q0 = ((ql.x >> qsh) & 0x03030303u) | (((hm.x >> hsh) & 0x01010101u) << 2);
        const uint32_t q1 = ((ql.y >> qsh) & 0x03030303u) | (((hm.y >> hsh) & 0x01010101u) << 2);
        const __half2 bias = h2_bias(1028.0f);
        bytes4_h2(q0, bias, h[0], h[1]);
        bytes4_h2(q1, bias, h[2], h[3]);
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __hmul2_rn(d, h[i]);
    } else if constexpr (QT == 10) {  // Q2_K
        const uint32_t sb = blk[v0 >> 4];
        const __half2 dl = __half2half2(__hmul_rn(h_of_bits(lds16(blk + 80)), h_int(sb & 0xFu, 0.f)));
        const __half2 ml = __half2half2(__hmul_rn(h_of_bits(lds16(blk + 82)), h_int(sb >> 4, 0.f)));
        const int r = v0 & 127;
        const uint2 qb = lds8_any(blk + 16 + (v0 >> 7) * 32 + (r & 31));
        const uint32_t qsh = (r >> 5) * 2;
        const __half2 bias = h2_bias(1024.0f);
        bytes4_h2((qb.x >> qsh) & 0x03030303u, bias, h[0], h[1]);
        bytes4_h2((qb.y >> qsh) & 0x03030303u, bias, h[2], h[3]);
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __hsub2_rn(__hmul2_rn(dl, h[i]), ml);
    }
}

// Eight float16 results written as dtype OUT: float16 as they are, bfloat16 by the packed RNE conversion of their
// float32 values (the reference's bit-level RNE gives the same bits on every non-NaN value), float32 widened.
template <int OUT, bool VEC>
__device__ __forceinline__ void store8_h(void *dst, const __half2 h[4]) {
    if constexpr (OUT == WF_F16) {
        if constexpr (VEC) {
            *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(h);
        } else {
            const __half *hs = reinterpret_cast<const __half *>(h);
            __half *ds = reinterpret_cast<__half *>(dst);
#pragma unroll
            for (int i = 0; i < 8; ++i) ds[i] = hs[i];
        }
    } else {
        float x[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(h[i]);
            x[2 * i] = f.x;
            x[2 * i + 1] = f.y;
        }
        store8<OUT, VEC>(dst, x);
    }
}

template <int QT, int MID>
__device__ __forceinline__ void decode8(const uint8_t *blk, int v0, float x[8]) {
    if constexpr (MID == WF_F16) {
        __half2 h[4];
        decode8_h<QT>(blk, v0, h);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(h[i]);
            x[2 * i] = f.x;
            x[2 * i + 1] = f.y;
        }
        return;
    }
    if constexpr (QT == 8) {  // Q8_0: x = R(R(d) * q), q the int8
        const float d = rnd<MID>(f16_bits_to_f32(lds16(blk)));
        const uint2 q = lds8_any(blk + 2 + v0);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            x[i] = rnd<MID>(__fmul_rn(d, s8_to_f32(q.x >> (8 * i))));
            x[4 + i] = rnd<MID>(__fmul_rn(d, s8_to_f32(q.y >> (8 * i))));
        }
    } else if constexpr (QT == 2 || QT == 3 || QT == 6 || QT == 7) {
        using L = Legacy<QT>;
        const float d = rnd<MID>(f16_bits_to_f32(lds16(blk)));
        // value j < 16: low nibble of byte j; j >= 16: high nibble of byte j - 16
        const uint2 b = lds8_any(blk + L::QS + (v0 & 15));
        const uint32_t sh = (v0 >> 4) * 4;
        uint32_t hb = 0;
        if constexpr (L::QH >= 0) hb = blk[L::QH + (v0 >> 3)];  // bits v0 .. v0 + 7 of the 32-bit qh
        float m = 0.f;
        if constexpr (L::HAS_M) m = rnd<MID>(f16_bits_to_f32(lds16(blk + 2)));
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t byte = ((i < 4 ? b.x : b.y) >> (8 * (i & 3))) & 0xFFu;
            uint32_t nib = (byte >> sh) & 0xFu;
            if constexpr (L::QH >= 0) nib |= ((hb >> i) & 1u) << 4;
            const float q = __fsub_rn(small_u2f(nib), static_cast<float>(L::SUB));  // exact
            float v = rnd<MID>(__fmul_rn(d, q));
            if constexpr (L::HAS_M) v = rnd<MID>(__fadd_rn(v, m));
            x[i] = v;
        }
    } else if constexpr (QT == 12 || QT == 13) {  // Q4_K / Q5_K (gguf_dequant.py:195-212)
        const int sub = v0 >> 5;
        const uint32_t dd = *reinterpret_cast<const uint32_t *>(blk);  // block starts are 16-aligned
        const float d = rnd<MID>(f16_bits_to_f32(dd));
        const float dmin = rnd<MID>(f16_bits_to_f32(dd >> 16));
        // get_scale_min (_sc / _mn, gguf_dequant.py:170-185): 12 scale bytes at offset 4
        const uint8_t *sc_b = blk + 4;
        uint32_t sc, mn;
        if (sub < 4) {
            sc = sc_b[sub] & 63u;
            mn = sc_b[4 + sub] & 63u;
        } else {
            const int j = sub - 4;
            sc = (sc_b[8 + j] & 0xFu) | ((sc_b[j] >> 2) & 0x30u);
            mn = (sc_b[8 + j] >> 4) | ((sc_b[4 + j] >> 2) & 0x30u);
        }
        const float ds = rnd<MID>(__fmul_rn(d, small_u2f(sc)));
        const float dm = rnd<MID>(__fmul_rn(dmin, small_u2f(mn)));
        constexpr int QS_OFF = (QT == 12) ? 16 : 48;
        const uint2 b = *reinterpret_cast<const uint2 *>(blk + QS_OFF + (sub >> 1) * 32 + (v0 & 31));
        const uint32_t sh = (sub & 1) * 4;
        uint2 h = make_uint2(0, 0);
        if constexpr (QT == 13) h = *reinterpret_cast<const uint2 *>(blk + 16 + (v0 & 31));
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            uint32_t q = (((i < 4 ? b.x : b.y) >> (8 * (i & 3))) >> sh) & 0xFu;
            if constexpr (QT == 13) q |= (((((i < 4 ? h.x : h.y) >> (8 * (i & 3))) & 0xFFu) >> sub) & 1u) << 4;
            x[i] = rnd<MID>(__fsub_rn(rnd<MID>(__fmul_rn(ds, small_u2f(q))), dm));
        }
    } else if constexpr (QT == 14) {  // Q6_K (gguf_dequant.py:213-224): ql 128, qh 64, 16 int8 scales, d
        const int h = v0 >> 7, r = v0 & 127;
        const uint2 lo = lds8_any(blk + h * 64 + (r & 63));
        const uint2 hi = lds8_any(blk + 128 + h * 32 + (r & 31));
        const uint32_t lsh = (r >> 6) * 4, hsh = (r >> 5) * 2;
        const float sc = s8_to_f32(blk[192 + (v0 >> 4)]);
        const float d = rnd<MID>(__fmul_rn(rnd<MID>(f16_bits_to_f32(lds16(blk + 208))), sc));
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t l = ((((i < 4 ? lo.x : lo.y) >> (8 * (i & 3))) & 0xFFu) >> lsh) & 0xFu;
            const uint32_t hh = ((((i < 4 ? hi.x : hi.y) >> (8 * (i & 3))) & 0xFFu) >> hsh) & 3u;
            const float q = __fsub_rn(small_u2f(l | (hh << 4)), 32.0f);
            x[i] = rnd<MID>(__fmul_rn(d, q));
        }
    } else if constexpr (QT == 11) {  // Q3_K (gguf_dequant.py:225-240): hmask 32, qs 64, 12 scale bytes, d
        const int i16 = v0 >> 4;
        const uint32_t ls = (blk[96 + (i16 & 7)] >> ((i16 >> 3) * 4)) & 0xFu;
        const uint32_t hs = (blk[104 + (i16 & 3)] >> ((i16 >> 2) * 2)) & 3u;
        const float sc = __fsub_rn(small_u2f(ls | (hs << 4)), 32.0f);
        const float d = rnd<MID>(__fmul_rn(rnd<MID>(f16_bits_to_f32(lds16(blk + 108))), sc));
        const int r = v0 & 127;
        const uint2 ql = lds8_any(blk + 32 + (v0 >> 7) * 32 + (r & 31));
        const uint2 hm = lds8_any(blk + (v0 & 31));
        const uint32_t qsh = (r >> 5) * 2, hsh = v0 >> 5;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t qv = ((((i < 4 ? ql.x : ql.y) >> (8 * (i & 3))) & 0xFFu) >> qsh) & 3u;
            const uint32_t hb = (((((i < 4 ? hm.x : hm.y) >> (8 * (i & 3))) & 0xFFu) >> hsh) & 1u) ^ 1u;
            const float q = __fsub_rn(small_u2f(qv), small_u2f(hb << 2));
            x[i] = rnd<MID>(__fmul_rn(d, q));
        }
    } else if constexpr (QT == 10) {  // Q2_K (gguf_dequant.py:241-249): 16 scale bytes, qs 64, d, dmin
        const uint32_t sb = blk[v0 >> 4];
        const float dl = rnd<MID>(__fmul_rn(rnd<MID>(f16_bits_to_f32(lds16(blk + 80))), small_u2f(sb & 0xFu)));
        const float ml = rnd<MID>(__fmul_rn(rnd<MID>(f16_bits_to_f32(lds16(blk + 82))), small_u2f(sb >> 4)));
        const int r = v0 & 127;
        const uint2 qb = lds8_any(blk + 16 + (v0 >> 7) * 32 + (r & 31));
        const uint32_t qsh = (r >> 5) * 2;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t qv = ((((i < 4 ? qb.x : qb.y) >> (8 * (i & 3))) & 0xFFu) >> qsh) & 3u;
            x[i] = rnd<MID>(__fsub_rn(rnd<MID>(__fmul_rn(dl, small_u2f(qv))), ml));
        }
    }
}

// ------------------------------------------------------------------------------------------------- chunk body
// Copy `nbytes` packed bytes of one chunk into shared memory: whole 16-byte units by cp.async (ALIGNED: the global
// address is 16-byte aligned), the ragged tail (end of tensor) byte by byte.
template <bool ALIGNED>
__device__ __forceinline__ void stage_chunk(uint8_t *sdst, const uint8_t *gsrc, int nbytes) {
    if constexpr (ALIGNED) {
        const int units = nbytes >> 4;
        for (int u = threadIdx.x; u < units; u += kThreads) cp_async16(sdst + 16 * u, gsrc + 16 * u);
        const int rem = nbytes & 15;
        if (static_cast<int>(threadIdx.x) < rem) sdst[units * 16 + threadIdx.x] = __ldg(gsrc + units * 16 + threadIdx.x);
    } else {
        for (int i = threadIdx.x; i < nbytes; i += kThreads) sdst[i] = __ldg(gsrc + i);
    }
}

// The chunk's float32 LoRA difference into shared memory by cp.async (16-byte aligned; a chunk holds a whole number
// of 32-value blocks, so its difference is whole 16-byte units).
__device__ __forceinline__ void stage_diff(float *sdst, const float *gsrc, int nvalues) {
    const int units = nvalues >> 2;
    for (int u = threadIdx.x; u < units; u += kThreads) cp_async16(sdst + 4 * u, gsrc + 4 * u);
}

// Eight float16 results plus the LoRA difference, written as dtype OUT (float16 or bfloat16):
// w = R_out(R_out(x) + R_out(diff * sa)) in packed pairs. R_out(x) is the same conversion store8_h makes; the product
// is rounded to float32 (__fmul_rn) and then to OUT by cvt.rn, as the reference's integer round does for non-NaN
// values; the sum of two OUT values is exact in float32 whenever their exponents are close (11 + 13 bits for
// float16, 8 + 16 for bfloat16), and otherwise the smaller one is far below half an ulp of the larger, so one
// correctly rounded add.rn.{f16x2, bf16x2} equals the reference's float32 add followed by its rounding.
// dl: the 8 differences, in shared memory when ALIGNED, else in global memory.
template <int OUT, bool ALIGNED>
__device__ __forceinline__ void store8_h_lora(void *dst, const __half2 h[4], const float *dl, float sa) {
    float d[8];
    if constexpr (ALIGNED) {
        const float4 a = *reinterpret_cast<const float4 *>(dl);
        const float4 b = *(reinterpret_cast<const float4 *>(dl) + 1);
        d[0] = a.x; d[1] = a.y; d[2] = a.z; d[3] = a.w; d[4] = b.x; d[5] = b.y; d[6] = b.z; d[7] = b.w;
    } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) d[k] = __ldg(dl + k);
    }
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float p0 = __fmul_rn(d[2 * i], sa), p1 = __fmul_rn(d[2 * i + 1], sa);
        if constexpr (OUT == WF_BF16) {
            const float2 f = __half22float2(h[i]);
            const __nv_bfloat162 r = __hadd2_rn(__floats2bfloat162_rn(f.x, f.y), __floats2bfloat162_rn(p0, p1));
            w[i] = *reinterpret_cast<const uint32_t *>(&r);
        } else {
            const __half2 r = __hadd2_rn(h[i], __floats2half2_rn(p0, p1));
            w[i] = *reinterpret_cast<const uint32_t *>(&r);
        }
    }
    if constexpr (ALIGNED) {
        *reinterpret_cast<uint4 *>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
        uint16_t *ds = static_cast<uint16_t *>(dst);
#pragma unroll
        for (int k = 0; k < 8; ++k) ds[k] = static_cast<uint16_t>(w[k >> 1] >> (16 * (k & 1)));
    }
}

// LORA: the first LoRA difference added on the way out, w = R_out(w + R_out(diff * sa)) (the DEQ branch of the
// reference's _deq_add, enhancers/gguf_dequant.py:99-133); diff_chunk is the chunk's float32 difference (in shared
// memory when ALIGNED, else in global memory).
template <int QT, int MID, int OUT, bool ALIGNED, bool LORA>
__device__ __forceinline__ void decode_chunk(const uint8_t *sbuf, void *dst_chunk, int valid_values,
                                             const float *diff_chunk, float sa) {
    constexpr int VPB = Fmt<QT>::VPB, TS = Fmt<QT>::TS;
    // the float16 chain stays packed up to the store, with or without LoRA (float32 output: the float path below)
    constexpr bool kHalf = MID == WF_F16 && (!LORA || OUT != WF_F32);
    if constexpr (kHalf && (QT == 12 || QT == 13)) {
        // Q4_K / Q5_K: each thread decodes one 32-value sub-block's (ds, dm) into shared memory once per chunk
        // (kChunkValues / 32 == kThreads), so the groups below read it with one load instead of unpacking the
        // 6-bit scales again for every 8 values
        static_assert(kChunkValues / 32 == kThreads, "one sub-block per thread");
        __shared__ uint2 s_kq[kThreads];
        const int sub_all = threadIdx.x;
        if (32 * sub_all < valid_values) {
            __half2 ds, dm;
            kq_scales(sbuf + (sub_all / 8) * TS, sub_all % 8, ds, dm);
            s_kq[sub_all] = make_uint2(*reinterpret_cast<uint32_t *>(&ds), *reinterpret_cast<uint32_t *>(&dm));
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < kGroupsPerThread; ++i) {
            const int v = 8 * (threadIdx.x + i * kThreads);
            if (v >= valid_values) break;
            const uint2 sd = s_kq[v >> 5];
            __half2 h[4];
            decode8_kq<QT>(sbuf + (v / VPB) * TS, v % VPB, *reinterpret_cast<const __half2 *>(&sd.x),
                           *reinterpret_cast<const __half2 *>(&sd.y), h);
            uint8_t *out = static_cast<uint8_t *>(dst_chunk) + static_cast<size_t>(v) * dtype_size(OUT);
            if constexpr (LORA) store8_h_lora<OUT, ALIGNED>(out, h, diff_chunk + v, sa);
            else store8_h<OUT, ALIGNED>(out, h);
        }
        return;
    }
#pragma unroll
    for (int i = 0; i < kGroupsPerThread; ++i) {
        const int g = threadIdx.x + i * kThreads;
        const int v = 8 * g;
        if (v >= valid_values) break;
        if constexpr (kHalf) {
            __half2 h[4];
            decode8_h<QT>(sbuf + (v / VPB) * TS, v % VPB, h);
            uint8_t *out = static_cast<uint8_t *>(dst_chunk) + static_cast<size_t>(v) * dtype_size(OUT);
            if constexpr (LORA) store8_h_lora<OUT, ALIGNED>(out, h, diff_chunk + v, sa);
            else store8_h<OUT, ALIGNED>(out, h);
            continue;
        }
        float x[8];
        decode8<QT, MID>(sbuf + (v / VPB) * TS, v % VPB, x);
        // the cast to OUT: store8's RNE conversion (bit-identical to the reference's rounding on non-NaN values);
        // the LoRA add needs the rounded weight as float first
        if constexpr (LORA || OUT == WF_F32) {
#pragma unroll
            for (int k = 0; k < 8; ++k) x[k] = rnd<OUT>(x[k]);
        }
        if constexpr (LORA) {
            float dl[8];
            if constexpr (ALIGNED) {  // diff_chunk: the chunk's difference, staged in shared memory
                const float4 a = *reinterpret_cast<const float4 *>(diff_chunk + v);
                const float4 b = *(reinterpret_cast<const float4 *>(diff_chunk + v) + 1);
                dl[0] = a.x; dl[1] = a.y; dl[2] = a.z; dl[3] = a.w; dl[4] = b.x; dl[5] = b.y; dl[6] = b.z; dl[7] = b.w;
            } else {
#pragma unroll
                for (int k = 0; k < 8; ++k) dl[k] = __ldg(diff_chunk + v + k);
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) x[k] = rnd<OUT>(__fadd_rn(x[k], rnd<OUT>(__fmul_rn(dl[k], sa))));
        }
        store8<OUT, ALIGNED>(static_cast<uint8_t *>(dst_chunk) + static_cast<size_t>(v) * dtype_size(OUT), x);
    }
}

// Where chunk c of a launch lives: source bytes, destination, and how many of its values are real.
struct ChunkRef {
    const uint8_t *src;
    uint8_t *dst;
    int nbytes;
    int nvalues;
};

struct Single {
    const uint8_t *src;
    uint8_t *dst;
    int64_t n_values;
    int64_t n_chunks;
    const float *diff;  // LoRA difference (LORA launches only)
    float sa;
};

struct Batch {
    int n;
    int64_t first_chunk[kMaxBatch + 1];  // prefix sums of the tasks' chunk counts
    const uint8_t *src[kMaxBatch];
    uint8_t *dst[kMaxBatch];
    int64_t n_values[kMaxBatch];
};

template <int QT, int OUT>
__device__ __forceinline__ ChunkRef chunk_of(const uint8_t *src, uint8_t *dst, int64_t n_values, int64_t c) {
    constexpr int VPB = Fmt<QT>::VPB, TS = Fmt<QT>::TS;
    const int64_t v0 = c * kChunkValues;
    const int nv = static_cast<int>(min(static_cast<int64_t>(kChunkValues), n_values - v0));
    ChunkRef r;
    r.src = src + (v0 / VPB) * TS;
    r.dst = dst + v0 * dtype_size(OUT);
    r.nvalues = nv;
    r.nbytes = nv / VPB * TS;
    return r;
}

template <int QT, int OUT>
__device__ __forceinline__ ChunkRef chunk_of(const Single &p, int64_t c) {
    return chunk_of<QT, OUT>(p.src, p.dst, p.n_values, c);
}

template <int QT, int OUT>
__device__ __forceinline__ ChunkRef chunk_of(const Batch &p, int64_t c) {
    int lo = 0, hi = p.n - 1;  // the task t with first_chunk[t] <= c < first_chunk[t + 1]
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (p.first_chunk[mid] <= c) lo = mid; else hi = mid - 1;
    }
    return chunk_of<QT, OUT>(p.src[lo], p.dst[lo], p.n_values[lo], c - p.first_chunk[lo]);
}

__device__ __forceinline__ int64_t total_chunks(const Single &p) { return p.n_chunks; }
__device__ __forceinline__ const float *lora_diff(const Single &p, int64_t c) { return p.diff + c * kChunkValues; }
__device__ __forceinline__ float lora_scale(const Single &p) { return p.sa; }
__device__ __forceinline__ const float *lora_diff(const Batch &, int64_t) { return nullptr; }
__device__ __forceinline__ float lora_scale(const Batch &) { return 0.f; }
__device__ __forceinline__ int64_t total_chunks(const Batch &p) { return p.first_chunk[p.n]; }

template <int QT, int MID, int OUT, bool ALIGNED, bool LORA, typename P>
__global__ void __launch_bounds__(kThreads) dequant_kernel(const __grid_constant__ P p, int64_t pf) {
    extern __shared__ __align__(16) uint8_t smem[];
    constexpr int kStride = buf_stride<QT>();
    const int64_t n_chunks = total_chunks(p);
    int64_t c = blockIdx.x;
    if (c >= n_chunks) return;
    // launched as a programmatic dependent: the previous kernel of the stream has finished and its writes are
    // visible once this returns (at once for a plain launch). No early trigger of this grid's own dependents: it runs
    // many waves, whose CTAs they would compete with.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // LORA && ALIGNED: the chunks' differences ride in the same double buffer, after the packed bytes
    constexpr bool kStageDiff = LORA && ALIGNED;
    float *sdiff = reinterpret_cast<float *>(smem + 2 * kStride);
    ChunkRef cur = chunk_of<QT, OUT>(p, c);
    stage_chunk<ALIGNED>(smem, cur.src, cur.nbytes);
    if constexpr (kStageDiff) stage_diff(sdiff, lora_diff(p, c), cur.nvalues);
    cp_async_commit();
    for (int it = 0; c < n_chunks; ++it, c += gridDim.x) {
        const int64_t cn = c + gridDim.x;
        ChunkRef nxt{};
        if (cn < n_chunks) {
            nxt = chunk_of<QT, OUT>(p, cn);
            stage_chunk<ALIGNED>(smem + ((it + 1) & 1) * kStride, nxt.src, nxt.nbytes);
            if constexpr (kStageDiff) stage_diff(sdiff + ((it + 1) & 1) * kChunkValues, lora_diff(p, cn), nxt.nvalues);
        }
        cp_async_commit();
        if constexpr (ALIGNED && std::is_same_v<P, Single>) {  // (the batched sweep runs many waves: none)
            if (pf > 0 && threadIdx.x == 0 && cn + pf < n_chunks) {
                // pull into L2 the packed bytes of the chunk pf past the next one (whole 16-byte units)
                const ChunkRef f = chunk_of<QT, OUT>(p, cn + pf);
                const uint32_t nb = static_cast<uint32_t>(f.nbytes) & ~15u;
                if (nb > 0)
                    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(f.src), "r"(nb) : "memory");
            }
        }
        cp_async_wait<1>();  // this thread's copies of the current chunk have landed
        __syncthreads();     // ... and every other thread's
        const float *dchunk = nullptr;
        if constexpr (kStageDiff) dchunk = sdiff + (it & 1) * kChunkValues;
        else if constexpr (LORA) dchunk = lora_diff(p, c);
        decode_chunk<QT, MID, OUT, ALIGNED, LORA>(smem + (it & 1) * kStride, cur.dst, cur.nvalues, dchunk,
                                                  lora_scale(p));
        __syncthreads();     // the buffer is free for the chunk after next
        cur = nxt;
    }
}

// ------------------------------------------------------------------------------------------------- host launch
// L2 prefetch distance past the double-buffered next chunk, in quarter grids (WEIGHTFERRY_DEQUANT_PREFETCH 0 - 9,
// 0 = off; unset: one grid -- the chunk after next of the same CTA -- when the launch is at most two waves of
// resident CTAs, as a single weight's is, off otherwise). Measured over rotating single weights (one wave): Q8_0 5120 x 5120 0.863 -> 0.886 of the copy
// peak, Q4_K 5120 x 13824 0.861 -> 0.878; on the multi-wave 36-block Q4_K sweep it costs (0.993 -> 0.959).
int dequant_prefetch(bool short_launch) {
    static const int w = env_digit("WEIGHTFERRY_DEQUANT_PREFETCH", -1);
    return w >= 0 ? w : (short_launch ? 4 : 0);
}

template <int QT, int MID, int OUT, bool ALIGNED, bool LORA = false, typename P>
int launch(const P &p, int64_t n_chunks, cudaStream_t stream) {
    if (n_chunks <= 0) return WF_OK;
    constexpr int smem = 2 * buf_stride<QT>() + (LORA && ALIGNED ? 2 * kChunkValues * 4 : 0);
    auto kern = dequant_kernel<QT, MID, OUT, ALIGNED, LORA, P>;
    // per instantiation and device: resident CTAs per SM
    // written by whichever host thread launches first (the compute thread and the SSD uploader's both do): atomic
    static std::atomic<int> occ[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return WF_ERR_DEVICE;
    if (occ[dev].load(std::memory_order_acquire) == 0) {
        int o = 0;
        cudaError_t e = cudaSuccess;
        if constexpr (smem > 48 * 1024) {
            e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e != cudaSuccess) return static_cast<int>(e);
        }
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, kern, kThreads, smem);
        if (e != cudaSuccess) return static_cast<int>(e);
        occ[dev].store(std::max(o, 1), std::memory_order_release);
    }
    // about kChunksPerCta chunks per CTA, never fewer CTAs than fit at once: many short-lived CTAs instead of one
    // persistent wave. Measured on the 36-block Q4_K sweep (1.73 M chunks): one persistent wave 6.50 ms, ~27 chunks
    // per CTA 5.55 ms, ~6 per CTA 5.44 ms, one per CTA 5.88 ms; targets of 4 / 8 / 16 chunks 5.53 / 5.49 / 5.53 ms
    // (three runs each) -- the HBM sustains more of this write-heavy mix when the CTAs in flight start and finish at
    // different times than when one wave walks the tensor in step.
    const int64_t resident = static_cast<int64_t>(occ[dev].load(std::memory_order_acquire)) * device_sm_count();
    const int64_t grid =
        std::min<int64_t>(n_chunks, std::max<int64_t>(resident, (n_chunks + kChunksPerCta - 1) / kChunksPerCta));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p, grid * dequant_prefetch(grid <= 2 * resident) / 4);
    return static_cast<int>(e != cudaSuccess ? e : cudaGetLastError());
}

template <int QT>
int geometry(int *vpb, int *ts) {
    *vpb = Fmt<QT>::VPB;
    *ts = Fmt<QT>::TS;
    return WF_OK;
}

int block_info(int qtype, int *vpb, int *ts) {
    switch (qtype) {
        case 2: return geometry<2>(vpb, ts);
        case 3: return geometry<3>(vpb, ts);
        case 6: return geometry<6>(vpb, ts);
        case 7: return geometry<7>(vpb, ts);
        case 8: return geometry<8>(vpb, ts);
        case 10: return geometry<10>(vpb, ts);
        case 11: return geometry<11>(vpb, ts);
        case 12: return geometry<12>(vpb, ts);
        case 13: return geometry<13>(vpb, ts);
        case 14: return geometry<14>(vpb, ts);
        default: return WF_ERR_UNSUPPORTED;
    }
}

template <int QT, int MID, int OUT>
int run_single(const void *src, void *dst, int64_t n_values, cudaStream_t stream, const float *diff = nullptr,
               float sa = 0.f) {
    Single p;
    p.src = static_cast<const uint8_t *>(src);
    p.dst = static_cast<uint8_t *>(dst);
    p.n_values = n_values;
    p.n_chunks = (n_values + kChunkValues - 1) / kChunkValues;
    p.diff = diff;
    p.sa = sa;
    const bool aligned = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) |
                           reinterpret_cast<uintptr_t>(diff)) & 15u) == 0;
    if (diff != nullptr) {
        return aligned ? launch<QT, MID, OUT, true, true>(p, p.n_chunks, stream)
                       : launch<QT, MID, OUT, false, true>(p, p.n_chunks, stream);
    }
    return aligned ? launch<QT, MID, OUT, true>(p, p.n_chunks, stream)
                   : launch<QT, MID, OUT, false>(p, p.n_chunks, stream);
}

template <int QT, int MID, int OUT>
int run_batch(const wf_dequant_task *tasks, int n_tasks, cudaStream_t stream) {
    // aligned tasks go through the table in groups of kMaxBatch; a misaligned one runs on its own
    Batch b;
    b.n = 0;
    b.first_chunk[0] = 0;
    auto flush = [&]() -> int {
        if (b.n == 0) return WF_OK;
        const int64_t n_chunks = b.first_chunk[b.n];
        const int rc = launch<QT, MID, OUT, true>(b, n_chunks, stream);
        b.n = 0;
        b.first_chunk[0] = 0;
        return rc;
    };
    for (int i = 0; i < n_tasks; ++i) {
        const wf_dequant_task &t = tasks[i];
        if (t.n_values == 0) continue;
        const bool aligned = ((reinterpret_cast<uintptr_t>(t.src) | reinterpret_cast<uintptr_t>(t.dst)) & 15u) == 0;
        if (!aligned) {
            const int rc = run_single<QT, MID, OUT>(t.src, t.dst, t.n_values, stream);
            if (rc != WF_OK) return rc;
            continue;
        }
        b.src[b.n] = static_cast<const uint8_t *>(t.src);
        b.dst[b.n] = static_cast<uint8_t *>(t.dst);
        b.n_values[b.n] = t.n_values;
        b.first_chunk[b.n + 1] = b.first_chunk[b.n] + (t.n_values + kChunkValues - 1) / kChunkValues;
        ++b.n;
        if (b.n == kMaxBatch) {
            const int rc = flush();
            if (rc != WF_OK) return rc;
        }
    }
    return flush();
}

// dispatch on (mid, out) to a template instance
template <int QT>
int single_qt(int mid, int out, const void *src, void *dst, int64_t n, cudaStream_t s, const float *diff = nullptr,
              float sa = 0.f) {
    switch (mid) {
        case WF_F16:
            switch (out) {
                case WF_F16: return run_single<QT, WF_F16, WF_F16>(src, dst, n, s, diff, sa);
                case WF_BF16: return run_single<QT, WF_F16, WF_BF16>(src, dst, n, s, diff, sa);
                case WF_F32: return run_single<QT, WF_F16, WF_F32>(src, dst, n, s, diff, sa);
            }
            break;
        case WF_BF16:
            switch (out) {
                case WF_F16: return run_single<QT, WF_BF16, WF_F16>(src, dst, n, s, diff, sa);
                case WF_BF16: return run_single<QT, WF_BF16, WF_BF16>(src, dst, n, s, diff, sa);
                case WF_F32: return run_single<QT, WF_BF16, WF_F32>(src, dst, n, s, diff, sa);
            }
            break;
        case WF_F32:
            switch (out) {
                case WF_F16: return run_single<QT, WF_F32, WF_F16>(src, dst, n, s, diff, sa);
                case WF_BF16: return run_single<QT, WF_F32, WF_BF16>(src, dst, n, s, diff, sa);
                case WF_F32: return run_single<QT, WF_F32, WF_F32>(src, dst, n, s, diff, sa);
            }
            break;
    }
    return WF_ERR_ARG;
}

template <int QT>
int batch_qt(int mid, int out, const wf_dequant_task *t, int n, cudaStream_t s) {
    switch (mid) {
        case WF_F16:
            switch (out) {
                case WF_F16: return run_batch<QT, WF_F16, WF_F16>(t, n, s);
                case WF_BF16: return run_batch<QT, WF_F16, WF_BF16>(t, n, s);
                case WF_F32: return run_batch<QT, WF_F16, WF_F32>(t, n, s);
            }
            break;
        case WF_BF16:
            switch (out) {
                case WF_F16: return run_batch<QT, WF_BF16, WF_F16>(t, n, s);
                case WF_BF16: return run_batch<QT, WF_BF16, WF_BF16>(t, n, s);
                case WF_F32: return run_batch<QT, WF_BF16, WF_F32>(t, n, s);
            }
            break;
        case WF_F32:
            switch (out) {
                case WF_F16: return run_batch<QT, WF_F32, WF_F16>(t, n, s);
                case WF_BF16: return run_batch<QT, WF_F32, WF_BF16>(t, n, s);
                case WF_F32: return run_batch<QT, WF_F32, WF_F32>(t, n, s);
            }
            break;
    }
    return WF_ERR_ARG;
}

}  // namespace
}  // namespace wf

extern "C" WF_API int wf_gguf_block_info(int qtype, int *values_per_block, int *bytes_per_block) {
    int vpb = 0, ts = 0;
    const int rc = wf::block_info(qtype, &vpb, &ts);
    if (rc != WF_OK) return rc;
    if (values_per_block) *values_per_block = vpb;
    if (bytes_per_block) *bytes_per_block = ts;
    return WF_OK;
}

extern "C" WF_API int wf_dequant_gguf(const void *src, int64_t src_bytes, void *dst, int64_t n_values, int qtype, int mid,
                               int out, wf_stream_t stream) {
    int vpb = 0, ts = 0;
    int rc = wf::block_info(qtype, &vpb, &ts);
    if (rc != WF_OK) return rc;
    if (mid < WF_F16 || mid > WF_F32 || out < WF_F16 || out > WF_F32 || n_values < 0 || src_bytes < 0)
        return WF_ERR_ARG;
    if (n_values % vpb != 0 || n_values / vpb * ts != src_bytes) return WF_ERR_SHAPE;
    if (n_values == 0) return WF_OK;
    if (src == nullptr || dst == nullptr) return WF_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(dst) % wf::dtype_size(out) != 0) return WF_ERR_ARG;  // element-aligned output
    rc = wf::check_device();
    if (rc != WF_OK) return rc;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    switch (qtype) {
        case 2: return wf::single_qt<2>(mid, out, src, dst, n_values, s);
        case 3: return wf::single_qt<3>(mid, out, src, dst, n_values, s);
        case 6: return wf::single_qt<6>(mid, out, src, dst, n_values, s);
        case 7: return wf::single_qt<7>(mid, out, src, dst, n_values, s);
        case 8: return wf::single_qt<8>(mid, out, src, dst, n_values, s);
        case 10: return wf::single_qt<10>(mid, out, src, dst, n_values, s);
        case 11: return wf::single_qt<11>(mid, out, src, dst, n_values, s);
        case 12: return wf::single_qt<12>(mid, out, src, dst, n_values, s);
        case 13: return wf::single_qt<13>(mid, out, src, dst, n_values, s);
        case 14: return wf::single_qt<14>(mid, out, src, dst, n_values, s);
    }
    return WF_ERR_UNSUPPORTED;
}

extern "C" WF_API int wf_dequant_gguf_batch(const wf_dequant_task *tasks, int n_tasks, int qtype, int mid, int out,
                                     wf_stream_t stream) {
    int vpb = 0, ts = 0;
    int rc = wf::block_info(qtype, &vpb, &ts);
    if (rc != WF_OK) return rc;
    if (mid < WF_F16 || mid > WF_F32 || out < WF_F16 || out > WF_F32 || n_tasks < 0) return WF_ERR_ARG;
    if (n_tasks == 0) return WF_OK;
    if (tasks == nullptr) return WF_ERR_ARG;
    for (int i = 0; i < n_tasks; ++i) {
        if (tasks[i].n_values < 0 || tasks[i].n_values % vpb != 0) return WF_ERR_SHAPE;
        if (tasks[i].n_values > 0 && (tasks[i].src == nullptr || tasks[i].dst == nullptr)) return WF_ERR_ARG;
        if (reinterpret_cast<uintptr_t>(tasks[i].dst) % wf::dtype_size(out) != 0) return WF_ERR_ARG;
    }
    rc = wf::check_device();
    if (rc != WF_OK) return rc;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    switch (qtype) {
        case 2: return wf::batch_qt<2>(mid, out, tasks, n_tasks, s);
        case 3: return wf::batch_qt<3>(mid, out, tasks, n_tasks, s);
        case 6: return wf::batch_qt<6>(mid, out, tasks, n_tasks, s);
        case 7: return wf::batch_qt<7>(mid, out, tasks, n_tasks, s);
        case 8: return wf::batch_qt<8>(mid, out, tasks, n_tasks, s);
        case 10: return wf::batch_qt<10>(mid, out, tasks, n_tasks, s);
        case 11: return wf::batch_qt<11>(mid, out, tasks, n_tasks, s);
        case 12: return wf::batch_qt<12>(mid, out, tasks, n_tasks, s);
        case 13: return wf::batch_qt<13>(mid, out, tasks, n_tasks, s);
        case 14: return wf::batch_qt<14>(mid, out, tasks, n_tasks, s);
    }
    return WF_ERR_UNSUPPORTED;
}

extern "C" WF_API int wf_dequant_gguf_lora(const void *src, int64_t src_bytes, const float *diff, void *dst,
                                          int64_t n_values, int qtype, int mid, int out, float sa,
                                          wf_stream_t stream) {
    int vpb = 0, ts = 0;
    int rc = wf::block_info(qtype, &vpb, &ts);
    if (rc != WF_OK) return rc;
    if (mid < WF_F16 || mid > WF_F32 || out < WF_F16 || out > WF_F32 || n_values < 0 || src_bytes < 0)
        return WF_ERR_ARG;
    if (n_values % vpb != 0 || n_values / vpb * ts != src_bytes) return WF_ERR_SHAPE;
    if (n_values == 0) return WF_OK;
    if (src == nullptr || dst == nullptr || diff == nullptr) return WF_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(dst) % wf::dtype_size(out) != 0 || reinterpret_cast<uintptr_t>(diff) % 4 != 0)
        return WF_ERR_ARG;
    rc = wf::check_device();
    if (rc != WF_OK) return rc;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    switch (qtype) {
        case 2: return wf::single_qt<2>(mid, out, src, dst, n_values, s, diff, sa);
        case 3: return wf::single_qt<3>(mid, out, src, dst, n_values, s, diff, sa);
        case 6: return wf::single_qt<6>(mid, out, src, dst, n_values, s, diff, sa);
        case 7: return wf::single_qt<7>(mid, out, src, dst, n_values, s, diff, sa);
        case 8: return wf::single_qt<8>(mid, out, src, dst, n_values, s, diff, sa);
        case 10: return wf::single_qt<10>(mid, out, src, dst, n_values, s, diff, sa);
        case 11: return wf::single_qt<11>(mid, out, src, dst, n_values, s, diff, sa);
        case 12: return wf::single_qt<12>(mid, out, src, dst, n_values, s, diff, sa);
        case 13: return wf::single_qt<13>(mid, out, src, dst, n_values, s, diff, sa);
        case 14: return wf::single_qt<14>(mid, out, src, dst, n_values, s, diff, sa);
    }
    return WF_ERR_UNSUPPORTED;
}

namespace wf {
namespace {

// w = R_out(w + R_out(diff * sa)) in place on a weight of dtype OUT (the non-DEQ branch of _deq_add,
// enhancers/gguf_dequant.py:124-133: a further LoRA added to an already dequantised weight).
template <int OUT>
__global__ void __launch_bounds__(256) lora_add_kernel(const float *__restrict__ diff, void *w, int64_t n, float sa) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        float x;
        if constexpr (OUT == WF_BF16) x = __bfloat162float(static_cast<const __nv_bfloat16 *>(w)[i]);
        else if constexpr (OUT == WF_F16) x = __half2float(static_cast<const __half *>(w)[i]);
        else x = static_cast<const float *>(w)[i];
        x = rnd<OUT>(__fadd_rn(x, rnd<OUT>(__fmul_rn(__ldg(diff + i), sa))));
        if constexpr (OUT == WF_BF16) static_cast<__nv_bfloat16 *>(w)[i] = __float2bfloat16_rn(x);
        else if constexpr (OUT == WF_F16) static_cast<__half *>(w)[i] = __float2half_rn(x);
        else static_cast<float *>(w)[i] = x;
    }
}

template <int OUT>
int run_lora_add(const float *diff, void *w, int64_t n, float sa, cudaStream_t s) {
    const int64_t blocks = std::min<int64_t>((n + 255) / 256, static_cast<int64_t>(device_sm_count()) * 8);
    lora_add_kernel<OUT><<<static_cast<unsigned>(blocks), 256, 0, s>>>(diff, w, n, sa);
    return static_cast<int>(cudaGetLastError());
}

}  // namespace
}  // namespace wf

extern "C" WF_API int wf_lora_add(const float *diff, void *w, int64_t n_values, int out, float sa,
                                 wf_stream_t stream) {
    if (out < WF_F16 || out > WF_F32 || n_values < 0) return WF_ERR_ARG;
    if (n_values == 0) return WF_OK;
    if (diff == nullptr || w == nullptr) return WF_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(w) % wf::dtype_size(out) != 0 || reinterpret_cast<uintptr_t>(diff) % 4 != 0)
        return WF_ERR_ARG;
    const int rc = wf::check_device();
    if (rc != WF_OK) return rc;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    switch (out) {
        case WF_F16: return wf::run_lora_add<WF_F16>(diff, w, n_values, sa, s);
        case WF_BF16: return wf::run_lora_add<WF_BF16>(diff, w, n_values, sa, s);
        default: return wf::run_lora_add<WF_F32>(diff, w, n_values, sa, s);
    }
}
