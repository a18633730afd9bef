/*
 * wf_oracle.c -- CPU restatement of the WeightFerry quantized-weight path, used as the CHECKER.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the product (the package comfyui-weightferry_b200/) links, loads or calls
 * this file. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm use it.
 *
 * Every function states, value by value, the arithmetic of the reference's kernels for the path (paths inside the
 * ComfyUI-WeightFerry package), with every rounding explicit:
 *   - rnd(D, x): float32 -> nearest value of dtype D as float32; float16 by the C conversion (round to nearest even,
 *     subnormals and overflow to inf, as cvt.rn.f16.f32 does), bfloat16 by the reference's integer form
 *     (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000 (enhancers/gguf_dequant.py:72-83 _round);
 *   - compiled with -ffp-contract=off: every product and sum rounded on its own; where the reference uses a fused
 *     multiply-add it is written as fmaf().
 * Parity pin: tests/golden/make_golden.py runs the reference's own Triton kernels under TRITON_INTERPRET=1 on small
 * seeded inputs and stores their outputs under tests/golden/; tests/test_oracle_golden.py checks this file against
 * them bit for bit.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define WFO_API __attribute__((visibility("default")))

enum { F16 = 0, BF16 = 1, F32 = 2 };

/* ------------------------------------------------------------------------------------------------ rounding */
static inline uint32_t f2u(float x) { uint32_t u; memcpy(&u, &x, 4); return u; }
static inline float u2f(uint32_t u) { float x; memcpy(&x, &u, 4); return x; }

static inline float r_f16(float x) { return (float)(_Float16)x; }
static inline float r_bf16(float x) {
    uint32_t u = f2u(x);
    u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
    return u2f(u);
}
static inline float rnd(int d, float x) { return d == F16 ? r_f16(x) : d == BF16 ? r_bf16(x) : x; }

static inline float f16_at(const uint8_t *p) {
    uint16_t b = (uint16_t)(p[0] | (p[1] << 8));
    _Float16 h;
    memcpy(&h, &b, 2);
    return (float)h;
}

/* store one value (already rounded to `out`) as dtype `out`; a NaN becomes the canonical NaN of the hardware
 * conversion the reference's final `.to(dtype)` uses (0x7FFF for bfloat16 and float16). */
static inline void store_out(void *dst, int64_t i, int out, float x) {
    if (out == F32) {
        ((float *)dst)[i] = x;
    } else if (out == BF16) {
        uint16_t b = isnan(x) ? (uint16_t)0x7FFF : (uint16_t)(f2u(x) >> 16);
        ((uint16_t *)dst)[i] = b;
    } else {
        uint16_t b;
        if (isnan(x)) {
            b = 0x7FFF;
        } else {
            _Float16 h = (_Float16)x;
            memcpy(&b, &h, 2);
        }
        ((uint16_t *)dst)[i] = b;
    }
}

static inline float load_out(const void *src, int64_t i, int out) {
    if (out == F32) return ((const float *)src)[i];
    uint16_t b = ((const uint16_t *)src)[i];
    if (out == BF16) return u2f((uint32_t)b << 16);
    _Float16 h;
    memcpy(&h, &b, 2);
    return (float)h;
}

/* ------------------------------------------------------------------------------------------------ GGUF */
/* (values per block, bytes per block) by GGML type id (enhancers/gguf_dequant.py:52-56) */
static int geometry(int qt, int *vpb, int *ts) {
    switch (qt) {
        case 2: *vpb = 32; *ts = 18; return 0;
        case 3: *vpb = 32; *ts = 20; return 0;
        case 6: *vpb = 32; *ts = 22; return 0;
        case 7: *vpb = 32; *ts = 24; return 0;
        case 8: *vpb = 32; *ts = 34; return 0;
        case 10: *vpb = 256; *ts = 84; return 0;
        case 11: *vpb = 256; *ts = 110; return 0;
        case 12: *vpb = 256; *ts = 144; return 0;
        case 13: *vpb = 256; *ts = 176; return 0;
        case 14: *vpb = 256; *ts = 210; return 0;
        default: return -2;
    }
}

/* value v of the legacy block at b (enhancers/gguf_dequant.py:136-167 _deq), rounded to mid */
static float legacy_value(const uint8_t *b, int qt, int v, int mid) {
    int has_m = (qt == 3 || qt == 7);
    int qh = qt == 6 ? 2 : qt == 7 ? 4 : -1;
    int qs = qt == 2 ? 2 : qt == 3 ? 4 : qt == 6 ? 6 : qt == 7 ? 8 : 2;
    int sub = qt == 2 ? 8 : qt == 6 ? 16 : 0;
    float d = rnd(mid, f16_at(b));
    float q;
    if (qt == 8) {
        q = (float)(int8_t)b[qs + v];
    } else {
        int nib = (b[qs + (v % 16)] >> ((v / 16) * 4)) & 0xF;
        if (qh >= 0) nib |= ((b[qh + v / 8] >> (v % 8)) & 1) << 4;
        q = (float)(nib - sub);
    }
    float x = rnd(mid, d * q);
    if (has_m) x = rnd(mid, x + rnd(mid, f16_at(b + 2)));
    return x;
}

/* get_scale_min of Q4_K / Q5_K (enhancers/gguf_dequant.py:170-185 _sc / _mn) */
static void scale_min(const uint8_t *b, int sub, int *sc, int *mn) {
    const uint8_t *s = b + 4;
    if (sub < 4) {
        *sc = s[sub] & 63;
        *mn = s[4 + sub] & 63;
    } else {
        int j = sub - 4;
        *sc = (s[8 + j] & 0xF) | ((s[j] >> 2) & 0x30);
        *mn = (s[8 + j] >> 4) | ((s[4 + j] >> 2) & 0x30);
    }
}

/* value v (0..255) of the K-quant super-block at b (enhancers/gguf_dequant.py:188-249 _deq_k), rounded to mid */
static float kquant_value(const uint8_t *b, int qt, int v, int mid) {
    if (qt == 12 || qt == 13) {
        int qs_off = qt == 12 ? 16 : 48;
        int sub = v / 32;
        int q = (b[qs_off + (sub / 2) * 32 + v % 32] >> ((sub % 2) * 4)) & 0xF;
        if (qt == 13) q |= ((b[16 + v % 32] >> sub) & 1) << 4;
        float d = rnd(mid, f16_at(b));
        float dmin = rnd(mid, f16_at(b + 2));
        int sc, mn;
        scale_min(b, sub, &sc, &mn);
        float ds = rnd(mid, d * (float)sc);
        float dm = rnd(mid, dmin * (float)mn);
        return rnd(mid, rnd(mid, ds * (float)q) - dm);
    }
    if (qt == 14) {
        int h = v / 128, r = v % 128;
        int lo = (b[h * 64 + r % 64] >> ((r / 64) * 4)) & 0xF;
        int hi = (b[128 + h * 32 + r % 32] >> ((r / 32) * 2)) & 3;
        int q = (lo | (hi << 4)) - 32;
        float sc = (float)(int8_t)b[192 + v / 16];
        float d = rnd(mid, rnd(mid, f16_at(b + 208)) * sc);
        return rnd(mid, d * (float)q);
    }
    if (qt == 11) {
        int i = v / 16;
        int ls = (b[96 + i % 8] >> ((i / 8) * 4)) & 0xF;
        int hs = (b[104 + i % 4] >> ((i / 4) * 2)) & 3;
        int sc = (ls | (hs << 4)) - 32;
        float d = rnd(mid, rnd(mid, f16_at(b + 108)) * (float)sc);
        int r = v % 128;
        int ql = (b[32 + (v / 128) * 32 + r % 32] >> ((r / 32) * 2)) & 3;
        int hb = ((b[v % 32] >> (v / 32)) & 1) ^ 1;
        int q = ql - (hb << 2);
        return rnd(mid, d * (float)q);
    }
    /* Q2_K */
    int sb = b[v / 16];
    float dl = rnd(mid, rnd(mid, f16_at(b + 80)) * (float)(sb & 0xF));
    float ml = rnd(mid, rnd(mid, f16_at(b + 82)) * (float)(sb >> 4));
    int r = v % 128;
    int q = (b[16 + (v / 128) * 32 + r % 32] >> ((r / 32) * 2)) & 3;
    return rnd(mid, rnd(mid, dl * (float)q) - ml);
}

static int set_threads(int threads) {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
    return omp_get_max_threads();
#else
    (void)threads;
    return 1;
#endif
}

/* dequantize(): n_values values of `out` from src_bytes packed bytes; diff != NULL adds the first LoRA
 * (enhancers/gguf_dequant.py:99-133 _deq_add, DEQ branch): w = R_out(w + R_out(diff * sa)). */
WFO_API int wfo_dequant_gguf(const uint8_t *src, int64_t src_bytes, void *dst, int64_t n_values, int qt, int mid,
                             int out, const float *diff, float sa, int threads) {
    int vpb, ts;
    if (geometry(qt, &vpb, &ts)) return -2;
    if (n_values % vpb || n_values / vpb * ts != src_bytes) return -3;
    const int64_t n_blocks = n_values / vpb;
    set_threads(threads);
#pragma omp parallel for schedule(static)
    for (int64_t bi = 0; bi < n_blocks; ++bi) {
        const uint8_t *b = src + bi * ts;
        for (int v = 0; v < vpb; ++v) {
            float x = vpb == 32 ? legacy_value(b, qt, v, mid) : kquant_value(b, qt, v, mid);
            float w = rnd(out, x);
            const int64_t i = bi * vpb + v;
            if (diff) w = rnd(out, w + rnd(out, diff[i] * sa));
            store_out(dst, i, out, w);
        }
    }
    return 0;
}

/* A further LoRA on a dequantised weight (the non-DEQ branch of _deq_add): w = R_out(w + R_out(diff * sa)). */
WFO_API int wfo_lora_add(const float *diff, void *w, int64_t n, int out, float sa, int threads) {
    set_threads(threads);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        float x = load_out(w, i, out);
        x = rnd(out, x + rnd(out, diff[i] * sa));
        store_out(w, i, out, x);
    }
    return 0;
}

WFO_API int wfo_max_threads(void) { return set_threads(0); }
