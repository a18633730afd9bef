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
WFO_API int wfo_set_threads(int threads) { return set_threads(threads); }

/* ================================================================================================ fused block */
static inline float bf(uint16_t b) { return u2f((uint32_t)b << 16); }
static inline uint16_t bf_bits(float x) { return isnan(x) ? (uint16_t)0x7FFF : (uint16_t)(f2u(r_bf16(x)) >> 16); }
/* the reference's rsqrt.approx.f32, restated as the correctly rounded reciprocal square root */
static inline float rsqrt_cr(float v) { return (float)(1.0 / sqrt((double)v)); }
/* x moved by k float32 ulps (k < 0: toward -inf): the tests evaluate a row with each reciprocal square root within
 * 2 ulps of the correctly rounded one, the error bound of the hardware approximation the kernels use */
static inline float ulp_shift(float x, int k) {
    while (k > 0) { x = nextafterf(x, INFINITY); --k; }
    while (k < 0) { x = nextafterf(x, -INFINITY); ++k; }
    return x;
}

/* modulate: out = R16(R16(x * s1) + shift), s1 = bf16(1 + scale) per group of rows
 * (enhancers/fused_kernels.py:51-62 _mod; fused_block.py:103-124) */
WFO_API void wfo_modulate(const uint16_t *x, const uint16_t *s1, const uint16_t *sh, uint16_t *out, int64_t rows,
                          int64_t d, int64_t rows_per_group, int threads) {
    set_threads(threads);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const int64_t g = r / rows_per_group;
        for (int64_t c = 0; c < d; ++c) {
            float t = r_bf16(bf(x[r * d + c]) * bf(s1[g * d + c]));
            out[r * d + c] = bf_bits(t + bf(sh[g * d + c]));
        }
    }
}

/* PyTorch's vectorized layer-norm statistics of one row of K (K % 512 == 0) as the reference reproduces them
 * (enhancers/fused_kernels.py:84-135 _wcombine / _whalf / _ln_stats): 128 threads, thread t updating a Welford
 * (mean, sigma2, count) with the 4-value vectors t, t + 128, ... in order; lanes merged by shuffle-down 16 .. 1
 * within each warp of 32, then warps 2, 3 into 0, 1 and warp 1 into 0. Returns mean and sigma2 / K. */
static void ln_stats(const uint16_t *row, int64_t K, float *mu_out, float *var_out) {
    float m[128], s[128], c[128];
    for (int t = 0; t < 128; ++t) {
        float mean = 0.f, sig = 0.f, cnt = 0.f;
        for (int64_t j = 0; j < K / 512; ++j)
            for (int ii = 0; ii < 4; ++ii) {
                float v = bf(row[(t + j * 128) * 4 + ii]);
                float delta = v - mean;
                cnt = cnt + 1.0f;
                mean = fmaf(delta, 1.0f / cnt, mean);
                sig = fmaf(delta, v - mean, sig);
            }
        m[t] = mean; s[t] = sig; c[t] = cnt;
    }
    /* combine(own = lower lane, other = upper lane) as _wcombine */
#define WCOMB(o, x)                                                   \
    do {                                                              \
        float delta = m[o] - m[x];                                    \
        float count = c[x] + c[o];                                    \
        float coef = 1.0f / count;                                    \
        float n_a = c[x] * coef, n_b = c[o] * coef;                   \
        float mean = fmaf(n_a, m[x], n_b * m[o]);                     \
        float sig = fmaf(delta * delta * c[x], n_b, s[x] + s[o]);     \
        m[o] = mean; s[o] = sig; c[o] = count;                        \
    } while (0)
    for (int w = 0; w < 4; ++w)
        for (int n = 32; n >= 2; n /= 2)
            for (int t = 0; t < n / 2; ++t) WCOMB(w * 32 + t, w * 32 + t + n / 2);
    WCOMB(0, 64);
    WCOMB(32, 96);
    WCOMB(0, 32);
#undef WCOMB
    *mu_out = m[0];
    *var_out = s[0] / (float)K;
}

/* LayerNorm (no affine) + modulate, one row (fused_kernels.py:219-232 _lnmod):
 * x = R16((x - mu) * rsqrt(var + eps)); out = R16(R16(x * s1) + shift) */
WFO_API void wfo_ln_modulate(const uint16_t *x, const uint16_t *s1, const uint16_t *sh, uint16_t *out, int64_t rows,
                             int64_t K, int64_t rows_per_group, float eps, int rstd_ulps, int threads) {
    set_threads(threads);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const uint16_t *xr = x + r * K;
        const int64_t g = r / rows_per_group;
        float mu, var;
        ln_stats(xr, K, &mu, &var);
        const float rstd = ulp_shift(rsqrt_cr(var + eps), rstd_ulps);
        for (int64_t c = 0; c < K; ++c) {
            float v = r_bf16((bf(xr[c]) - mu) * rstd);
            float t = r_bf16(v * bf(s1[g * K + c]));
            out[r * K + c] = bf_bits(t + bf(sh[g * K + c]));
        }
    }
}

/* RMSNorm over rows of 128 (fused_kernels.py:189-217 _rms128): thread t of 32 sums the squares of values 4t .. 4t+3
 * as ((a + b) + c) + d, a pairwise tree 16 .. 1 over the threads, rstd = rsqrt(sum / 128 + eps),
 * y = R16((x * rstd) * w) */
WFO_API void wfo_rms_norm_128(const uint16_t *x, const uint16_t *w, uint16_t *out, int64_t n_rows, float eps,
                              int rstd_ulps, int threads) {
    set_threads(threads);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < n_rows; ++r) {
        const uint16_t *xr = x + r * 128;
        float acc[32];
        for (int t = 0; t < 32; ++t) {
            float a = bf(xr[4 * t]), b = bf(xr[4 * t + 1]), c = bf(xr[4 * t + 2]), d = bf(xr[4 * t + 3]);
            acc[t] = ((a * a + b * b) + c * c) + d * d;
        }
        for (int n = 32; n >= 2; n /= 2)
            for (int t = 0; t < n / 2; ++t) acc[t] = acc[t] + acc[t + n / 2];
        const float rstd = ulp_shift(rsqrt_cr(acc[0] / 128.0f + eps), rstd_ulps);
        for (int c = 0; c < 128; ++c) out[r * 128 + c] = bf_bits((bf(xr[c]) * rstd) * bf(w[c]));
    }
}

/* RMSNorm-128 + split-half RoPE of contiguous (B, L, H, 128) rows (sage_fused.py:246-272 _rms_rope128, :159-176
 * _rope_rows): lane t of 32 sums the squares of values t, t+32, t+64, t+96 by fma from 0, a pairwise tree 16 .. 1,
 * rr = rsqrt(sum / 128 + eps), n = R16((x * rr) * w); then for d < 64, with f = freqs[token, d] (2 x 2, float32):
 * out[d] = R16(fma(f00, n[d], f01 * n[d+64])), out[d+64] = R16(fma(f10, n[d], f11 * n[d+64])).
 * w is given as float32 (the reference loads bf16 / fp16 / fp32 weights and widens them). */
WFO_API void wfo_rms_rope128(const uint16_t *x, const float *freqs, const float *w, uint16_t *out, int64_t n_rows,
                             int64_t heads, int64_t tokens, float eps, int rstd_ulps, int threads) {
    set_threads(threads);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < n_rows; ++r) {
        const uint16_t *xr = x + r * 128;
        const int64_t tok = (r / heads) % tokens;
        float acc[32];
        for (int t = 0; t < 32; ++t) {
            float v0 = bf(xr[t]), v1 = bf(xr[t + 32]), v2 = bf(xr[t + 64]), v3 = bf(xr[t + 96]);
            float a = v0 * v0;
            a = fmaf(v1, v1, a);
            a = fmaf(v2, v2, a);
            a = fmaf(v3, v3, a);
            acc[t] = a;
        }
        for (int n = 32; n >= 2; n /= 2)
            for (int t = 0; t < n / 2; ++t) acc[t] = acc[t] + acc[t + n / 2];
        const float rr = ulp_shift(rsqrt_cr(acc[0] / 128.0f + eps), rstd_ulps);
        float nv[128];
        for (int c = 0; c < 128; ++c) nv[c] = r_bf16((bf(xr[c]) * rr) * w[c]);
        for (int d = 0; d < 64; ++d) {
            const float *f = freqs + (tok * 64 + d) * 4;
            float lo = nv[d], hi = nv[d + 64];
            out[r * 128 + d] = bf_bits(fmaf(f[0], lo, f[1] * hi));
            out[r * 128 + d + 64] = bf_bits(fmaf(f[2], lo, f[3] * hi));
        }
    }
}

/* 256-wide Hadamard of comfy_kitchen's ConvRot as the reference computes it (fused_kernels.py:64-81 _h4): four
 * radix-4 stages of stride 1, 4, 16, 64, each mapping the 4-tuple (a, b, c, d) at stride S to
 * (a + b + c - d, a + b - c + d, a - b + c + d, -a + b + c + d) summed left to right; then x 1/16. */
static void hadamard256(float *g) {
    for (int S = 1; S <= 64; S *= 4) {
        float y[256];
        for (int blk = 0; blk < 256 / (4 * S); ++blk)
            for (int s = 0; s < S; ++s) {
                int base = blk * 4 * S + s;
                float a = g[base], b = g[base + S], c = g[base + 2 * S], d = g[base + 3 * S];
                y[base] = ((a + b) + c) - d;
                y[base + S] = ((a + b) - c) + d;
                y[base + 2 * S] = ((a - b) + c) + d;
                y[base + 3 * S] = ((-a + b) + c) + d;
            }
        memcpy(g, y, sizeof(y));
    }
    for (int i = 0; i < 256; ++i) g[i] = g[i] * 0.0625f;
}

/* int8 row quantiser (fused_kernels.py:137-174 _quant_row). pre: 0 none, 1 GELU by table (gelu[bits of x]),
 * 2 modulate, 3 LayerNorm + modulate. rotate: the ConvRot Hadamard (the reference always rotates; rotate = 0 is the
 * plain per-token absmax quantiser of the same arithmetic). amax = min(max |x|, 3.38953139e38),
 * scale = max(amax / 127, 1e-30) (stored), q = rint(R16(R16(x) / R16(scale))) clamped to [-128, 127].
 * The reference divides with the GPU's approximate division; this restatement divides exactly (IEEE). */
WFO_API void wfo_quant_rows(const uint16_t *x, const uint16_t *s1, const uint16_t *sh, const uint16_t *gelu,
                            int8_t *q, float *scale_out, int64_t rows, int64_t K, int64_t rows_per_group, float eps,
                            int pre, int rotate, int threads) {
    set_threads(threads);
#pragma omp parallel
    {
        float *v = (float *)__builtin_alloca(sizeof(float) * (size_t)K);
#pragma omp for schedule(static)
        for (int64_t r = 0; r < rows; ++r) {
            const uint16_t *xr = x + r * K;
            const int64_t g = r / rows_per_group;
            if (pre == 3) {
                float mu, var;
                ln_stats(xr, K, &mu, &var);
                const float rstd = rsqrt_cr(var + eps);
                for (int64_t c = 0; c < K; ++c) {
                    float t = r_bf16((bf(xr[c]) - mu) * rstd);
                    v[c] = r_bf16(r_bf16(t * bf(s1[g * K + c])) + bf(sh[g * K + c]));
                }
            } else if (pre == 1) {
                for (int64_t c = 0; c < K; ++c) v[c] = bf(gelu[xr[c]]);
            } else if (pre == 2) {
                for (int64_t c = 0; c < K; ++c)
                    v[c] = r_bf16(r_bf16(bf(xr[c]) * bf(s1[g * K + c])) + bf(sh[g * K + c]));
            } else {
                for (int64_t c = 0; c < K; ++c) v[c] = bf(xr[c]);
            }
            if (rotate)
                for (int64_t c = 0; c < K; c += 256) hadamard256(v + c);
            float amax = 0.f;
            for (int64_t c = 0; c < K; ++c) amax = fmaxf(amax, fabsf(v[c]));
            amax = fminf(amax, 3.38953139e38f);
            float scale = fmaxf(amax / 127.0f, 1.0e-30f);
            scale_out[r] = scale;
            const float sb = r_bf16(scale);
            for (int64_t c = 0; c < K; ++c) {
                float t = rintf(r_bf16(r_bf16(v[c]) / sb));
                t = fminf(fmaxf(t, -128.0f), 127.0f);
                q[r * K + c] = (int8_t)t;
            }
        }
    }
}
