/*
 * weightferry_b200.h -- C ABI of the B200 (sm_100a) kernels behind the WeightFerry quantized-weight path.
 *
 * Conventions shared by every entry point:
 *   - all buffers are device pointers allocated by the caller; no entry point allocates device memory;
 *   - `stream` is a cudaStream_t (the caller's current stream: the reference launches on
 *     torch.cuda.current_stream(), enhancers/fused_int8.py:151); NULL means the legacy default stream;
 *   - the return value is WF_OK (0), a negative WF_ERR_* for a rejected argument (nothing was launched), or a
 *     positive cudaError_t reported by the launch;
 *   - dtype codes follow the reference's _DT table (enhancers/gguf_dequant.py:58): 0 float16, 1 bfloat16, 2 float32.
 *
 * Reference citations are paths inside the ComfyUI-WeightFerry package.
 */
#ifndef WEIGHTFERRY_B200_H
#define WEIGHTFERRY_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define WF_API __attribute__((visibility("default")))
#else
#define WF_API
#endif

typedef struct CUstream_st *wf_stream_t; /* identical to cudaStream_t */

enum {
    WF_OK = 0,
    WF_ERR_ARG = -1,         /* a size, pointer or dtype outside the contract */
    WF_ERR_UNSUPPORTED = -2, /* a GGML type id (or mode) this library does not decode */
    WF_ERR_SHAPE = -3,       /* byte count and value count disagree for the format */
    WF_ERR_DEVICE = -4,      /* the current device is not an sm_100 part, or no device */
    WF_ERR_TOO_LARGE = -5    /* the problem exceeds a fixed-size buffer of the library */
};

enum { WF_F16 = 0, WF_BF16 = 1, WF_F32 = 2 };

/* Library version (major * 10000 + minor * 100 + patch). No reference counterpart (a library utility). */
WF_API int wf_version(void);

/* A static, human-readable string for a status returned by any entry point. No reference counterpart: the reference's
 * Python entry points raise exceptions (or answer None), which the Python layer over this library reproduces. */
WF_API const char *wf_status_string(int status);

/* Block geometry of a GGML quantisation type: values per block (32 or 256) and bytes per block.
 * Replaces the reference's _FORMATS / _KFORMATS tables (enhancers/gguf_dequant.py:52-56).
 * Returns WF_ERR_UNSUPPORTED for a type id outside Q4_0 (2), Q4_1 (3), Q5_0 (6), Q5_1 (7), Q8_0 (8), Q2_K (10),
 * Q3_K (11), Q4_K (12), Q5_K (13), Q6_K (14). */
WF_API int wf_gguf_block_info(int qtype, int *values_per_block, int *bytes_per_block);

/* GGUF dequantisation of one packed tensor: `src_bytes` bytes of blocks -> `n_values` values of dtype `out`, every
 * intermediate product / sum rounded to dtype `mid` exactly as ComfyUI-GGUF's PyTorch chain does.
 * Replaces the Triton launches of dequantize() / _dequantize_k() (enhancers/gguf_dequant.py:277-326; kernels
 * _deq :136-167 and _deq_k :188-256). src_bytes must equal n_values / values_per_block * bytes_per_block; dst must be
 * aligned to the output element (16-byte aligned src and dst take the vectorised path). */
WF_API int wf_dequant_gguf(const void *src, int64_t src_bytes, void *dst, int64_t n_values, int qtype, int mid, int out,
                    wf_stream_t stream);

/* One tensor of a batched (checkpoint-wide) dequantisation. */
typedef struct wf_dequant_task {
    const void *src; /* packed blocks */
    void *dst;       /* n_values outputs */
    int64_t n_values;
} wf_dequant_task;

/* Dequantise many tensors of one GGML type in one launch (a table of tensors, one persistent grid). Same arithmetic
 * as wf_dequant_gguf on each task. The reference dequantises per tensor on use (enhancers/gguf_dequant.py:296); this
 * is the sweep the streaming loader runs over a block's (or a shard's) tensors. n_tasks >= 0. */
WF_API int wf_dequant_gguf_batch(const wf_dequant_task *tasks, int n_tasks, int qtype, int mid, int out, wf_stream_t stream);

/* dequantisation with the first plain LoRA difference added in the same pass:
 *   w = R_out(R_out(x) + R_out(diff * sa)),  x the value wf_dequant_gguf produces before its cast,
 * diff the float32 (up @ down) of n_values, sa = float32(strength * alpha). Replaces the DEQ launch of _deq_add
 * (enhancers/gguf_dequant.py:99-133, launched by _add_loras :387-406). Every GGML type of wf_dequant_gguf. */
WF_API int wf_dequant_gguf_lora(const void *src, int64_t src_bytes, const float *diff, void *dst, int64_t n_values,
                                int qtype, int mid, int out, float sa, wf_stream_t stream);

/* One further LoRA difference added in place to a dequantised weight w of dtype `out`:
 *   w = R_out(w + R_out(diff * sa)).
 * Replaces the non-DEQ launch of _deq_add (enhancers/gguf_dequant.py:124-133). */
WF_API int wf_lora_add(const float *diff, void *w, int64_t n_values, int out, float sa, wf_stream_t stream);

/* ---------------------------------------------------------------------------------------- fused block prologue
 * bf16 tensors, contiguous rows. */

/* out = R16(R16(x * s1) + shift) for rows of d (d % 8 == 0; 16-byte aligned buffers); s1 = bf16(1 + scale) and
 * shift are [rows / rows_per_group, d]. Replaces the Triton launch of modulate() (enhancers/fused_block.py:103-124,
 * kernel _mod fused_kernels.py:51-62). */
WF_API int wf_modulate(const void *x, const void *s1, const void *shift, void *out, int64_t rows, int64_t d,
                       int64_t rows_per_group, wf_stream_t stream);

/* Gated residual update out[r, c] = bf16_rn(x[r, c] + f32(gate[r / rows_per_group, c] * o[r, c])) on bf16 [rows, d]
 * (d % 8 == 0, all pointers 16-byte aligned; out may be x): PyTorch's bf16 addcmul(x, gate, o) with the same bits, in
 * one vectorised pass. Replaces the block's residual addcmul (enhancers/fused_block.py:527-532, _add_residual) where
 * the residual is not folded into an int8 GEMM's epilogue. */
WF_API int wf_gated_residual(const void *x, const void *gate, const void *o, void *out, int64_t rows, int64_t d,
                             int64_t rows_per_group, wf_stream_t stream);

/* LayerNorm (no affine, PyTorch's vectorized Welford order) + modulate in one pass over rows of K (K % 512 == 0,
 * K <= 8192): x = R16((x - mean) * rsqrt(var + eps)); out = R16(R16(x * s1) + shift). Replaces ln_modulate()'s
 * launch (enhancers/fused_block.py:165-179, kernel _lnmod fused_kernels.py:219-232). */
WF_API int wf_ln_modulate(const void *x, const void *s1, const void *shift, void *out, int64_t rows, int64_t K,
                          int64_t rows_per_group, float eps, wf_stream_t stream);

/* RMSNorm over rows of 128: y = R16((x * rsqrt(mean(x^2) + eps)) * w), w of dtype w_dtype [128]. Replaces
 * rms_norm_128()'s launch (enhancers/fused_block.py:127-139, kernel _rms128 fused_kernels.py:189-217). */
WF_API int wf_rms_norm_128(const void *x, const void *w, int w_dtype, void *out, int64_t n_rows, float eps,
                           wf_stream_t stream);

/* RMSNorm-128 + split-half RoPE of a contiguous (batch, tokens, heads, 128) tensor with float32 rotations
 * freqs[token, d, i, j] (element strides given; (1, tokens, 1, 64, 2, 2) contiguous is (256, 4, 2, 1)), weight w
 * [128] of dtype w_dtype. Replaces rms_rope()'s launch (enhancers/sage_fused.py:325-334, kernels _rope_rows :159-176
 * / _rms_rope128 :246-272). */
WF_API int wf_rms_rope128(const void *x, const float *freqs, int64_t f_stride_token, int64_t f_stride_d,
                          int64_t f_stride_i, int64_t f_stride_j, const void *w, int w_dtype, void *out,
                          int64_t batch, int64_t tokens, int64_t heads, float eps, wf_stream_t stream);

/* wf_rms_rope128 of q and k (same shape, same rotations, weights wq / wk of one dtype) in one launch: the
 * self-attention's two rms_rope() calls (enhancers/sage_fused.py:325-334, called for q and k by the patched block,
 * enhancers/fused_block.py:652-703). Bit for bit the two single launches. */
WF_API int wf_rms_rope128_pair(const void *q, const void *k, const float *freqs, int64_t f_stride_token,
                               int64_t f_stride_d, int64_t f_stride_i, int64_t f_stride_j, const void *wq,
                               const void *wk, int w_dtype, void *q_out, void *k_out, int64_t batch, int64_t tokens,
                               int64_t heads, float eps, wf_stream_t stream);

/* Per-token int8 quantisation of rows of K: q [rows, K] int8, scale [rows] float32 (scale = max(amax / 127,
 * 1e-30)). pre: 0 none, 1 GELU by a 65536-entry bf16 table (gelu_table), 2 modulate (s1, shift), 3 LayerNorm +
 * modulate (K % 512 == 0, K <= 8192); rotate: the 256-wide ConvRot Hadamard (K % 256 == 0) -- the reference always
 * rotates, rotate = 0 is the plain absmax quantiser of BASELINE's W8A8 configuration. Replaces the quant_row launches
 * of _quantise_pre / _int8_quantised (enhancers/fused_int8.py:60-75, :172-176; kernel fused_kernels.py:137-174). */
WF_API int wf_quant_rows(const void *x, const void *s1, const void *shift, const void *gelu_table, int8_t *q,
                         float *scale, int64_t rows, int64_t K, int64_t rows_per_group, float eps, int pre, int rotate,
                         wf_stream_t stream);

/* Measurement helper of the benchmark (no reference counterpart): one streaming pass that reads in_bytes and writes
 * out_bytes (both multiples of 16, 16-byte aligned, each below 32 GiB, in_bytes <= out_bytes) with coalesced 16-byte
 * accesses, each input byte read from DRAM once: the HBM rate a plain kernel reaches for the dequantisation's
 * read : write mix. */
WF_API int wf_hbm_probe(const void *in, int64_t in_bytes, void *out, int64_t out_bytes, wf_stream_t stream);

/* ---------------------------------------------------------------------------------------- W8A8 linear */

/* y[m, n] = bf16_rn((float(acc[m, n]) * xs[m]) * ws[n]), acc = sum_k xq[m, k] * wq[n, k] in int32:
 * xq [m, k] and wq [n, k] int8 row-major (k % 16 == 0, 16-byte aligned), xs [m] and ws [n] float32 (ws 16-byte
 * aligned), y [m, n] bf16 (n % 8 == 0, 16-byte aligned); acc_dbg (optional, may be NULL) receives the raw int32
 * accumulators [m, n]. tcgen05 kind::i8 tensor-core GEMM with TMA-fed shared-memory stages and TMEM accumulators.
 * Replaces comfy_kitchen's cutlass_int8_dequant as the reference calls it (enhancers/fused_int8.py:200-203; the
 * per-channel ws expanded as at :185-186). */
WF_API int wf_w8a8_gemm(const int8_t *xq, const int8_t *wq, const float *xs, const float *ws, void *y,
                        int32_t *acc_dbg, int64_t m, int64_t n, int64_t k, wf_stream_t stream);

/* The W8A8 linear with the block's gated residual in its epilogue:
 *   out[r, c] = bf16_rn(float(resid[r, c]) + float(gate[r / rows_per_group, c]) * float(y[r, c]))
 * with y[r, c] the bf16 value wf_w8a8_gemm computes (one float32 product, one float32 sum, each rounded to nearest:
 * the bits of wf_w8a8_gemm followed by PyTorch's bf16 addcmul(resid, gate, y)). resid and out [m, n] bf16 and gate
 * [ceil(m / rows_per_group), n] bf16, all row-major and 16-byte aligned; rows_per_group >= 1 (the rows of one
 * (batch, frame) group; m or more: one gate row for all rows). out may be resid (in place). Operand rules otherwise
 * as wf_w8a8_gemm. Replaces comfy_kitchen's cutlass_int8_dequant_residual as the reference calls it, once per
 * group or once for all rows when the gates are equal (enhancers/fused_int8.py:212-268). */
WF_API int wf_w8a8_gemm_residual(const int8_t *xq, const int8_t *wq, const float *xs, const float *ws,
                                 const void *resid, const void *gate, int64_t rows_per_group, void *out, int64_t m,
                                 int64_t n, int64_t k, wf_stream_t stream);

/* Status word of the GEMM kernel: 0, or the code of a pipeline wait that ran out of time (the kernel then stopped
 * early and its output is incomplete). Reading it synchronises the device and clears it. No reference counterpart
 * (the reference's GEMM is a closed library call); it is this library's failure report. */
WF_API int wf_w8a8_gemm_status(int *status);

/* Test hook: the time limit, in nanoseconds, of the GEMM kernels' pipeline waits (default and maximum 2 s; 0 restores
 * the default). A short limit makes a wait run out on purpose, so that a test can check the abort path -- the status
 * code above, the kernel's bounded drain of its own copies and MMAs, and a correct GEMM afterwards -- without any
 * fault or hang. The drain waits themselves keep the 2 s limit. No reference counterpart. */
WF_API int wf_w8a8_gemm_set_wait_limit(uint64_t limit_ns);

/* W8A8 linear that allocates nothing: y = bf16((float(xq @ wq^T) * xs) * ws) where xq / xs are the per-token absmax
 * int8 quantisation of the bf16 activations x [m, k] (what wf_quant_rows with pre 0, rotate 0 produces), kept in a
 * fixed buffer inside the library instead of caller memory. For callers that cannot allocate device memory when
 * they run (an application whose allocator owns the GPU's memory, or a path where a cudaMalloc and its possible
 * device synchronisation are not allowed). Limits: m * k <= 16,777,216 and m <= 65,536, else WF_ERR_TOO_LARGE;
 * k <= 51,200 (the quantiser's row width), else WF_ERR_UNSUPPORTED; the operand rules of wf_quant_rows and
 * wf_w8a8_gemm apply. The buffer (about 16.3 MB per GPU that loads the library) is shared by every call: calls that
 * overlap on the GPU race. The first call on a device looks the buffer up for that device and keeps its address;
 * make it before any stream capture. A device reset (cudaDeviceReset) while the library is loaded is not supported:
 * the kept address would be stale. This entry point has no counterpart in the reference. */
WF_API int wf_w8a8_linear_noalloc(const void *x, const int8_t *wq, const float *ws, void *y, int64_t m, int64_t n,
                                  int64_t k, wf_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* WEIGHTFERRY_B200_H */
