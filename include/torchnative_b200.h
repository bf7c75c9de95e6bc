/*
 * torchnative_b200.h -- C ABI of the B200 (sm_100a) backend for torchnative's
 * two hot operators: the GGML Q4_0 weight-only linear and
 * scaled_dot_product_attention (flash attention with GQA and a KV cache).
 *
 * Plain pointers and sizes only; every device pointer is CUDA global memory on
 * the current device; `stream` is a cudaStream_t passed as void* (NULL = the
 * legacy default stream). Every entry point returns a tn_status and never
 * throws; on failure tn_last_error() holds a message naming the operator, in
 * the reference's wording where the reference has one.
 *
 * Each declaration names the reference interface it replaces (paths relative
 * to the torchnative project root), or says that it has none.
 */
#ifndef TORCHNATIVE_B200_H
#define TORCHNATIVE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TN_ABI_VERSION 1

#if defined(TN_BUILD) && defined(__GNUC__)
#define TN_API __attribute__((visibility("default")))
#else
#define TN_API
#endif

/* Status codes. The Rust side maps them the way torch_c/src/err.rs does:
 * TN_ERR_NOT_IMPLEMENTED -> NotImplementedError (err.rs::not_implemented),
 * everything else -> RuntimeError naming the op. */
typedef enum {
    TN_OK = 0,
    TN_ERR_NOT_IMPLEMENTED = 1, /* unsupported dtype / format / shape family, refused by name */
    TN_ERR_SHAPE = 2,           /* shapes that do not describe one operation */
    TN_ERR_INVALID = 3,         /* null or misaligned pointer, bad stride */
    TN_ERR_CUDA = 4,            /* a CUDA runtime call or launch failed */
    TN_ERR_OOM = 5,             /* device allocation failed */
    TN_ERR_TIMEOUT = 6          /* a bounded device-side wait gave up */
} tn_status;

/* Element types, in torch's naming. */
typedef enum { TN_F32 = 0, TN_F16 = 1, TN_BF16 = 2, TN_F64 = 3 } tn_dtype;

/* How the Q4_0 linear treats its activations.
 * TN_ACT_Q8_0: the reference's arithmetic -- each activation row is quantised
 *   to GGML Q8_0 (k_quants.rs:676-706), block dots are exact integers and the
 *   per-block scales are applied in float32 (k_quants.rs:312-330).
 * TN_ACT_FLOAT: no activation quantisation; weights are dequantised exactly
 *   to float32 and multiplied with the float activations (fp32 accumulate).
 *   tn_q4_0_linear runs it for up to 16 activation rows (refused by name
 *   above); the Q8_0 and Q4_K linears refuse it. */
typedef enum { TN_ACT_Q8_0 = 0, TN_ACT_FLOAT = 1 } tn_act_mode;

/* ---------------------------------------------------------------- runtime -- */

TN_API int tn_abi_version(void);
/* Message of the last failed call on this host thread ("" if none). */
TN_API const char *tn_last_error(void);
TN_API const char *tn_status_name(int status);

/* Device facts the kernels size themselves by. Replaces the device resolve /
 * arch check in torch_c/src/device.rs:370-392 (cuda_device) and :1505
 * (cuda_arch_mismatch): TN_ERR_NOT_IMPLEMENTED when the device is not sm_100. */
TN_API int tn_device_info(int device, int *sm_count, int *cc_major, int *cc_minor, int64_t *l2_bytes,
                   int64_t *smem_optin_per_block);

/* Synchronises the current device and reads its device-side error word: every
 * spin-wait in these kernels is bounded, and a wait that gives up records a
 * code there and returns instead of hanging. TN_ERR_TIMEOUT if set (cleared
 * when reset != 0). No reference counterpart (candle's kernels never wait). */
TN_API int tn_device_status(int reset);

/* The budget (GPU clock cycles, default 2^31, ~1 s) that every bounded wait of
 * these kernels on the current device allows before it gives up and records
 * TN_ERR_TIMEOUT; cycles <= 0 restores the default. *previous (if not NULL)
 * receives the budget in force. For tests and failure drills: a short budget
 * makes a wait on a peer that never signals end quickly. No reference
 * counterpart. */
TN_API int tn_set_wait_budget(int64_t cycles, int64_t *previous);

/* The stream calls on `device` run on when they pass stream == NULL (the
 * reference's one CudaStream per device, vendor/candle-core/src/cuda_backend/
 * device.rs:388-389); default NULL, the legacy default stream. Every entry
 * point given a non-NULL stream uses that one. */
TN_API int tn_stream_set(int device, void *stream);
TN_API int tn_stream_get(int device, void **stream);

/* Caching device allocator (replaces candle's per-tensor cudarc alloc,
 * vendor/candle-core/src/cuda_backend/device.rs:78-90). Blocks are reused
 * for requests of the same rounded size on the same stream; tn_empty_cache
 * returns unused blocks to the driver. */
TN_API int tn_alloc(void **ptr, size_t bytes, void *stream);
TN_API int tn_free(void *ptr, void *stream);
TN_API int tn_empty_cache(void);
TN_API int tn_memory_stats(size_t *allocated_bytes, size_t *reserved_bytes);

/* Per-process call counters, the evidence of which path ran (the reference's
 * _cuda_counters, torch_c/src/device.rs:1671-1700). */
typedef struct {
    uint64_t q4_linear_calls;
    uint64_t q4_gemv_launches;     /* decode GEMV (TMA-staged) launches */
    uint64_t q4_gemv_generic;      /* decode GEMV launches on the unstaged path (K % 256 != 0) */
    uint64_t q4_gemm_launches;     /* prefill launches */
    uint64_t q8_quant_launches;
    uint64_t q4_codec_launches;
    uint64_t sdpa_calls;
    uint64_t sdpa_decode_launches; /* split-KV decode kernels */
    uint64_t sdpa_prefill_launches;
    uint64_t bytes_allocated;
    uint64_t q4_skinny_launches;   /* batched-decode (9..32 rows) tensor-core launches */
    uint64_t decode_token_launches; /* persistent whole-token decode kernels (tn_llama_decode_token) */
    uint64_t refusals;             /* calls refused by name (TN_ERR_NOT_IMPLEMENTED) */
    uint64_t resolves;             /* devices resolved (first use of a device's facts) */
    uint64_t reserved[2];
} tn_counters;
TN_API int tn_get_counters(tn_counters *out);
TN_API int tn_reset_counters(void);

/* ------------------------------------------------------- Q4_0 op family -- */

/* Q4_0 writer on the device: rows x cols float32 -> rows * cols/32 blocks of
 * 18 bytes. Byte-identical to BlockQ4_0::from_float
 * (vendor/candle-core/src/quantized/k_quants.rs:241-277), which
 * torch._C._quantize(t, "q4_0") runs (torch_c/src/quant.rs:124-172). */
TN_API int tn_q4_0_quantize(const float *x, void *blob, int64_t rows, int64_t cols, void *stream);

/* Q4_0 reader: blob -> float32 [rows, cols], bit-identical to
 * BlockQ4_0::to_float (k_quants.rs:219-239); replaces candle's
 * dequantize_block_q4_0_f32 (vendor/candle-core/src/quantized/cuda.rs:105-160)
 * behind torch._C._dequantize (quant.rs:180-189). */
TN_API int tn_q4_0_dequantize(const void *blob, float *out, int64_t rows, int64_t cols, void *stream);

/* Q8_0 writer for activations: x [rows, cols] (row stride x_row_stride
 * elements, dtype x_dtype in {F32, BF16, F16}; bf16/f16 widened exactly) ->
 * GGML Q8_0 blocks of 34 bytes, byte-identical to BlockQ8_0::from_float
 * (k_quants.rs:676-706). Replaces candle's quantize_q8_1
 * (vendor/candle-core/src/quantized/cuda.rs:48). */
TN_API int tn_q8_0_quantize(const void *x, int x_dtype, int64_t x_row_stride, void *blob, int64_t rows,
                     int64_t cols, void *stream);

/* Q8_0 reader: blob -> float32 [rows, cols], bit-identical to
 * BlockQ8_0::to_float (k_quants.rs:658-674), behind torch._C._dequantize for a
 * q8_0 weight (quant.rs:180-189); replaces candle's dequantize_block_q8_0_f32
 * (vendor/candle-core/src/quantized/cuda.rs:105-160). Writer: tn_q8_0_quantize (the
 * same BlockQ8_0::from_float serves weights and activations). */
TN_API int tn_q8_0_dequantize(const void *blob, float *out, int64_t rows, int64_t cols, void *stream);

/* torch._C._quantized_linear(input, weight, bias) (torch_c/src/quant.rs:286-369):
 * y[M, N] = x[M, K] @ W[N, K]^T (+ bias[N]).
 *   x: device [M, K], dtype x_dtype in {F32, BF16, F16}, row stride
 *      x_row_stride elements (>= K), unit inner stride.
 *   w_blob: device, the GGML Q4_0 blob of W exactly as _quantized_blob /
 *      _quantized_to hold it: N rows of K/32 blocks of 18 bytes.
 *   bias: device float32 [N] or NULL (added in float32 after the product,
 *      quant.rs:350-365).
 *   y: device [M, N] row-major, dtype y_dtype in {F32, BF16, F16}.
 *   act_mode: tn_act_mode.
 * Replaces QMatMul::forward's CUDA arm (vendor/candle-core/src/quantized/
 * mod.rs:1007-1043 -> quantized/cuda.rs:846-877: fast_mmvq for M <= 8,
 * fast_mmq above). K must be a multiple of 32 (a Q4_0 row is whole blocks);
 * otherwise TN_ERR_SHAPE in upstream's wording. M == 0 or N == 0 is a no-op.
 * May allocate a workspace through the caching allocator on first use of a
 * size (activation blocks); stream-ordered. */
TN_API int tn_q4_0_linear(const void *x, int x_dtype, int64_t x_row_stride, const void *w_blob,
                   const float *bias, void *y, int y_dtype, int64_t M, int64_t N, int64_t K,
                   int act_mode, void *stream);

/* The same torch._C._quantized_linear for a Q8_0 weight (quant.rs:286-369 with
 * format "q8_0"): w_blob is N rows of K/32 GGML BlockQ8_0 blocks of 34 bytes
 * (f16 d, then 32 int8 codes; k_quants.rs:652-756). The activations are
 * quantised to Q8_0 as for Q4_0 and every output element is
 * sum over blocks of (i32 sum q8_w * q8_x) * d_w * d_x in f32, the arithmetic
 * of BlockQ8_0::vec_dot_unopt (k_quants.rs:737-756). Replaces candle's CUDA
 * arm for GgmlDType::Q8_0 (quantized/cuda.rs:846-877). Every M runs on the
 * decode GEMV (chunks of at most 16 rows). Same arguments, refusals and
 * workspace rules as tn_q4_0_linear. */
TN_API int tn_q8_0_linear(const void *x, int x_dtype, int64_t x_row_stride, const void *w_blob,
                          const float *bias, void *y, int y_dtype, int64_t M, int64_t N, int64_t K,
                          int act_mode, void *stream);

/* Q4_K reader: blob of rows * cols/256 BlockQ4K super-blocks (144 bytes: f16
 * d, f16 dmin, 12 bytes of 6-bit scales and mins, 128 bytes of nibbles;
 * vendor/candle-core/src/quantized/k_quants.rs:153-159) -> float32 [rows,
 * cols], bit-identical to BlockQ4K::to_float (k_quants.rs:1722-1748), behind
 * torch._C._dequantize of a q4_k weight (quant.rs:180-189); replaces candle's
 * dequantize_block_q4_K (quantized/cuda.rs:105-160). */
TN_API int tn_q4_k_dequantize(const void *blob, float *out, int64_t rows, int64_t cols, void *stream);

/* torch._C._quantized_linear for a Q4_K weight (quant.rs:286-369 with format
 * "q4_k"): the activation rows are quantised to Q8_K (BlockQ8K::from_float,
 * k_quants.rs:2376-2410: per 256 elements iscale = -127/max, f32 d = 1/iscale)
 * and every output element is BlockQ4K::vec_dot_unopt's sum (k_quants.rs:
 * 1478-1544) of d_w*d_x * sum sc*(q4.q8) - dmin_w*d_x * sum m*(code sums), with
 * exact integer sub-block sums. K % 256 == 0, w_blob 16-byte aligned; every M
 * on the decode GEMV (chunks of up to 16 rows). Same arguments and refusals as
 * tn_q4_0_linear. Replaces candle's CUDA arm for GgmlDType::Q4K
 * (quantized/cuda.rs:846-877). */
TN_API int tn_q4_k_linear(const void *x, int x_dtype, int64_t x_row_stride, const void *w_blob,
                          const float *bias, void *y, int y_dtype, int64_t M, int64_t N, int64_t K,
                          int act_mode, void *stream);

/* The same linear split in two, for callers that fuse the activation
 * quantisation into the kernel that produces the activations (an RMSNorm or a
 * SiLU*mul epilogue) -- the reference does the two steps back to back too
 * (k_quants.rs:2479-2510 then 2512-2553).
 *
 * Planar Q8_0 layout of M activation rows of K elements:
 *   codes   int8  [M][codes_row_stride]  the Q8_0 codes, 32 per block in order
 *   scales  f32   [M][K/32]              f32 of the block's f16 scale d
 *   offsets f32   [M][K/32]              12582912 + 8 * sum(codes of the block)
 * (12582912 = 1.5 * 2^23 is the magic number of the kernels' exact int->float
 * step; the 8 * sum term removes the Q4_0 "-8" offset.) The blocks are the
 * GGML Q8_0 blocks of tn_q8_0_quantize, byte for byte, rearranged. */
TN_API int tn_q8_0_quantize_planar(const void *x, int x_dtype, int64_t x_row_stride, int8_t *codes,
                                   int64_t codes_row_stride, float *scales, float *offsets,
                                   int64_t rows, int64_t cols, void *stream);
/* flags: TN_WEIGHTS_STATIC -- the caller vouches that no work queued before
 * this call on the stream writes w_blob (true of a model's weights), so the
 * kernel may start streaming the weights before the previous kernel in the
 * stream has finished (programmatic dependent launch). 0 = always wait. */
#define TN_WEIGHTS_STATIC 1
/* flags: TN_EPILOGUE_SILU_MUL_PAIRS -- the weight's rows come in (gate, up)
 * pairs (row 2i = gate_i, row 2i+1 = up_i: LlamaMLP's gate_proj and up_proj
 * interleaved row by row, which a Q4_0 blob allows since rows are whole
 * blocks); y receives, for each pair, bf16(bf16(silu(gate_i)) * up_i) with
 * gate_i and up_i first rounded to bf16, i.e. N/2 columns of row stride N/2.
 * N even, y bf16. */
#define TN_EPILOGUE_SILU_MUL_PAIRS 2
TN_API int tn_q4_0_linear_q8(const int8_t *codes, int64_t codes_row_stride, const float *scales,
                             const float *offsets, const void *w_blob, const float *bias, void *y,
                             int y_dtype, int64_t M, int64_t N, int64_t K, int flags, void *stream);

/* The linear with its activation quantisation fused into the GEMV's prologue,
 * for decode (M <= 4 rows): every CTA builds the same planar Q8_0 tile from
 * bf16 rows, so the kernel that would otherwise quantise (and the norm or
 * SiLU kernel before it) disappears from the step. x_mode:
 *   TN_X_BF16      x [M][K] as is;
 *   TN_X_RMSNORM   transformers' LlamaRMSNorm of h = bf16(x + delta)
 *                  (delta may be NULL): norm_weight * bf16(h32 * rsqrt(mean(h32^2) + eps));
 *                  h is also written to h_out (if not NULL; must not alias x or delta);
 *                  x, delta, h_out and norm_weight 16-byte aligned, rows of x_row_stride
 *                  elements (a multiple of 8) in all three;
 *   TN_X_SILU_MUL  bf16(bf16(silu(gate)) * up) from rows [gate (K) | up (K)].
 * Then the Q8_0 quantiser (k_quants.rs:676-706) and the same GEMV as
 * tn_q4_0_linear_q8. No reference counterpart as one call: the reference runs
 * these as separate ops in the transformers model around _quantized_linear. */
#define TN_X_BF16 1
#define TN_X_RMSNORM 2
#define TN_X_SILU_MUL 3
TN_API int tn_q4_0_linear_fused(int x_mode, const void *x, int64_t x_row_stride, const void *delta,
                                void *h_out, const void *norm_weight, float eps, const void *w_blob,
                                const float *bias, void *y, int y_dtype, int64_t M, int64_t N,
                                int64_t K, int flags, void *stream);

/* tn_q4_0_linear_fused whose launch also writes the planar Q8_0 of its own
 * bf16 output y (the layout of tn_q8_0_quantize_planar, with K = y's column
 * count: N, or N/2 under TN_EPILOGUE_SILU_MUL_PAIRS) -- the next linear's
 * activations, byte for byte what tn_q8_0_quantize_planar(y) writes, without
 * its launch. y bf16, y's columns a multiple of 32. The decode step uses it for
 * LlamaMLP's act = SiLU(gate) * up ahead of down_proj. No reference counterpart
 * as one call: the reference quantises the activation inside the next
 * _quantized_linear (k_quants.rs:676-706). */
TN_API int tn_q4_0_linear_fused_q8out(int x_mode, const void *x, int64_t x_row_stride, const void *delta,
                                      void *h_out, const void *norm_weight, float eps, const void *w_blob,
                                      const float *bias, void *y, int y_dtype, int64_t M, int64_t N, int64_t K,
                                      int flags, int8_t *codes, int64_t codes_row_stride, float *scales,
                                      float *offsets, void *stream);

/* tn_q4_0_linear without any device allocation. No counterpart in the
 * reference: it exists for hosts that cannot let a library call cudaMalloc
 * while they run -- an engine that owns a preplanned arena of HBM, work being
 * recorded into a CUDA graph under global capture mode, a loop that cannot
 * absorb cudaMalloc's implicit synchronisation. Same arguments and arithmetic
 * as tn_q4_0_linear in TN_ACT_Q8_0 mode, through the decode GEMV: the same
 * result bit for bit up to 8 rows; from 9 rows tn_q4_0_linear takes the
 * tensor-core kernel, whose summation order differs (both lie within the
 * counted error bound of the exact value). The Q8_0 activation blocks go
 * to a fixed __device__ array inside this library (320 KB, held on every GPU
 * that loads the library until the process exits) instead of the allocator.
 * Limits: M <= TN_NOALLOC_MAX_ROWS and K <= TN_NOALLOC_MAX_IN; larger calls
 * return TN_ERR_SHAPE and allocate nothing. The first call on a device looks
 * up the array's device address (cudaGetSymbolAddress, that device current);
 * make it before any stream capture. The address is cached for the context
 * current at that call: it does not survive cudaDeviceReset or a switch to
 * another context on the device. All calls share the one array, so calls
 * that can overlap on the GPU (unordered streams) race. Counted in
 * tn_counters.q4_linear_calls like tn_q4_0_linear. K == 0 is refused
 * (TN_ERR_NOT_IMPLEMENTED) as tn_q4_0_linear refuses it. */
#define TN_NOALLOC_MAX_ROWS 16
#define TN_NOALLOC_MAX_IN 16384
TN_API int tn_q4_0_linear_noalloc(const void *x, int x_dtype, int64_t x_row_stride, const void *w_blob,
                                  const float *bias, void *y, int y_dtype, int64_t M, int64_t N,
                                  int64_t K, void *stream);

/* ------------------------------------------------------------ SDPA family -- */

/* aten._scaled_dot_product_flash_attention_for_cpu.default(query, key, value,
 *     dropout_p=0.0, is_causal=False, *, attn_mask=None, scale=None)
 *     -> (out, logsumexp)
 * reached through _C._aten_dispatch (torch_c/src/aten.rs:1524 -> 2687 ->
 * routed 2771 -> CUDA arm 2861-2865 -> 7057 -> sdpa_flash_cpu 10092-10460).
 *   q [B, Hq, L, D], k/v [B, Hkv, S, D]: device, dtype in {F32, BF16, F16},
 *     element strides q_strides[4] etc. in [b, h, t, d] order with unit d
 *     stride -- a KV-cache view narrowed out of a [B, Hkv, cap, D] buffer
 *     (kv_cache.py:92-114) is read in place.
 *   Grouped-query attention: query head h reads kv head h / (Hq / Hkv)
 *     (repeat_kv_heads, aten.rs:17106-17130); Hq % Hkv != 0 is refused.
 *   is_causal: upper-left aligned (row i attends keys 0..i), aten.rs:10038.
 *   attn_mask: NULL or an additive mask in mask_dtype (query dtype or F32),
 *     broadcast to [B, Hq, L, S] through mask_strides[4] (0 = broadcast).
 *   scale: <= 0 or NaN means the default 1/sqrt(D).
 *   out: device row-major [B, Hq, L, D] in the input dtype (the CUDA result
 *     stays row-major, aten.rs:10436). lse: device row-major [B, Hq, L]
 *     float32, or NULL when the caller does not read it.
 * Refusals (aten.rs:10113-10172): dropout is not an argument here (the
 * Rust/Python side refuses dropout_p > 0 with upstream's text); D not in
 * {64, 128} or another unsupported combination -> TN_ERR_NOT_IMPLEMENTED. */
TN_API int tn_sdpa_flash_attention(const void *q, const void *k, const void *v, const void *attn_mask,
                            int mask_dtype, const int64_t *mask_strides, void *out, float *lse,
                            int dtype, int64_t B, int64_t Hq, int64_t Hkv, int64_t L, int64_t S,
                            int64_t D, const int64_t *q_strides, const int64_t *k_strides,
                            const int64_t *v_strides, int is_causal, double scale, void *stream);

/* Decode-time SDPA against a KV cache whose length lives on the device:
 * query [B, Hq, 1, D]; k_cache/v_cache [B, Hkv, capacity, D] (any b/h
 * strides, unit d stride); the first *len_dev + len_add keys are attended
 * (clamped to capacity). The work is planned for `capacity`, so one CUDA graph
 * of a decode step stays valid while the cache grows. Non-causal (a single
 * query row attends every cached key, as transformers calls it at decode).
 * Same arithmetic as tn_sdpa_flash_attention. */
TN_API int tn_sdpa_decode_cache(const void *q, const void *k_cache, const void *v_cache, void *out,
                                float *lse, int dtype, int64_t B, int64_t Hq, int64_t Hkv, int64_t D,
                                int64_t capacity, const int64_t *q_strides, const int64_t *k_strides,
                                const int64_t *v_strides, const int *len_dev, int64_t len_add,
                                double scale, void *stream);

/* The attention block of one decode token in one launch (bf16): from the
 * q/k/v projection rows qkv [B][(Hq + 2 Hkv) D] at position pos = *pos_dev,
 * rotate q and k (as tn_llama_rope_append), append k and v to cache slot pos,
 * attend keys [0, pos] (as tn_sdpa_decode_cache) and merge the key splits in
 * the last CTA of each KV head (no separate combine kernel). out: [B, Hq, D].
 * Hq / Hkv <= 8. Transformers runs these as apply_rotary_pos_emb, the cache
 * update and sdpa_attention_forward (-> aten.rs:10092 on the reference). */
TN_API int tn_sdpa_decode_step(const void *qkv, const float *inv_freq, void *k_cache, void *v_cache,
                               void *out, float *lse, int64_t B, int64_t Hq, int64_t Hkv, int64_t D,
                               int64_t capacity, const int64_t *k_strides, const int64_t *v_strides,
                               const int *pos_dev, double scale, void *stream);
/* The same, and out also as the next Q4_0 linear's planar Q8_0 activation
 * (codes [B][Hq D], scales / offsets [B][Hq D / 32]; the bytes
 * tn_q8_0_quantize_planar writes for out), each KV head's merging CTA
 * quantising its own rows. */
TN_API int tn_sdpa_decode_step_q8(const void *qkv, const float *inv_freq, void *k_cache, void *v_cache,
                                  void *out, float *lse, int8_t *codes, float *scales, float *offsets,
                                  int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t capacity,
                                  const int64_t *k_strides, const int64_t *v_strides, const int *pos_dev,
                                  double scale, void *stream);

/* ------------------------------------------------ decode-step glue (bf16) --
 * The work between the hot operators in one greedy token of transformers'
 * LlamaForCausalLM (modeling_llama.py: LlamaRMSNorm, apply_rotary_pos_emb,
 * LlamaMLP, the residual adds, argmax in generate), each producing what the
 * next Q4_0 linear reads: planar Q8_0 activations (see tn_q8_0_quantize_planar).
 * All tensors are bf16 unless stated; rows are contiguous. */

/* h_out = bf16(h + delta) (delta may be NULL; h_out may be NULL or == h);
 * y = weight * bf16(h32 * rsqrt(mean(h32^2) + eps)); y -> planar Q8_0. H % 32 == 0, H <= 8192. */
TN_API int tn_llama_add_rmsnorm_q8(const void *h, const void *delta, void *h_out, const void *weight,
                                   float eps, int64_t rows, int64_t H, int8_t *codes, float *scales,
                                   float *offsets, void *stream);
/* act = bf16(bf16(silu(gate)) * up) from rows [gate (I) | up (I)]; act -> planar Q8_0. */
TN_API int tn_llama_silu_mul_q8(const void *gate_up, int64_t rows, int64_t I, int8_t *codes,
                                float *scales, float *offsets, void *stream);
/* Rotary embedding (rotate_half convention, cos/sin rounded to bf16 as
 * transformers does) of the q and k heads of rows [q (Hq*D) | k (Hkv*D) | v (Hkv*D)]
 * at position pos = pos_dev ? *pos_dev : pos_host; q -> q_out [B, Hq, D];
 * rotated k and v -> slot pos of k_cache/v_cache (element strides cache_b_stride,
 * cache_h_stride, slot stride D). inv_freq: f32 [D/2] on the device. */
TN_API int tn_llama_rope_append(const void *qkv, const float *inv_freq, const int *pos_dev,
                                int64_t pos_host, int64_t B, int64_t Hq, int64_t Hkv, int64_t D,
                                void *q_out, void *k_cache, void *v_cache, int64_t cache_b_stride,
                                int64_t cache_h_stride, void *stream);
/* tokens[r] = argmax(logits[r]) (first index of the maximum); h[r] = embed[tokens[r]];
 * if pos_dev, *pos_dev += 1. */
TN_API int tn_llama_argmax_embed(const void *logits, int64_t rows, int64_t V, int *tokens,
                                 const void *embed, int64_t H, void *h, int *pos_dev, void *stream);
/* h[r] = embed[tokens[r]]. */
TN_API int tn_llama_embed(const int *tokens, int64_t rows, const void *embed, int64_t H, void *h,
                          void *stream);

/* ---- one greedy decode token in one persistent kernel (batch 1) ---------------
 * The whole token of a Llama-shaped Q4_0 model -- per layer RMSNorm + q/k/v,
 * RoPE + KV append + attention, o_proj + residual, RMSNorm + gate/up +
 * SiLU*up, down_proj + residual; then the final norm, lm_head and argmax --
 * as ONE launch of one CTA per SM. Each CTA streams its rows of every weight
 * matrix and its split of every layer's past K/V through a bulk-copy ring
 * while its math waits on grid-wide phase barriers for activations only.
 * Same arithmetic per operator as the separate kernels (Q8_0 activations and
 * exact integer block dots for every Q4_0 linear, k_quants.rs:312-330; the
 * default SDPA arithmetic, aten.rs:10327-10420). No reference counterpart as
 * one call: the reference runs these as transformers' modules around
 * _quantized_linear (quant.rs:286-369) and the flash op (aten.rs:10092), one
 * op at a time.
 *
 * The model: every pointer device memory except the per-layer arrays, which
 * are host arrays of `layers` device pointers. Q4_0 blobs as tn_q4_0_linear
 * reads them (16-byte aligned); qkv rows are q heads, then k heads, then v
 * heads; gate_up rows interleave gate_proj and up_proj row by row; caches are
 * bf16 [1][kv_heads][capacity][head_dim]; norms and the embedding bf16;
 * inv_freq f32 [head_dim / 2]. Supported: head_dim 128, heads = 4 kv_heads,
 * hidden and inter multiples of 256 (hidden <= 5632, inter <= 16384). */
typedef struct {
    int32_t layers, hidden, inter, heads, kv_heads, head_dim, vocab;
    float eps;
    const void *embed, *final_norm, *lm_head;
    const void *const *attn_norm, *const *qkv, *const *o, *const *mlp_norm, *const *gate_up, *const *down;
    void *const *k_cache, *const *v_cache;
    int64_t capacity;
    const float *inv_freq;
} tn_llama_q4_model;
/* The kernel's workspace, owned by the caller: byte offsets (256-aligned) of
 * its buffers and the total size. After a token: h the residual stream
 * (bf16 [hidden], the last layer's output), qkv (bf16 q/k/v rows of the last
 * layer), attn (bf16 attention output [heads * head_dim]) with its planar
 * Q8_0 (aq codes, ad scales, ac offsets), o_out (bf16 o_proj output), act
 * (bf16 SiLU(gate) * up [inter]) with its planar Q8_0 (gq, gd, gc), down_out
 * (bf16 down_proj output); layers, part_o, part_ml, amax, sync are the
 * kernel's own. */
typedef struct {
    int64_t total, layers, h, qkv, attn, act, o_out, down_out, aq, ad, ac, gq, gd, gc, part_o, part_ml, amax, sync;
} tn_llama_decode_layout;
TN_API int tn_llama_decode_layout_of(const tn_llama_q4_model *model, tn_llama_decode_layout *layout);
/* Build the launch plan over a caller-provided workspace (256-byte aligned
 * device memory of layout.total bytes, zero-filled before the first token):
 * copies the layer table into it (cudaMemcpy) and checks the kernel fits;
 * allocates no device memory. The plan is a small host object. */
TN_API int tn_llama_decode_plan(const tn_llama_q4_model *model, void *workspace, int64_t workspace_bytes,
                                void **plan);
/* One token: reads tokens[0] (the current token id) and *pos (its position;
 * the cache holds positions [0, pos)), writes the bf16 logits [vocab], the
 * next token id into tokens[0] and pos + 1 into *pos; appends this token's
 * K/V at slot pos. tokens and pos are device ints. trace (or NULL): device
 * bytes of tn_llama_decode_trace_bytes(plan), receiving the exact Q8_0 input
 * tiles of trace_layer's q/k/v and gate/up linears and of lm_head (for
 * checking each linear on its own inputs). A bounded wait that gives up makes
 * the launch record TN_ERR_TIMEOUT (tn_device_status); call
 * tn_llama_decode_reset before the next token. Cooperative launch: every
 * CTA is resident at once. */
TN_API int tn_llama_decode_token(void *plan, int *tokens, int *pos, void *logits, void *trace, int trace_layer,
                                 void *stream);
TN_API int64_t tn_llama_decode_trace_bytes(const void *plan);
/* tn_llama_decode_token that also records its phase timeline (models of two or
 * more layers): stamps, device uint64 [grid CTAs][64], receives %globaltimer
 * (ns) per CTA for layer 1 -- [0] kernel start; [1..10] after the grid wait and
 * after the work of the Q (RMSNorm + q/k/v), A (attention), O (o_proj), G
 * (gate/up) and D (down_proj) phases; [11..16] when the CTA's producer started
 * issuing the ring items of each of those phases and finished the layer's;
 * [17] the CTA's final arrival; [18..61] finer points inside the Q and A
 * phases (prologue done, per-warp item and K/V-tile times). The grid size is
 * the device's SM count. A diagnostic of the kernel's schedule. */
TN_API int tn_llama_decode_token_timeline(void *plan, int *tokens, int *pos, void *logits, uint64_t *stamps,
                                          void *stream);
/* Zero the plan's barrier counter, epoch and merge tickets (stream-ordered). */
TN_API int tn_llama_decode_reset(void *plan, void *stream);
TN_API int tn_llama_decode_plan_free(void *plan);

/* ---- tensor parallelism (column-sharded linears, KV-head-group attention) -----
 * The reference has no multi-GPU path; this is the layout step of the
 * north star's per-layer all-gather: an all-gather of per-rank [rows][cols]
 * blocks of 16-bit elements lands as src [G][rows][cols]; dst [rows][G*cols]
 * is what the next layer reads. src and dst must not overlap. */
TN_API int tn_tp_unshard(const void *src, void *dst, int64_t G, int64_t rows, int64_t cols, void *stream);

/* The same all-gather over peer memory (NVLink / NVSwitch) instead of a
 * library collective. Each rank allocates one exchange region (zeroed; its
 * first tn_tp_region_data_offset() bytes hold the step epoch and the
 * per-gather counters) and shares it through a CUDA IPC handle of
 * TN_IPC_HANDLE_BYTES bytes; every other rank opens it. tn_tp_allgather then
 * stores this rank's [rows][cols] slice of 16-bit elements (local, row stride
 * local_row_stride elements) into row r, columns [rank*cols, (rank+1)*cols)
 * of the [rows][dst_row_stride] buffer at byte `dst_offset` of every rank's
 * data area, signals, and returns (in stream order) once every rank's slice
 * has arrived in this rank's region. `slot` numbers the gathers of one step
 * (each used once per step; consecutive gathers must use different buffers);
 * tn_tp_step_end advances the epoch after the step's last gather. bases[g] is
 * rank g's region as mapped in this process (its own base for g == rank).
 * Waits are bounded: a rank that never signals makes the call record
 * TN_ERR_TIMEOUT for tn_device_status instead of hanging. */
#define TN_IPC_HANDLE_BYTES 64
TN_API int tn_tp_region_alloc(size_t bytes, void **base, void *ipc_handle);
TN_API int tn_tp_region_open(const void *ipc_handle, void **peer_base);
TN_API int tn_tp_region_close(void *peer_base);
TN_API int tn_tp_region_free(void *base);
TN_API int64_t tn_tp_region_data_offset(void);
TN_API int tn_tp_allgather(void *const *bases, int rank, int world, const void *local, int64_t local_row_stride,
                           int64_t rows, int64_t cols, int64_t dst_offset, int64_t dst_row_stride, int slot,
                           void *stream);
TN_API int tn_tp_step_end(void *local_base, void *stream);

/* The all-gather fused into the Q4_0 GEMV itself. As producer (slot >= 0)
 * the GEMV stores its output rows straight into every rank's region (row m,
 * columns [rank*N_out, (rank+1)*N_out) of the [M][dst_row_stride] buffer at
 * byte dst_offset of the data area, N_out its output columns) instead of y,
 * and its last CTA signals every rank; as consumer (wait_slot >= 0) it waits,
 * bounded, until every rank's producer of wait_slot has signalled this step
 * before reading its activations. Slots share the numbering of
 * tn_tp_allgather; a slot is fed either by tn_tp_allgather or by fused
 * producers, never both.
 *
 * reduce = 1 makes the GEMV a row-parallel linear with its all-reduce fused
 * in (transformers' "rowwise" plan: each rank holds a K-slice of the weight,
 * whole Q4_0 blocks of every row): every CTA stores its f32 partial outputs,
 * each as one 8-byte word {value, tag = epoch * 256 + slot + 1}, into every
 * rank's [M][dst_row_stride] buffer of 8-byte words at row m, columns
 * [rank*N, (rank+1)*N) (dst_row_stride >= world*N), then polls (bounded)
 * the words of its own columns until every rank's carries this launch's tag,
 * and writes y = sum over ranks g = 0..world-1, in that order, of the
 * partials -- the same bits on every rank; no fence and no separate signal.
 * `slot` numbers the reductions of a step (< TN_TP_REDUCE_SLOTS, each once
 * per step, tn_tp_step_end after the step); consecutive reductions must
 * alternate between two buffers. No bias, no pair epilogue, wait_slot -1.
 * The result differs from the one-GPU linear only in the association of its
 * f32 sum (within the same counted bound). */
#define TN_TP_REDUCE_SLOTS 256
typedef struct {
    int world, rank;
    void *bases[8];
    int64_t dst_offset;
    int64_t dst_row_stride;
    int slot;
    int wait_slot;
    int reduce;
    int reserved;
} tn_tp_link;
TN_API int tn_q4_0_linear_q8_tp(const int8_t *codes, int64_t codes_row_stride, const float *scales,
                                const float *offsets, const void *w_blob, const float *bias, void *y,
                                int y_dtype, int64_t M, int64_t N, int64_t K, int flags,
                                const tn_tp_link *link, void *stream);
TN_API int tn_q4_0_linear_fused_tp(int x_mode, const void *x, int64_t x_row_stride, const void *delta,
                                   void *h_out, const void *norm_weight, float eps, const void *w_blob,
                                   const float *bias, void *y, int y_dtype, int64_t M, int64_t N, int64_t K,
                                   int flags, const tn_tp_link *link, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* TORCHNATIVE_B200_H */
