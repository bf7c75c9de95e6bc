/*
 * tn_oracle.h -- CPU restatement of torchnative's arithmetic for the two hot
 * operators (GGML Q4_0 weight-only linear, and
 * aten._scaled_dot_product_flash_attention_for_cpu).
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker and the timed
 * CPU baseline. Nothing in the product path (torchnative_b200/) links, loads
 * or calls it; only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference arms do.
 *
 * Parity pinning: the Q4_0/Q8_0 codec functions are checked byte for byte and
 * bit for bit against llama.cpp gguf-py's answers frozen in
 * tests/golden/q4_gguf_golden.json (extracted from the reference's
 * scripts/q4quality/golden_gguf_py.json), and against the installed gguf-py
 * codec on seeded inputs. The SDPA restatement is checked against upstream
 * torch 2.11's CPU kernel on the reference's golden SDPA cases
 * (tests/golden/sdpa_golden.json), within the reference's per-dtype
 * tolerances.
 *
 * All paths below are relative to the reference project root.
 */
#ifndef TN_ORACLE_H
#define TN_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- scalar conversions (IEEE 754, round to nearest even) ---------------- */
uint16_t tno_f32_to_f16(float f);
float tno_f16_to_f32(uint16_t h);
uint16_t tno_f32_to_bf16(float f);
float tno_bf16_to_f32(uint16_t b);

/* ---- GGML Q4_0 / Q8_0 block codecs --------------------------------------- */
/* Q4_0 writer: BlockQ4_0::from_float,
 * torchnative/rust/vendor/candle-core/src/quantized/k_quants.rs:241-277.
 * n must be a multiple of 32; blob receives n/32 blocks of 18 bytes. */
void tno_q4_0_quantize(const float *x, uint8_t *blob, int64_t n);
/* Q4_0 reader: BlockQ4_0::to_float, k_quants.rs:219-239. */
void tno_q4_0_dequantize(const uint8_t *blob, float *y, int64_t n);
/* Q8_0 writer (the activation quantiser of the CPU matmul):
 * BlockQ8_0::from_float, k_quants.rs:676-706. 34-byte blocks. */
void tno_q8_0_quantize(const float *x, uint8_t *blob, int64_t n);
/* Q8_0 reader: BlockQ8_0::to_float, k_quants.rs:660-674. */
void tno_q8_0_dequantize(const uint8_t *blob, float *y, int64_t n);

/* One output element: BlockQ4_0::vec_dot_unopt, k_quants.rs:312-330 -- the
 * arithmetic of the x86_64 wheel (built without target-feature avx2). */
float tno_q4_0_q8_0_dot(const uint8_t *w_row, const uint8_t *xq_row, int64_t nblocks);

/* torch._C._quantized_linear on CPU (quant.rs:286-369): y[M,N] = x[M,K] W^T
 * (+ bias). Activations are quantised row by row to Q8_0 first, then every
 * output element is one tno_q4_0_q8_0_dot; the 4-column quads are split over
 * `threads` workers as k_quants::matmul does (k_quants.rs:2430-2580); the
 * partition does not change any value. Bias, if given, is added afterwards in
 * float32 (quant.rs:350-365). */
void tno_q4_0_linear(const float *x, const uint8_t *w_blob, const float *bias, float *y,
                     int64_t M, int64_t N, int64_t K, int threads);

/* One output element for a Q8_0 weight: BlockQ8_0::vec_dot_unopt,
 * k_quants.rs:737-756 (integer block sum, then (sum * d_w) * d_x added in
 * order). */
float tno_q8_0_q8_0_dot(const uint8_t *w_row, const uint8_t *xq_row, int64_t nblocks);

/* Q4_K reader: BlockQ4K::to_float, k_quants.rs:1722-1748 (144-byte
 * super-blocks of 256, 6-bit scales/mins by get_scale_min_k4, utils.rs:50-60). */
void tno_q4_k_dequantize(const uint8_t *blob, float *y, int64_t n);
/* Q8_K activation writer: BlockQ8K::from_float, k_quants.rs:2376-2410
 * (292-byte blocks: f32 d, 256 int8 codes, 16 int16 sums of 16). */
void tno_q8_k_quantize(const float *x, uint8_t *blob, int64_t n);
/* One output element for a Q4_K weight: BlockQ4K::vec_dot_unopt,
 * k_quants.rs:1478-1544. */
float tno_q4_k_q8_k_dot(const uint8_t *w_row, const uint8_t *xq_row, int64_t nsuper);
/* torch._C._quantized_linear for a Q4_K weight (N rows of K/256 super-blocks),
 * activations quantised to Q8_K row by row. */
void tno_q4_k_linear(const float *x, const uint8_t *w_blob, const float *bias, float *y,
                     int64_t M, int64_t N, int64_t K, int threads);

/* torch._C._quantized_linear for a Q8_0 weight (N rows of 34-byte blocks):
 * the same steps as tno_q4_0_linear with tno_q8_0_q8_0_dot per element. */
void tno_q8_0_linear(const float *x, const uint8_t *w_blob, const float *bias, float *y,
                     int64_t M, int64_t N, int64_t K, int threads);

/* ---- scaled_dot_product_attention ----------------------------------------
 * sdpa_flash_cpu's default branch, torchnative/rust/torch_c/src/aten.rs:
 * 10092-10460 (arithmetic 10327-10420), GQA through repeat_kv_heads
 * (aten.rs:17106-17130: query head h reads key/value head h / (Hq/Hkv)).
 *
 * dtype: 0 = f32, 1 = f16, 2 = bf16 (inputs widened to f32, output narrowed
 * back, logsumexp f32), 3 = f64 (all in f64, logsumexp f64).
 * Strides are in elements, [b, h, t, d] order. mask (optional) is an additive
 * mask in `mask_dtype` (same codes) broadcast with the given strides (0 for a
 * broadcast dimension), shape [B, Hq, L, S] after broadcasting.
 * Output `out` is row-major [B, Hq, L, D] in `dtype`; `lse` is row-major
 * [B, Hq, L] in f32 (f64 when dtype == 3). */
void tno_sdpa(const void *q, const void *k, const void *v, const void *mask, int mask_dtype,
              const int64_t *mask_strides, void *out, void *lse, int dtype, int64_t B, int64_t Hq,
              int64_t Hkv, int64_t L, int64_t S, int64_t D, const int64_t *q_strides,
              const int64_t *k_strides, const int64_t *v_strides, int is_causal, double scale,
              int threads);

#ifdef __cplusplus
}
#endif
#endif
