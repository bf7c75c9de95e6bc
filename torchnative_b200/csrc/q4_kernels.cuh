// q4_kernels.cuh -- internal launchers shared by the Q4_0 translation units.
#pragma once

#include "tn_common.cuh"

namespace tn {

// Planar Q8_0 activations (see q4_codec.cu): codes [rows][xq_row_stride] int8,
// xd [rows][nb] f32 widened scale, xc [rows][nb] f32 = 12582912 + 8 * sum(codes).
int launch_q8_planar(const void *x, int x_dtype, int64_t row_stride, int8_t *xq, float *xd, float *xc, int64_t rows,
                     int64_t nb, int64_t xq_row_stride, cudaStream_t stream);

// Planar Q8_0 with the codes as f16 (the tensor-core GEMM's A operand):
// xq [rows][xq_row_stride] f16, xd [rows][nb] f32.
int launch_q8_planar_f16(const void *x, int x_dtype, int64_t row_stride, __half *xq, float *xd, int64_t rows,
                         int64_t nb, int64_t xq_row_stride, cudaStream_t stream);

// Prefill Q4_0 x Q8_0 GEMM on tcgen05 (M > 16): codes f16 [M][xq_row_stride],
// xd [M][K/32]; needs K % 256 == 0 and a 16-byte aligned blob.
bool q4_gemm_applies(const void *w_blob, int64_t M, int64_t N, int64_t K);
// Activation-row count from which tn_q4_0_linear takes the GEMM instead of
// row chunks of the decode GEMV.
constexpr int64_t kQ4GemmMinRows = 48;
int launch_q4_gemm(const __half *xq, int64_t xq_row_stride, const float *xd, const uint8_t *w, const float *bias,
                   void *y, int y_dtype, int64_t y_row_stride, int64_t M, int64_t N, int64_t K, cudaStream_t stream);

// Batched decode (kQ4SkinnyMinRows <= M <= kQ4SkinnyMaxRows) on tcgen05 with
// the weights on the MMA's 128-row side: planar Q8_0 activations (codes
// [M][xq_row_stride] int8, 16-byte aligned rows; xd and xc [M][K/32], 16-byte
// aligned); needs K % 256 == 0 and a 16-byte aligned blob. flags:
// TN_EPILOGUE_SILU_MUL_PAIRS.
// From 9 rows on (below, the GEMV's 2-CTA plans stream faster; at 16 rows the
// GEMV needs row chunks for K = 14336 and this kernel halves down_proj).
constexpr int64_t kQ4SkinnyMinRows = 9, kQ4SkinnyMaxRows = 32;
bool q4_skinny_applies(const void *w_blob, const float *xd, const float *xc, int64_t M, int64_t N, int64_t K,
                       int flags);
int launch_q4_skinny(const int8_t *xq, int64_t xq_row_stride, const float *xd, const float *xc, const uint8_t *w,
                     const float *bias, void *y, int y_dtype, int64_t y_row_stride, int M, int64_t N, int64_t K,
                     int flags, cudaStream_t stream);

// Largest activation-row count (<= 16) one GEMV launch holds in shared memory
// for this K (wfmt 0: Q4_0 weights, 1: Q8_0 weights); 0 if even one row does
// not fit.
int q4_gemv_max_rows(int64_t K, int wfmt = 0);

// Decode GEMV of Q8_0 weights (34-byte GGML blocks) over planar Q8_0
// activations (offsets unused): y[m, n] for m < M (M <= 16).
int launch_q8w_gemv(const uint8_t *w, const int8_t *xq, const float *xd, const float *xc, int64_t xq_row_stride,
                    const float *bias, void *y, int y_dtype, int64_t y_row_stride, int M, int64_t N, int64_t K,
                    int flags, cudaStream_t stream);

// Decode GEMV of Q4_K weights (144-byte super-blocks of 256) over planar Q8_K
// activations: codes, per 32-block the super-block's d (xd) and the block's
// code sum (xc); y[m, n] for m < M (M <= 16). Rows must be 16-byte aligned.
int launch_q4k_gemv(const uint8_t *w, const int8_t *xq, const float *xd, const float *xc, int64_t xq_row_stride,
                    const float *bias, void *y, int y_dtype, int64_t y_row_stride, int M, int64_t N, int64_t K,
                    cudaStream_t stream);

// The float-activation mode (TN_ACT_FLOAT) for M <= 16: weights dequantised
// exactly to f32, x widened from f32 / bf16 / f16, f32 accumulate (q4_float.cu).
int launch_q4_float_gemv(const uint8_t *w, const void *x, int x_dtype, int64_t x_row_stride, const float *bias,
                         void *y, int y_dtype, int64_t y_row_stride, int M, int64_t N, int64_t K,
                         cudaStream_t stream);

// Decode GEMV over planar Q8_0 activations: y[m, n] for m < M (M <= 16).
int launch_q4_gemv_q8(const uint8_t *w, const int8_t *xq, const float *xd, const float *xc, int64_t xq_row_stride,
                      const float *bias, void *y, int y_dtype, int64_t y_row_stride, int M, int64_t N, int64_t K,
                      int flags, cudaStream_t stream, const tn_tp_link *link = nullptr);

// Planar Q8_0 of a GEMV's own bf16 output (the next linear's activations):
// codes [M][codes_row_stride], scales and offsets [M][out_cols / 32].
struct Q8Out {
    int8_t *codes;
    int64_t codes_row_stride;
    float *scales;
    float *offsets;
};

// Decode GEMV whose planar Q8_0 activations are built in each CTA from bf16
// rows (x_mode: 1 = x itself, 2 = RMSNorm(h + delta) with h + delta written to
// xh_out by CTA 0, 3 = silu(gate) * up from [gate | up] rows); M <= 4. With
// `q8` (bf16 y, out_cols % 32 == 0, no link), each CTA also quantises its
// whole 32-column blocks of y.
int launch_q4_gemv_fused(int x_mode, const void *xb, int64_t xb_row_stride, const void *xdelta, void *xh_out,
                         const void *norm_w, float eps, const uint8_t *w, const float *bias, void *y, int y_dtype,
                         int64_t y_row_stride, int M, int64_t N, int64_t K, int flags, cudaStream_t stream,
                         const tn_tp_link *link = nullptr, const Q8Out *q8 = nullptr);

}  // namespace tn
