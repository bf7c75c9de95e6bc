// q4_linear.cu -- tn_q4_0_linear: the C-ABI door of torch._C._quantized_linear
// (torch_c/src/quant.rs:286-369) on a B200. Checks in the reference's order and
// wording, quantises the activations to Q8_0 (k_quants.rs:2479-2510 does the
// same on the CPU), and launches the decode GEMV in chunks of at most 16
// activation rows.
#include "q4_kernels.cuh"

namespace tn {
namespace {

int check_link(const std::string &op, const tn_tp_link *l, int64_t out_cols, int flags = 0,
               const float *bias = nullptr) {
    if (l->world < 1 || l->world > kTpMaxRanks || l->rank < 0 || l->rank >= l->world)
        return set_error(TN_ERR_INVALID, op + ": tensor-parallel link: rank/world out of range (at most 8 ranks)");
    for (int g = 0; g < l->world; ++g)
        if (!l->bases[g]) return set_error(TN_ERR_INVALID, op + ": tensor-parallel link: null region base");
    if (l->reduce) {
        if (l->reduce != 1) return set_error(TN_ERR_INVALID, op + ": tensor-parallel link: reduce is 0 or 1");
        if (l->slot < 0 || l->slot >= kTpRedSlots || l->wait_slot >= 0)
            return set_error(TN_ERR_INVALID, op + ": tensor-parallel reduce: slot in [0, 256) and no wait_slot");
        if (bias || (flags & TN_EPILOGUE_SILU_MUL_PAIRS))
            return set_error(TN_ERR_NOT_IMPLEMENTED,
                             op + ": tensor-parallel reduce: no bias and no pair epilogue (partials are summed)");
        if (l->dst_offset < 0 || (l->dst_offset & 3) != 0 || l->dst_row_stride < l->world * out_cols)
            return set_error(TN_ERR_SHAPE, op + ": tensor-parallel reduce: 4-byte aligned destination with a row "
                                                "stride of at least world * columns");
        return TN_OK;
    }
    const int64_t max_slot = (kTpTicketOff - kTpCountOff) / 4 / l->world;
    if (l->slot >= max_slot || l->wait_slot >= max_slot)
        return set_error(TN_ERR_INVALID, op + ": tensor-parallel link: slot out of range");
    if (l->slot >= 0 && (l->dst_offset < 0 || l->dst_row_stride < l->world * out_cols))
        return set_error(TN_ERR_SHAPE, op + ": tensor-parallel link: destination row stride below world * columns");
    return TN_OK;
}

}  // namespace
}  // namespace tn

extern "C" int tn_q4_0_linear(const void *x, int x_dtype, int64_t x_row_stride, const void *w_blob, const float *bias,
                              void *y, int y_dtype, int64_t M, int64_t N, int64_t K, int act_mode, void *stream_) {
    const std::string op = "torch._C._quantized_linear";
    cudaStream_t stream = tn::stream_of(stream_);
    __atomic_fetch_add(&tn::counters().q4_linear_calls, 1ull, __ATOMIC_RELAXED);
    if (x_dtype != TN_F32 && x_dtype != TN_BF16 && x_dtype != TN_F16)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": the activation must be torch.float32, torch.bfloat16 or "
                                                          "torch.float16 on CUDA, got " +
                                                          tn_dtype_name(x_dtype));
    if (y_dtype != TN_F32 && y_dtype != TN_BF16 && y_dtype != TN_F16)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": unsupported output dtype " + tn_dtype_name(y_dtype));
    if (act_mode != TN_ACT_Q8_0 && act_mode != TN_ACT_FLOAT)
        return tn::set_error(TN_ERR_INVALID, op + ": unknown activation mode " + std::to_string(act_mode));
    if (M < 0 || N < 0 || K < 0)
        return tn::set_error(TN_ERR_SHAPE, op + ": negative size");
    if (K % 32 != 0)
        return tn::set_error(TN_ERR_SHAPE, op + ": mat1 and mat2 shapes cannot be multiplied ([" + std::to_string(M) +
                                               ", " + std::to_string(K) + "] and " + std::to_string(K) + "x" +
                                               std::to_string(N) + "): a q4_0 row is whole 32-element blocks");
    if (M == 0 || N == 0) return TN_OK;
    if (K == 0) return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": in_features == 0 is not implemented");
    if (!x || !w_blob || !y) return tn::set_error(TN_ERR_INVALID, op + ": null device pointer");
    if (x_row_stride < K) return tn::set_error(TN_ERR_INVALID, op + ": activation row stride smaller than in_features");
    if ((reinterpret_cast<uintptr_t>(w_blob) & 1) != 0)
        return tn::set_error(TN_ERR_INVALID, op + ": the q4_0 blob must be at least 2-byte aligned");
    if (act_mode == TN_ACT_FLOAT) {
        // no activation quantisation: exact f32 weights times the widened
        // activations, f32 accumulate (decode-sized inputs)
        if (M > 16)
            return tn::set_error(TN_ERR_NOT_IMPLEMENTED,
                                 op + ": the float-activation mode runs at most 16 activation rows on CUDA; use the "
                                      "Q8_0 mode (the reference's arithmetic) for more");
        return tn::launch_q4_float_gemv(static_cast<const uint8_t *>(w_blob), x, x_dtype, x_row_stride, bias, y,
                                        y_dtype, N, (int)M, N, K, stream);
    }

    const int64_t nb = K / 32;
    void *ws = nullptr;
    int st;
    if (x_dtype == TN_BF16 && M == 1 && K <= 4096 && K % 256 == 0 &&
        ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w_blob) | (uintptr_t)(x_row_stride * 2)) &
         15) == 0)
        // One bf16 row of a short K: every CTA quantises it to Q8_0 in its own
        // prologue (the same codes tn_q8_0_quantize_planar writes, 128 blocks
        // per CTA), one launch instead of quantiser + GEMV. (At 4 rows the
        // repeated prologue costs more than the launch it saves.)
        return tn::launch_q4_gemv_fused(TN_X_BF16, x, x_row_stride, nullptr, nullptr, nullptr, 0.0f,
                                        static_cast<const uint8_t *>(w_blob), bias, y, y_dtype, N, (int)M, N, K, 0,
                                        stream, nullptr, nullptr);
    if (M >= tn::kQ4GemmMinRows && tn::q4_gemm_applies(w_blob, M, N, K)) {
        // Many rows: f16 Q8 codes [M][K] and scales [M][nb] for the tensor-core GEMM.
        const size_t codes16 = ((size_t)M * K * 2 + 255) & ~size_t(255);
        st = tn::workspace(&ws, codes16 + (size_t)M * nb * 4 + 256, stream, /*slot=*/0);
        if (st) return st;
        __half *xq16 = static_cast<__half *>(ws);
        float *xd16 = reinterpret_cast<float *>(static_cast<uint8_t *>(ws) + codes16);
        st = tn::launch_q8_planar_f16(x, x_dtype, x_row_stride, xq16, xd16, M, nb, K, stream);
        if (st) return st;
        return tn::launch_q4_gemm(xq16, K, xd16, static_cast<const uint8_t *>(w_blob), bias, y, y_dtype, N, M, N, K,
                                  stream);
    }
    // Workspace: codes [M][K] int8, scales [M][nb] f32, offsets [M][nb] f32.
    const size_t codes = (size_t)M * K, scal = (size_t)M * nb * 4;
    st = tn::workspace(&ws, codes + 2 * scal + 256, stream, /*slot=*/0);
    if (st) return st;
    int8_t *xq = static_cast<int8_t *>(ws);
    float *xd = reinterpret_cast<float *>(static_cast<uint8_t *>(ws) + ((codes + 15) & ~size_t(15)));
    float *xc = xd + (size_t)M * nb;
    st = tn::launch_q8_planar(x, x_dtype, x_row_stride, xq, xd, xc, M, nb, K, stream);
    if (st) return st;
    if (tn::q4_skinny_applies(w_blob, xd, xc, M, N, K, 0))  // batched decode: the tensor cores
        return tn::launch_q4_skinny(xq, K, xd, xc, static_cast<const uint8_t *>(w_blob), bias, y, y_dtype, N, (int)M,
                                    N, K, 0, stream);

    const int chunk = tn::q4_gemv_max_rows(K);
    if (chunk <= 0)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": in_features " + std::to_string(K) +
                                                         " is too large for the decode kernel's shared memory");
    const size_t ysz = tn_dtype_size(y_dtype);
    for (int64_t m0 = 0; m0 < M; m0 += chunk) {
        const int mc = (int)((M - m0) < chunk ? (M - m0) : chunk);
        st = tn::launch_q4_gemv_q8(static_cast<const uint8_t *>(w_blob), xq + m0 * K, xd + m0 * nb, xc + m0 * nb, K,
                                   bias, static_cast<uint8_t *>(y) + (size_t)m0 * N * ysz, y_dtype, N, mc, N, K,
                                   0, stream);
        if (st) return st;
    }
    return TN_OK;
}

extern "C" int tn_q8_0_linear(const void *x, int x_dtype, int64_t x_row_stride, const void *w_blob, const float *bias,
                              void *y, int y_dtype, int64_t M, int64_t N, int64_t K, int act_mode, void *stream_) {
    const std::string op = "torch._C._quantized_linear";
    cudaStream_t stream = tn::stream_of(stream_);
    __atomic_fetch_add(&tn::counters().q4_linear_calls, 1ull, __ATOMIC_RELAXED);
    if (x_dtype != TN_F32 && x_dtype != TN_BF16 && x_dtype != TN_F16)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": the activation must be torch.float32, torch.bfloat16 or "
                                                          "torch.float16 on CUDA, got " +
                                                          tn_dtype_name(x_dtype));
    if (y_dtype != TN_F32 && y_dtype != TN_BF16 && y_dtype != TN_F16)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": unsupported output dtype " + tn_dtype_name(y_dtype));
    if (act_mode != TN_ACT_Q8_0 && act_mode != TN_ACT_FLOAT)
        return tn::set_error(TN_ERR_INVALID, op + ": unknown activation mode " + std::to_string(act_mode));
    if (M < 0 || N < 0 || K < 0) return tn::set_error(TN_ERR_SHAPE, op + ": negative size");
    if (K % 32 != 0)
        return tn::set_error(TN_ERR_SHAPE, op + ": mat1 and mat2 shapes cannot be multiplied ([" + std::to_string(M) +
                                               ", " + std::to_string(K) + "] and " + std::to_string(K) + "x" +
                                               std::to_string(N) + "): a q8_0 row is whole 32-element blocks");
    if (M == 0 || N == 0) return TN_OK;
    if (K == 0) return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": in_features == 0 is not implemented");
    if (!x || !w_blob || !y) return tn::set_error(TN_ERR_INVALID, op + ": null device pointer");
    if (x_row_stride < K) return tn::set_error(TN_ERR_INVALID, op + ": activation row stride smaller than in_features");
    if ((reinterpret_cast<uintptr_t>(w_blob) & 1) != 0)
        return tn::set_error(TN_ERR_INVALID, op + ": the q8_0 blob must be at least 2-byte aligned");
    if (act_mode == TN_ACT_FLOAT)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED,
                             op + ": the float-activation mode is not implemented on CUDA yet; use the Q8_0 mode "
                                  "(the reference's arithmetic)");
    const int chunk = tn::q4_gemv_max_rows(K, 1);
    if (chunk <= 0)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": in_features " + std::to_string(K) +
                                                         " is too large for the decode kernel's shared memory");
    const int64_t nb = K / 32;
    void *ws = nullptr;
    const size_t codes = (size_t)M * K, scal = (size_t)M * nb * 4;
    int st = tn::workspace(&ws, codes + 2 * scal + 256, stream, /*slot=*/0);
    if (st) return st;
    int8_t *xq = static_cast<int8_t *>(ws);
    float *xd = reinterpret_cast<float *>(static_cast<uint8_t *>(ws) + ((codes + 15) & ~size_t(15)));
    float *xc = xd + (size_t)M * nb;
    st = tn::launch_q8_planar(x, x_dtype, x_row_stride, xq, xd, xc, M, nb, K, stream);
    if (st) return st;
    const size_t ysz = tn_dtype_size(y_dtype);
    for (int64_t m0 = 0; m0 < M; m0 += chunk) {
        const int mc = (int)((M - m0) < chunk ? (M - m0) : chunk);
        st = tn::launch_q8w_gemv(static_cast<const uint8_t *>(w_blob), xq + m0 * K, xd + m0 * nb, xc + m0 * nb, K,
                                 bias, static_cast<uint8_t *>(y) + (size_t)m0 * N * ysz, y_dtype, N, mc, N, K, 0,
                                 stream);
        if (st) return st;
    }
    return TN_OK;
}

extern "C" int tn_q8_0_quantize_planar(const void *x, int x_dtype, int64_t x_row_stride, int8_t *codes,
                                       int64_t codes_row_stride, float *scales, float *offsets, int64_t rows,
                                       int64_t cols, void *stream) {
    const std::string op = "torch._C._quantize";
    if (x_dtype != TN_F32 && x_dtype != TN_BF16 && x_dtype != TN_F16)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": q8_0 activations must be torch.float32, torch.bfloat16 "
                                                          "or torch.float16, got " +
                                                          tn_dtype_name(x_dtype));
    if (rows < 0 || cols < 0 || cols % 32 != 0 || x_row_stride < cols || codes_row_stride < cols ||
        codes_row_stride % 16 != 0)
        return tn::set_error(TN_ERR_SHAPE, op + ": planar q8_0 needs cols % 32 == 0 and code rows of a 16-byte "
                                                "multiple stride");
    if (rows == 0 || cols == 0) return TN_OK;
    if (!x || !codes || !scales || !offsets) return tn::set_error(TN_ERR_INVALID, op + ": null device pointer");
    if ((reinterpret_cast<uintptr_t>(codes) & 15) != 0)
        return tn::set_error(TN_ERR_INVALID, op + ": codes must be 16-byte aligned");
    return tn::launch_q8_planar(x, x_dtype, x_row_stride, codes, scales, offsets, rows, cols / 32, codes_row_stride,
                                tn::stream_of(stream));
}

extern "C" int tn_q4_0_linear_q8_tp(const int8_t *codes, int64_t codes_row_stride, const float *scales,
                                    const float *offsets, const void *w_blob, const float *bias, void *y,
                                    int y_dtype, int64_t M, int64_t N, int64_t K, int flags,
                                    const tn_tp_link *link, void *stream_) {
    const std::string op = "torch._C._quantized_linear";
    cudaStream_t stream = tn::stream_of(stream_);
    __atomic_fetch_add(&tn::counters().q4_linear_calls, 1ull, __ATOMIC_RELAXED);
    if (y_dtype != TN_F32 && y_dtype != TN_BF16 && y_dtype != TN_F16)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": unsupported output dtype " + tn_dtype_name(y_dtype));
    if (M < 0 || N < 0 || K < 0 || K % 32 != 0)
        return tn::set_error(TN_ERR_SHAPE, op + ": a q4_0 row is whole 32-element blocks (K % 32 == 0)");
    if (M == 0 || N == 0) return TN_OK;
    if (!codes || !scales || !offsets || !w_blob || !y)
        return tn::set_error(TN_ERR_INVALID, op + ": null device pointer");
    if (codes_row_stride < K || codes_row_stride % 16 != 0 || (reinterpret_cast<uintptr_t>(codes) & 15) != 0)
        return tn::set_error(TN_ERR_INVALID, op + ": planar codes need 16-byte aligned rows");
    if ((reinterpret_cast<uintptr_t>(w_blob) & 1) != 0)
        return tn::set_error(TN_ERR_INVALID, op + ": the q4_0 blob must be at least 2-byte aligned");
    const int64_t nb = K / 32;
    const int chunk = tn::q4_gemv_max_rows(K);
    if (chunk <= 0)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": in_features " + std::to_string(K) +
                                                         " is too large for the decode kernel's shared memory");
    const bool pairs = (flags & TN_EPILOGUE_SILU_MUL_PAIRS) != 0;
    if (pairs && (N % 2 != 0 || y_dtype != TN_BF16))
        return tn::set_error(TN_ERR_INVALID, op + ": the SiLU*up pair epilogue needs an even N and a bf16 output");
    const int64_t ycols = pairs ? N / 2 : N;
    if (link) {
        int st = tn::check_link(op, link, ycols, flags, bias);
        if (st) return st;
        if (M > chunk) return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": a tensor-parallel link needs one launch (M <= " +
                                                                        std::to_string(chunk) + ")");
    }
    if (!link && tn::q4_skinny_applies(w_blob, scales, offsets, M, N, K, flags))  // batched decode: tensor cores
        return tn::launch_q4_skinny(codes, codes_row_stride, scales, offsets, static_cast<const uint8_t *>(w_blob),
                                    bias, y, y_dtype, ycols, (int)M, N, K, flags, stream);
    const size_t ysz = tn_dtype_size(y_dtype);
    for (int64_t m0 = 0; m0 < M; m0 += chunk) {
        const int mc = (int)((M - m0) < chunk ? (M - m0) : chunk);
        int st = tn::launch_q4_gemv_q8(static_cast<const uint8_t *>(w_blob), codes + m0 * codes_row_stride,
                                       scales + m0 * nb, offsets + m0 * nb, codes_row_stride, bias,
                                       static_cast<uint8_t *>(y) + (size_t)m0 * ycols * ysz, y_dtype, ycols, mc, N,
                                       K, flags, stream, link);
        if (st) return st;
    }
    return TN_OK;
}

extern "C" int tn_q4_0_linear_q8(const int8_t *codes, int64_t codes_row_stride, const float *scales,
                                 const float *offsets, const void *w_blob, const float *bias, void *y, int y_dtype,
                                 int64_t M, int64_t N, int64_t K, int flags, void *stream) {
    return tn_q4_0_linear_q8_tp(codes, codes_row_stride, scales, offsets, w_blob, bias, y, y_dtype, M, N, K, flags,
                                nullptr, stream);
}

namespace {

int linear_fused(const std::string &op, int x_mode, const void *x, int64_t x_row_stride, const void *delta,
                 void *h_out, const void *norm_weight, float eps, const void *w_blob, const float *bias, void *y,
                 int y_dtype, int64_t M, int64_t N, int64_t K, int flags, const tn_tp_link *link,
                 const tn::Q8Out *q8, void *stream) {
    __atomic_fetch_add(&tn::counters().q4_linear_calls, 1ull, __ATOMIC_RELAXED);
    if (x_mode != TN_X_BF16 && x_mode != TN_X_RMSNORM && x_mode != TN_X_SILU_MUL)
        return tn::set_error(TN_ERR_INVALID, op + ": unknown x_mode " + std::to_string(x_mode));
    if (y_dtype != TN_F32 && y_dtype != TN_BF16 && y_dtype != TN_F16)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": unsupported output dtype " + tn_dtype_name(y_dtype));
    if (M < 0 || N < 0 || K <= 0 || K % 32 != 0)
        return tn::set_error(TN_ERR_SHAPE, op + ": K must be a positive multiple of 32");
    if (M > 4)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": at most 4 activation rows (quantise separately and call "
                                                          "tn_q4_0_linear_q8 for more)");
    if (M == 0 || N == 0) return TN_OK;
    if (!x || !w_blob || !y || (x_mode == TN_X_RMSNORM && !norm_weight))
        return tn::set_error(TN_ERR_INVALID, op + ": null device pointer");
    if (x_mode == TN_X_RMSNORM && h_out && (h_out == x || h_out == delta))
        return tn::set_error(TN_ERR_INVALID, op + ": h_out must not alias the inputs (every CTA reads them)");
    if (x_row_stride < (x_mode == TN_X_SILU_MUL ? 2 * K : K))
        return tn::set_error(TN_ERR_INVALID, op + ": row stride too small");
    if ((reinterpret_cast<uintptr_t>(w_blob) & 1) != 0)
        return tn::set_error(TN_ERR_INVALID, op + ": the q4_0 blob must be at least 2-byte aligned");
    const uintptr_t a = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(delta) |
                        reinterpret_cast<uintptr_t>(norm_weight) | reinterpret_cast<uintptr_t>(h_out);
    if ((a & 15) != 0 || (x_row_stride * 2) % 16 != 0)
        return tn::set_error(TN_ERR_INVALID, op + ": bf16 rows must be 16-byte aligned");
    const bool pairs = (flags & TN_EPILOGUE_SILU_MUL_PAIRS) != 0;
    if (pairs && (N % 2 != 0 || y_dtype != TN_BF16))
        return tn::set_error(TN_ERR_INVALID, op + ": the SiLU*up pair epilogue needs an even N and a bf16 output");
    if (link) {
        int st = tn::check_link(op, link, pairs ? N / 2 : N, flags, bias);
        if (st) return st;
        if (link->reduce && q8)
            return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": tensor-parallel reduce with a planar Q8_0 output");
    }
    return tn::launch_q4_gemv_fused(x_mode, x, x_row_stride, delta, h_out, norm_weight, eps,
                                    static_cast<const uint8_t *>(w_blob), bias, y, y_dtype, pairs ? N / 2 : N, (int)M,
                                    N, K, flags, tn::stream_of(stream), link, q8);
}

}  // namespace

extern "C" int tn_q4_0_linear_fused_tp(int x_mode, const void *x, int64_t x_row_stride, const void *delta,
                                       void *h_out, const void *norm_weight, float eps, const void *w_blob,
                                       const float *bias, void *y, int y_dtype, int64_t M, int64_t N, int64_t K,
                                       int flags, const tn_tp_link *link, void *stream) {
    return linear_fused("tn_q4_0_linear_fused", x_mode, x, x_row_stride, delta, h_out, norm_weight, eps, w_blob, bias,
                        y, y_dtype, M, N, K, flags, link, nullptr, stream);
}

extern "C" int tn_q4_0_linear_fused_q8out(int x_mode, const void *x, int64_t x_row_stride, const void *delta,
                                          void *h_out, const void *norm_weight, float eps, const void *w_blob,
                                          const float *bias, void *y, int y_dtype, int64_t M, int64_t N, int64_t K,
                                          int flags, int8_t *codes, int64_t codes_row_stride, float *scales,
                                          float *offsets, void *stream) {
    const std::string op = "tn_q4_0_linear_fused_q8out";
    const int64_t cols = (flags & TN_EPILOGUE_SILU_MUL_PAIRS) ? N / 2 : N;
    if (y_dtype != TN_BF16)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": the planar Q8_0 output is quantised from a bf16 y");
    if (N < 0 || cols % 32 != 0)
        return tn::set_error(TN_ERR_SHAPE, op + ": the output's columns must be whole 32-element blocks");
    if (M > 0 && N > 0) {
        if (!codes || !scales || !offsets) return tn::set_error(TN_ERR_INVALID, op + ": null planar Q8_0 output");
        if (codes_row_stride < cols)
            return tn::set_error(TN_ERR_INVALID, op + ": codes row stride smaller than the output's columns");
        if (((reinterpret_cast<uintptr_t>(scales) | reinterpret_cast<uintptr_t>(offsets)) & 3) != 0)
            return tn::set_error(TN_ERR_INVALID, op + ": scales and offsets must be 4-byte aligned");
    }
    const tn::Q8Out q8{codes, codes_row_stride, scales, offsets};
    return linear_fused(op, x_mode, x, x_row_stride, delta, h_out, norm_weight, eps, w_blob, bias, y, y_dtype, M, N,
                        K, flags, nullptr, &q8, stream);
}

extern "C" int tn_q4_0_linear_fused(int x_mode, const void *x, int64_t x_row_stride, const void *delta, void *h_out,
                                    const void *norm_weight, float eps, const void *w_blob, const float *bias,
                                    void *y, int y_dtype, int64_t M, int64_t N, int64_t K, int flags, void *stream) {
    return tn_q4_0_linear_fused_tp(x_mode, x, x_row_stride, delta, h_out, norm_weight, eps, w_blob, bias, y, y_dtype,
                                   M, N, K, flags, nullptr, stream);
}
