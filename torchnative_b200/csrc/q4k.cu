// q4k.cu -- GGML Q4_K weights on the B200 (row f4 of the format family):
// the reader, the Q8_K activation quantiser and the decode GEMV of
// torch._C._quantized_linear for a "q4_k" weight.
//
// BlockQ4K (vendor/candle-core/src/quantized/k_quants.rs:153-159): 144 bytes
// per 256 elements -- f16 d, f16 dmin, 12 bytes of 6-bit sub-block scales and
// mins (get_scale_min_k4, quantized/utils.rs:50-60), 128 bytes of nibbles:
// bytes 32c..32c+31 hold sub-block 2c in their low nibbles and 2c+1 in their
// high nibbles. Its dot product runs against Q8_K activations (BlockQ8K,
// :185-190: f32 d, 256 int8 codes, sums of 16 codes), BlockQ4K::vec_dot_unopt
// (:1478-1544): per super-block d_w*d_x * sum_s sc_s * (q4 . q8)_s
// - dmin_w*d_x * sum_s m_s * (sum of sub-block s's codes), exact integers
// between the scale products.
//
// The GEMV is the staged decode GEMV of q4_gemv.cu with the Q4_K weight
// format: a lane takes one 64-element sub-block pair (the super-block's
// 16-byte header and 32 nibble bytes) against the staged Q8_K codes, with the
// super-block's d and each 32-element block's code sum in the planar scale and
// offset slots.
#include "q4_kernels.cuh"

namespace tn {
namespace {

constexpr int QK = 256, QKB = 144;

__device__ __forceinline__ void scale_min(int j, const uint8_t *q, int &sc, int &m) {
    if (j < 4) {
        sc = q[j] & 63;
        m = q[j + 4] & 63;
    } else {
        sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// BlockQ4K::to_float (k_quants.rs:1722-1748): thread = (super-block, sub-block
// pair c), 64 outputs; each product rounded, then the subtraction (no FMA).
__global__ void q4k_dequantize_kernel(const uint8_t *__restrict__ blob, float *__restrict__ out, int64_t nsb) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= nsb * 4) return;
    const int64_t sb = i >> 2;
    const int c = (int)(i & 3);
    const uint8_t *blk = blob + sb * QKB;
    const float d = half_bits_to_f32((uint32_t)blk[0] | ((uint32_t)blk[1] << 8));
    const float mn = half_bits_to_f32((uint32_t)blk[2] | ((uint32_t)blk[3] << 8));
    int s0, m0, s1, m1;
    scale_min(2 * c, blk + 4, s0, m0);
    scale_min(2 * c + 1, blk + 4, s1, m1);
    const float d1 = __fmul_rn(d, (float)s0), mm1 = __fmul_rn(mn, (float)m0);
    const float d2 = __fmul_rn(d, (float)s1), mm2 = __fmul_rn(mn, (float)m1);
    const uint8_t *qs = blk + 16 + 32 * c;
    float *o = out + sb * QK + 64 * c;
#pragma unroll 8
    for (int l = 0; l < 32; ++l) {
        const int q = qs[l];
        o[l] = __fsub_rn(__fmul_rn(d1, (float)(q & 0xF)), mm1);
        o[32 + l] = __fsub_rn(__fmul_rn(d2, (float)(q >> 4)), mm2);
    }
}

__device__ __forceinline__ int sat_i8_nan0(float v) {
    if (!(v == v)) return 0;
    if (v <= -128.0f) return -128;
    if (v >= 127.0f) return 127;
    return __float2int_rz(v);
}

// BlockQ8K::from_float (k_quants.rs:2376-2410) for one 256-element super-block
// per warp (lane = 8 consecutive elements): the signed value of largest
// magnitude (the first one on ties), iscale = -127 / max, codes
// clamp(round(iscale * x)), d = 1 / iscale; an all-zero block is d = 0 with
// zero codes. Written in the planar layout the staged GEMV reads: codes
// [rows][K], and per 32-element block [rows][K/32] the super-block's d and the
// block's code sum (the reference's two 16-element sums added) as a float.
template <typename T>
__global__ void __launch_bounds__(32) q8k_quantize_planar_kernel(const void *__restrict__ x, int64_t x_row_stride,
                                                                 int8_t *__restrict__ codes, int64_t codes_row_stride,
                                                                 float *__restrict__ xd, float *__restrict__ xs32,
                                                                 int nsb) {
    pdl_launch_dependents();
    pdl_wait();
    const int sb = blockIdx.x, r = blockIdx.y, lane = threadIdx.x;
    const T *src = static_cast<const T *>(x) + (int64_t)r * x_row_stride + (int64_t)sb * QK + lane * 8;
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = to_f32<T>(src[e]);
    float ba = 0.0f, bv = 0.0f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int e = 0; e < 8; ++e)
        if (ba < fabsf(v[e])) {
            ba = fabsf(v[e]);
            bv = v[e];
            bi = lane * 8 + e;
        }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, ba, off), ov = __shfl_xor_sync(0xffffffffu, bv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (oa > ba || (oa == ba && oi < bi)) {
            ba = oa;
            bv = ov;
            bi = oi;
        }
    }
    int q[8];
    float d = 0.0f;
    if (ba == 0.0f) {
#pragma unroll
        for (int e = 0; e < 8; ++e) q[e] = 0;
    } else {
        const float iscale = __fdiv_rn(-127.0f, bv);
#pragma unroll
        for (int e = 0; e < 8; ++e) q[e] = sat_i8_nan0(roundf(__fmul_rn(iscale, v[e])));
        d = __fdiv_rn(1.0f, iscale);
    }
    const uint32_t lo = __byte_perm(__byte_perm((uint32_t)q[0], (uint32_t)q[1], 0x0040),
                                    __byte_perm((uint32_t)q[2], (uint32_t)q[3], 0x0040), 0x5410);
    const uint32_t hi = __byte_perm(__byte_perm((uint32_t)q[4], (uint32_t)q[5], 0x0040),
                                    __byte_perm((uint32_t)q[6], (uint32_t)q[7], 0x0040), 0x5410);
    *reinterpret_cast<uint2 *>(codes + (int64_t)r * codes_row_stride + (int64_t)sb * QK + lane * 8) = make_uint2(lo, hi);
    int s = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) s += q[e];
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if ((lane & 3) == 0) {
        const int64_t b = (int64_t)r * nsb * 8 + sb * 8 + (lane >> 2);
        xs32[b] = (float)s;
        xd[b] = d;
    }
}

}  // namespace
}  // namespace tn

extern "C" int tn_q4_k_dequantize(const void *blob, float *out, int64_t rows, int64_t cols, void *stream) {
    const std::string op = "torch._C._dequantize";
    if (rows < 0 || cols < 0) return tn::set_error(TN_ERR_SHAPE, op + ": negative size");
    if (cols % 256 != 0)
        return tn::set_error(TN_ERR_SHAPE, op + ": q4_k rows are whole 256-element super-blocks, got " +
                                               std::to_string(cols) + " columns");
    const int64_t nsb = rows * (cols / 256);
    if (nsb == 0) return TN_OK;
    if (!blob || !out) return tn::set_error(TN_ERR_INVALID, op + ": null pointer");
    const int threads = 128;
    tn::q4k_dequantize_kernel<<<(unsigned)((nsb * 4 + threads - 1) / threads), threads, 0, tn::stream_of(stream)>>>(
        static_cast<const uint8_t *>(blob), out, nsb);
    __atomic_fetch_add(&tn::counters().q4_codec_launches, 1ull, __ATOMIC_RELAXED);
    return tn::check_launch(op.c_str());
}

extern "C" int tn_q4_k_linear(const void *x, int x_dtype, int64_t x_row_stride, const void *w_blob, const float *bias,
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
    if (K % 256 != 0)
        return tn::set_error(TN_ERR_SHAPE, op + ": mat1 and mat2 shapes cannot be multiplied ([" + std::to_string(M) +
                                               ", " + std::to_string(K) + "] and " + std::to_string(K) + "x" +
                                               std::to_string(N) + "): a q4_k row is whole 256-element super-blocks");
    if (M == 0 || N == 0) return TN_OK;
    if (K == 0) return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": in_features == 0 is not implemented");
    if (!x || !w_blob || !y) return tn::set_error(TN_ERR_INVALID, op + ": null device pointer");
    if (x_row_stride < K) return tn::set_error(TN_ERR_INVALID, op + ": activation row stride smaller than in_features");
    if ((reinterpret_cast<uintptr_t>(w_blob) & 15) != 0)
        return tn::set_error(TN_ERR_INVALID, op + ": the q4_k blob must be 16-byte aligned (144-byte super-blocks "
                                                  "are read 16 bytes at a time)");
    if (act_mode == TN_ACT_FLOAT)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED,
                             op + ": the float-activation mode is not implemented on CUDA yet; use the Q8_K mode "
                                  "(the reference's arithmetic)");
    const int nsb = (int)(K / 256);
    const int chunk = tn::q4_gemv_max_rows(K, 2);
    if (chunk <= 0)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": in_features " + std::to_string(K) +
                                                         " is too large for the decode kernel's shared memory");
    // Workspace: Q8_K codes [M][K], per 32-block d [M][K/32] and code sums [M][K/32].
    const int64_t nb = K / 32;
    const size_t codes = ((size_t)M * K + 255) & ~size_t(255), scal = ((size_t)M * nb * 4 + 255) & ~size_t(255);
    void *ws = nullptr;
    int st = tn::workspace(&ws, codes + 2 * scal + 256, stream, /*slot=*/0);
    if (st) return st;
    int8_t *xq = static_cast<int8_t *>(ws);
    float *xd = reinterpret_cast<float *>(static_cast<uint8_t *>(ws) + codes);
    float *xs32 = reinterpret_cast<float *>(static_cast<uint8_t *>(ws) + codes + scal);
    {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)nsb, (unsigned)M);
        cfg.blockDim = dim3(32);
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cudaError_t e;
        if (x_dtype == TN_F32)
            e = cudaLaunchKernelEx(&cfg, tn::q8k_quantize_planar_kernel<float>, x, x_row_stride, xq, K, xd, xs32, nsb);
        else if (x_dtype == TN_BF16)
            e = cudaLaunchKernelEx(&cfg, tn::q8k_quantize_planar_kernel<__nv_bfloat16>, x, x_row_stride, xq, K, xd, xs32,
                                   nsb);
        else
            e = cudaLaunchKernelEx(&cfg, tn::q8k_quantize_planar_kernel<__half>, x, x_row_stride, xq, K, xd, xs32, nsb);
        st = tn::check_cuda(e, op.c_str(), "cudaLaunchKernelEx (q8_k activations)");
        if (st) return st;
        __atomic_fetch_add(&tn::counters().q8_quant_launches, 1ull, __ATOMIC_RELAXED);
    }
    const size_t ysz = tn_dtype_size(y_dtype);
    for (int64_t m0 = 0; m0 < M; m0 += chunk) {
        const int mc = (int)((M - m0) < chunk ? (M - m0) : chunk);
        st = tn::launch_q4k_gemv(static_cast<const uint8_t *>(w_blob), xq + m0 * K, xd + m0 * nb, xs32 + m0 * nb, K,
                                 bias, static_cast<uint8_t *>(y) + (size_t)m0 * N * ysz, y_dtype, N, mc, N, K, stream);
        if (st) return st;
    }
    return TN_OK;
}
