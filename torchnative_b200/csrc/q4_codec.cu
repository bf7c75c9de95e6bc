// q4_codec.cu -- GGML Q4_0 / Q8_0 block codecs on the device, byte- and
// bit-identical to candle's CPU codecs (k_quants.rs), plus the planar Q8_0
// activation layout the linear kernels read.
//
// Every float operation below is an explicitly rounded intrinsic (__fdiv_rn,
// __fmul_rn, __fadd_rn) so that no contraction or approximate division can
// change a byte relative to the reference's IEEE f32 arithmetic.
#include "q4_kernels.cuh"

namespace tn {

namespace {

// Rust `v as u8`: truncate toward zero, saturate at 0 and 255, NaN -> 0.
__device__ __forceinline__ uint32_t sat_u8_trunc(float v) {
    if (!(v == v) || v <= 0.0f) return 0u;
    if (v >= 255.0f) return 255u;
    return static_cast<uint32_t>(__float2uint_rz(v));
}

// Rust `v as i8` after f32::round: saturate at -128 and 127, NaN -> 0.
__device__ __forceinline__ int sat_i8(float v) {
    if (!(v == v)) return 0;
    if (v <= -128.0f) return -128;
    if (v >= 127.0f) return 127;
    return __float2int_rz(v);
}

template <typename T>
__device__ __forceinline__ float load_x(const void *x, int64_t i) {
    return to_f32<T>(static_cast<const T *>(x)[i]);
}

// BlockQ4_0::from_float, k_quants.rs:241-277. One thread per 32-element block.
__global__ void q4_0_quantize_kernel(const float *__restrict__ x, uint8_t *__restrict__ blob, int64_t nblocks) {
    int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= nblocks) return;
    const float *xs = x + i * 32;
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = xs[j];
    float amax = 0.0f, mx = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        float a = fabsf(v[j]);
        if (amax < a) {
            amax = a;
            mx = v[j];
        }
    }
    float d = __fdiv_rn(mx, -8.0f);
    float id = (d != 0.0f) ? __fdiv_rn(1.0f, d) : 0.0f;
    // Stored as nine little-endian 16-bit halves: blocks are 18 bytes, so
    // every block starts on a 2-byte boundary.
    unsigned short *out = reinterpret_cast<unsigned short *>(blob + i * 18);
    out[0] = __half_as_ushort(__float2half_rn(d));
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
        uint32_t a0 = sat_u8_trunc(__fadd_rn(__fmul_rn(v[j], id), 8.5f));
        uint32_t a1 = sat_u8_trunc(__fadd_rn(__fmul_rn(v[16 + j], id), 8.5f));
        uint32_t b0 = sat_u8_trunc(__fadd_rn(__fmul_rn(v[j + 1], id), 8.5f));
        uint32_t b1 = sat_u8_trunc(__fadd_rn(__fmul_rn(v[16 + j + 1], id), 8.5f));
        a0 = a0 < 15u ? a0 : 15u;
        a1 = a1 < 15u ? a1 : 15u;
        b0 = b0 < 15u ? b0 : 15u;
        b1 = b1 < 15u ? b1 : 15u;
        out[1 + j / 2] = static_cast<unsigned short>((a0 | (a1 << 4)) | ((b0 | (b1 << 4)) << 8));
    }
}

// BlockQ4_0::to_float, k_quants.rs:219-239: (code - 8) as f32 * f32(d), exact.
__global__ void q4_0_dequantize_kernel(const uint8_t *__restrict__ blob, float *__restrict__ out, int64_t nblocks) {
    int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= nblocks) return;
    const uint8_t *b = blob + i * 18;
    float d = half_bits_to_f32((uint32_t)b[0] | ((uint32_t)b[1] << 8));
    float *o = out + i * 32;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        int q = b[2 + j];
        o[j] = __fmul_rn(static_cast<float>((q & 15) - 8), d);
        o[16 + j] = __fmul_rn(static_cast<float>((q >> 4) - 8), d);
    }
}

// BlockQ8_0::to_float, k_quants.rs:658-674: code * f32(d), exact in f32
// (an 8-bit integer times an 11-bit significand).
__global__ void q8_0_dequantize_kernel(const uint8_t *__restrict__ blob, float *__restrict__ out, int64_t nblocks) {
    int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= nblocks) return;
    const uint8_t *b = blob + i * 34;
    const float d = half_bits_to_f32((uint32_t)b[0] | ((uint32_t)b[1] << 8));
    float *o = out + i * 32;
#pragma unroll
    for (int j = 0; j < 32; ++j) o[j] = __fmul_rn(static_cast<float>(static_cast<int8_t>(b[2 + j])), d);
}

// BlockQ8_0::from_float, k_quants.rs:676-706, for one 32-element block of row
// `r`, block `b`. Returns the f16 scale bits and writes the 32 codes.
template <typename T>
__device__ __forceinline__ uint32_t q8_0_block(const void *x, int64_t base, int8_t *codes, int *sum) {
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = load_x<T>(x, base + j);
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(v[j]));
    float d = __fdiv_rn(amax, 127.0f);
    float id = (d != 0.0f) ? __fdiv_rn(1.0f, d) : 0.0f;
    int s = 0;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        int q = sat_i8(roundf(__fmul_rn(v[j], id)));
        codes[j] = static_cast<int8_t>(q);
        s += q;
    }
    *sum = s;
    return __half_as_ushort(__float2half_rn(d));
}

template <typename T>
__global__ void q8_0_quantize_blob_kernel(const void *__restrict__ x, int64_t row_stride, uint8_t *__restrict__ blob,
                                          int64_t rows, int64_t nb) {
    int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= rows * nb) return;
    int64_t r = i / nb, b = i % nb;
    int8_t codes[32];
    int sum;
    uint32_t db = q8_0_block<T>(x, r * row_stride + b * 32, codes, &sum);
    // Seventeen little-endian 16-bit halves (34-byte blocks start on 2-byte boundaries).
    unsigned short *out = reinterpret_cast<unsigned short *>(blob + i * 34);
    out[0] = static_cast<unsigned short>(db);
#pragma unroll
    for (int j = 0; j < 32; j += 2)
        out[1 + j / 2] = static_cast<unsigned short>((uint32_t)(uint8_t)codes[j] |
                                                     ((uint32_t)(uint8_t)codes[j + 1] << 8));
}

// Planar Q8_0: the same blocks, split into codes [rows][K] int8, the widened
// scale xd[rows][nb] = f32(f16 d), and xc[rows][nb] = 12582912 + 8 * sum(codes),
// the offset the GEMV subtracts after its magic-number int -> float step.
template <typename T>
__global__ void q8_0_quantize_planar_kernel(const void *__restrict__ x, int64_t row_stride, int8_t *__restrict__ xq,
                                            float *__restrict__ xd, float *__restrict__ xc, int64_t rows, int64_t nb,
                                            int64_t xq_row_stride) {
    // Launched as a programmatic dependent: let the consumer GEMV start its
    // weight prefetch now, and wait for whatever produced x.
    pdl_launch_dependents();
    pdl_wait();
    int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= rows * nb) return;
    int64_t r = i / nb, b = i % nb;
    __align__(16) int8_t codes[32];
    int sum;
    uint32_t db = q8_0_block<T>(x, r * row_stride + b * 32, codes, &sum);
    int4 *dst = reinterpret_cast<int4 *>(xq + r * xq_row_stride + b * 32);
    dst[0] = reinterpret_cast<const int4 *>(codes)[0];
    dst[1] = reinterpret_cast<const int4 *>(codes)[1];
    xd[r * nb + b] = half_bits_to_f32(db);
    xc[r * nb + b] = 12582912.0f + 8.0f * static_cast<float>(sum);
}

// Planar Q8_0 for the tensor-core GEMM: the codes written as f16 (exact:
// |code| <= 127) so they are an MMA operand as they stand, and the widened
// scale xd[rows][nb] = f32(f16 d). Within each 32-block the codes are stored
// in the order the GEMM's weight unpacking produces (a block's sum does not
// depend on the order of its terms, all of them exact integers): 16-byte chunk
// c holds elements 4c + {0, 2, 16, 18, 1, 3, 17, 19}.
template <typename T>
__global__ void q8_0_quantize_planar_f16_kernel(const void *__restrict__ x, int64_t row_stride,
                                                __half *__restrict__ xq, float *__restrict__ xd, int64_t rows,
                                                int64_t nb, int64_t xq_row_stride) {
    pdl_launch_dependents();
    pdl_wait();
    int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= rows * nb) return;
    int64_t r = i / nb, b = i % nb;
    int8_t codes[32];
    int sum;
    uint32_t db = q8_0_block<T>(x, r * row_stride + b * 32, codes, &sum);
    uint4 *dst = reinterpret_cast<uint4 *>(xq + r * xq_row_stride + b * 32);
    constexpr int kPairLo[4] = {0, 16, 1, 17};  // pair e of chunk c: elements 4c + kPairLo[e] and + 2
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int i0 = 4 * c + kPairLo[e];
            const __half2 h = __halves2half2(__int2half_rn(codes[i0]), __int2half_rn(codes[i0 + 2]));
            w[e] = *reinterpret_cast<const uint32_t *>(&h);
        }
        dst[c] = make_uint4(w[0], w[1], w[2], w[3]);
    }
    xd[r * nb + b] = half_bits_to_f32(db);
}

int check_dtype_in(const char *op, int dtype) {
    if (dtype == TN_F32 || dtype == TN_BF16 || dtype == TN_F16) return TN_OK;
    return set_error(TN_ERR_NOT_IMPLEMENTED,
                     std::string(op) + ": activations must be torch.float32, torch.bfloat16 or torch.float16, got " +
                         tn_dtype_name(dtype));
}

}  // namespace

int launch_q8_planar(const void *x, int x_dtype, int64_t row_stride, int8_t *xq, float *xd, float *xc, int64_t rows,
                     int64_t nb, int64_t xq_row_stride, cudaStream_t stream) {
    int64_t n = rows * nb;
    if (n == 0) return TN_OK;
    int threads = 128;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((n + threads - 1) / threads));
    cfg.blockDim = dim3(threads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    switch (x_dtype) {
    case TN_F32:
        e = cudaLaunchKernelEx(&cfg, q8_0_quantize_planar_kernel<float>, x, row_stride, xq, xd, xc, rows, nb,
                               xq_row_stride);
        break;
    case TN_BF16:
        e = cudaLaunchKernelEx(&cfg, q8_0_quantize_planar_kernel<__nv_bfloat16>, x, row_stride, xq, xd, xc, rows, nb,
                               xq_row_stride);
        break;
    default:
        e = cudaLaunchKernelEx(&cfg, q8_0_quantize_planar_kernel<__half>, x, row_stride, xq, xd, xc, rows, nb,
                               xq_row_stride);
        break;
    }
    int st = check_cuda(e, "torch._C._quantized_linear (activation Q8_0)", "cudaLaunchKernelEx");
    if (st) return st;
    __atomic_fetch_add(&counters().q8_quant_launches, 1ull, __ATOMIC_RELAXED);
    return check_launch("torch._C._quantized_linear (activation Q8_0)");
}

int launch_q8_planar_f16(const void *x, int x_dtype, int64_t row_stride, __half *xq, float *xd, int64_t rows,
                         int64_t nb, int64_t xq_row_stride, cudaStream_t stream) {
    int64_t n = rows * nb;
    if (n == 0) return TN_OK;
    int threads = 128;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((n + threads - 1) / threads));
    cfg.blockDim = dim3(threads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    switch (x_dtype) {
    case TN_F32:
        e = cudaLaunchKernelEx(&cfg, q8_0_quantize_planar_f16_kernel<float>, x, row_stride, xq, xd, rows, nb,
                               xq_row_stride);
        break;
    case TN_BF16:
        e = cudaLaunchKernelEx(&cfg, q8_0_quantize_planar_f16_kernel<__nv_bfloat16>, x, row_stride, xq, xd, rows, nb,
                               xq_row_stride);
        break;
    default:
        e = cudaLaunchKernelEx(&cfg, q8_0_quantize_planar_f16_kernel<__half>, x, row_stride, xq, xd, rows, nb,
                               xq_row_stride);
        break;
    }
    int st = check_cuda(e, "torch._C._quantized_linear (activation Q8_0, f16 codes)", "cudaLaunchKernelEx");
    if (st) return st;
    __atomic_fetch_add(&counters().q8_quant_launches, 1ull, __ATOMIC_RELAXED);
    return TN_OK;
}

}  // namespace tn

extern "C" {

int tn_q4_0_quantize(const float *x, void *blob, int64_t rows, int64_t cols, void *stream) {
    const char *op = "torch._C._quantize";
    if (rows < 0 || cols < 0) return tn::set_error(TN_ERR_SHAPE, std::string(op) + ": negative size");
    if (cols % 32 != 0)
        return tn::set_error(TN_ERR_SHAPE, std::string(op) + ": q4_0 needs the last dimension to be a multiple of 32, got " +
                                               std::to_string(cols));
    int64_t nb = rows * (cols / 32);
    if (nb == 0) return TN_OK;
    if (!x || !blob) return tn::set_error(TN_ERR_INVALID, std::string(op) + ": null pointer");
    int threads = 128;
    tn::q4_0_quantize_kernel<<<(unsigned)((nb + threads - 1) / threads), threads, 0, tn::stream_of(stream)>>>(
        x, static_cast<uint8_t *>(blob), nb);
    __atomic_fetch_add(&tn::counters().q4_codec_launches, 1ull, __ATOMIC_RELAXED);
    return tn::check_launch(op);
}

int tn_q4_0_dequantize(const void *blob, float *out, int64_t rows, int64_t cols, void *stream) {
    const char *op = "torch._C._dequantize";
    if (rows < 0 || cols < 0) return tn::set_error(TN_ERR_SHAPE, std::string(op) + ": negative size");
    if (cols % 32 != 0)
        return tn::set_error(TN_ERR_SHAPE, std::string(op) + ": q4_0 rows are whole 32-element blocks, got " +
                                               std::to_string(cols) + " columns");
    int64_t nb = rows * (cols / 32);
    if (nb == 0) return TN_OK;
    if (!blob || !out) return tn::set_error(TN_ERR_INVALID, std::string(op) + ": null pointer");
    int threads = 128;
    tn::q4_0_dequantize_kernel<<<(unsigned)((nb + threads - 1) / threads), threads, 0, tn::stream_of(stream)>>>(
        static_cast<const uint8_t *>(blob), out, nb);
    __atomic_fetch_add(&tn::counters().q4_codec_launches, 1ull, __ATOMIC_RELAXED);
    return tn::check_launch(op);
}

int tn_q8_0_dequantize(const void *blob, float *out, int64_t rows, int64_t cols, void *stream) {
    const char *op = "torch._C._dequantize";
    if (rows < 0 || cols < 0) return tn::set_error(TN_ERR_SHAPE, std::string(op) + ": negative size");
    if (cols % 32 != 0)
        return tn::set_error(TN_ERR_SHAPE, std::string(op) + ": q8_0 rows are whole 32-element blocks, got " +
                                               std::to_string(cols) + " columns");
    int64_t nb = rows * (cols / 32);
    if (nb == 0) return TN_OK;
    if (!blob || !out) return tn::set_error(TN_ERR_INVALID, std::string(op) + ": null pointer");
    int threads = 128;
    tn::q8_0_dequantize_kernel<<<(unsigned)((nb + threads - 1) / threads), threads, 0, tn::stream_of(stream)>>>(
        static_cast<const uint8_t *>(blob), out, nb);
    __atomic_fetch_add(&tn::counters().q4_codec_launches, 1ull, __ATOMIC_RELAXED);
    return tn::check_launch(op);
}

int tn_q8_0_quantize(const void *x, int x_dtype, int64_t x_row_stride, void *blob, int64_t rows, int64_t cols,
                     void *stream) {
    const char *op = "torch._C._quantize";
    int st = tn::check_dtype_in(op, x_dtype);
    if (st) return st;
    if (rows < 0 || cols < 0 || x_row_stride < cols)
        return tn::set_error(TN_ERR_SHAPE, std::string(op) + ": bad shape or row stride");
    if (cols % 32 != 0)
        return tn::set_error(TN_ERR_SHAPE, std::string(op) + ": q8_0 needs the last dimension to be a multiple of 32, got " +
                                               std::to_string(cols));
    int64_t nb = cols / 32, n = rows * nb;
    if (n == 0) return TN_OK;
    if (!x || !blob) return tn::set_error(TN_ERR_INVALID, std::string(op) + ": null pointer");
    int threads = 128;
    unsigned grid = (unsigned)((n + threads - 1) / threads);
    cudaStream_t s = tn::stream_of(stream);
    uint8_t *b = static_cast<uint8_t *>(blob);
    if (x_dtype == TN_F32)
        tn::q8_0_quantize_blob_kernel<float><<<grid, threads, 0, s>>>(x, x_row_stride, b, rows, nb);
    else if (x_dtype == TN_BF16)
        tn::q8_0_quantize_blob_kernel<__nv_bfloat16><<<grid, threads, 0, s>>>(x, x_row_stride, b, rows, nb);
    else
        tn::q8_0_quantize_blob_kernel<__half><<<grid, threads, 0, s>>>(x, x_row_stride, b, rows, nb);
    __atomic_fetch_add(&tn::counters().q8_quant_launches, 1ull, __ATOMIC_RELAXED);
    return tn::check_launch(op);
}

}  // extern "C"
