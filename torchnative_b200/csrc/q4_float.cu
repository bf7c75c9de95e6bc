// q4_float.cu -- the float-activation mode of the Q4_0 linear (TN_ACT_FLOAT)
// for decode-sized inputs (M <= 16 rows).
//
// Arithmetic: every weight is dequantised exactly to f32, w = (code - 8) * d
// (an integer of at most 4 bits times an f16 value: exact in f32), and
// y[m, n] = sum over k of x[m, k] * w[n, k] in f32, plus the f32 bias. No
// activation quantisation: x is widened exactly from its dtype. The sum is
// formed block by block -- s = sum over the 32 elements of x * (code - 8),
// then acc += s * d -- in a fixed order per output (each lane's blocks in
// order, then a butterfly over the warp), so the result is deterministic and
// every term passes through at most 32 + ceil(K / 1024) + 6 roundings: within
// gamma_(38 + ceil(K / 1024)) * sum |x * w| of the exact value.
//
// One warp per weight row (grid-stride over rows); lane l takes blocks l,
// l + 32, ... of the row; the block's 18 bytes are read as nine 16-bit loads
// (rows are 2-byte aligned), x through the read-only cache (every warp reads
// the same few KB of activations). Bound by the dequantise-and-FMA work at a
// few instructions per weight, not by HBM; it is the exactness mode, not the
// fast one.
#include "q4_kernels.cuh"

namespace tn {
namespace {

constexpr int kFloatThreads = 256;

template <typename T>
__device__ __forceinline__ float ldx(const T *p) {
    return to_f32<T>(__ldg(p));
}

template <typename T, int MT>
__global__ void __launch_bounds__(kFloatThreads) q4_float_gemv_kernel(const uint8_t *w, const T *x,
                                                                      int64_t x_row_stride, const float *bias,
                                                                      void *y, int y_dtype, int64_t y_row_stride,
                                                                      int M, int64_t N, int nb) {
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (kFloatThreads / 32);
    const int64_t rowbytes = (int64_t)nb * 18;
    for (int64_t n = blockIdx.x * (int64_t)(kFloatThreads / 32) + (threadIdx.x >> 5); n < N; n += warps) {
        float acc[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[m] = 0.0f;
        const uint8_t *row = w + n * rowbytes;
        for (int b = lane; b < nb; b += 32) {
            const unsigned short *h = reinterpret_cast<const unsigned short *>(row + (int64_t)b * 18);
            uint32_t u[9];
#pragma unroll
            for (int i = 0; i < 9; ++i) u[i] = __ldg(h + i);
            const float d = half_bits_to_f32(u[0]);
            // codes - 8 as exact f32: byte j holds element j (low nibble) and
            // element j + 16 (high nibble)
            float c[32];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint32_t two = u[1 + i];  // bytes 2i and 2i + 1
#pragma unroll
                for (int k = 0; k < 2; ++k) {
                    const uint32_t byte = (two >> (8 * k)) & 0xffu;
                    c[2 * i + k] = (float)(int)(byte & 0xfu) - 8.0f;
                    c[16 + 2 * i + k] = (float)(int)(byte >> 4) - 8.0f;
                }
            }
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                if (m >= M) break;
                const T *xr = x + m * x_row_stride + (int64_t)b * 32;
                float s = 0.0f;
#pragma unroll
                for (int j = 0; j < 32; ++j) s = fmaf(ldx(xr + j), c[j], s);
                acc[m] = fmaf(s, d, acc[m]);
            }
        }
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            if (m >= M) break;
            float v = acc[m];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            if (lane == 0) store_out(y, y_dtype, m * y_row_stride + n, bias ? v + __ldg(bias + n) : v);
        }
    }
}

template <typename T, int MT>
int launch_typed(const uint8_t *w, const void *x, int64_t x_row_stride, const float *bias, void *y, int y_dtype,
                 int64_t y_row_stride, int M, int64_t N, int64_t K, int grid, cudaStream_t stream) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kFloatThreads);
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return check_cuda(cudaLaunchKernelEx(&cfg, q4_float_gemv_kernel<T, MT>, w, static_cast<const T *>(x),
                                         x_row_stride, bias, y, y_dtype, y_row_stride, M, N, (int)(K / 32)),
                      "torch._C._quantized_linear", "cudaLaunchKernelEx (float mode)");
}

template <typename T>
int launch_rows(const uint8_t *w, const void *x, int64_t x_row_stride, const float *bias, void *y, int y_dtype,
                int64_t y_row_stride, int M, int64_t N, int64_t K, int grid, cudaStream_t stream) {
    if (M <= 1) return launch_typed<T, 1>(w, x, x_row_stride, bias, y, y_dtype, y_row_stride, M, N, K, grid, stream);
    if (M <= 4) return launch_typed<T, 4>(w, x, x_row_stride, bias, y, y_dtype, y_row_stride, M, N, K, grid, stream);
    return launch_typed<T, 16>(w, x, x_row_stride, bias, y, y_dtype, y_row_stride, M, N, K, grid, stream);
}

}  // namespace

int launch_q4_float_gemv(const uint8_t *w, const void *x, int x_dtype, int64_t x_row_stride, const float *bias,
                         void *y, int y_dtype, int64_t y_row_stride, int M, int64_t N, int64_t K,
                         cudaStream_t stream) {
    DeviceFacts f{};
    int st = device_facts(&f);
    if (st) return st;
    const int64_t warps_needed = N, per_cta = kFloatThreads / 32;
    int64_t grid = (int64_t)f.sm_count * 8;
    if ((warps_needed + per_cta - 1) / per_cta < grid) grid = (warps_needed + per_cta - 1) / per_cta;
    if (grid < 1) grid = 1;
    switch (x_dtype) {
    case TN_F32:
        st = launch_rows<float>(w, x, x_row_stride, bias, y, y_dtype, y_row_stride, M, N, K, (int)grid, stream);
        break;
    case TN_BF16:
        st = launch_rows<__nv_bfloat16>(w, x, x_row_stride, bias, y, y_dtype, y_row_stride, M, N, K, (int)grid,
                                        stream);
        break;
    default:
        st = launch_rows<__half>(w, x, x_row_stride, bias, y, y_dtype, y_row_stride, M, N, K, (int)grid, stream);
    }
    if (st) return st;
    __atomic_fetch_add(&counters().q4_gemv_generic, 1ull, __ATOMIC_RELAXED);
    return TN_OK;
}

}  // namespace tn
