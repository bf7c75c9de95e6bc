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
// The GEMV: 8 warps per CTA, each warp two weight rows at a time; a lane pair
// owns one super-block of the row (lane 2p+1 the upper four sub-blocks) and
// reads its 16-byte scale chunk and its 64 bytes of nibbles with 16-byte loads
// (a warp covers 16 consecutive super-blocks, 2304 contiguous bytes per row);
// the activation codes of the launch's rows sit in shared memory with their
// 16-byte chunks XOR-swizzled so a quarter-warp's loads hit distinct bank
// groups. Sub-block sums are dp4a chains, kept as integers per lane (at most
// 4 * 63 * 32 * 15 * 128 < 2^24, exact in f32) until one FMA per scale product.
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
// zero codes. Planar output: codes [rows][K], d [rows][K/256] and, per
// 32-element sub-block, the sum of its codes [rows][K/32] (the reference's
// two 16-element sums added).
template <typename T>
__global__ void __launch_bounds__(32) q8k_quantize_planar_kernel(const void *__restrict__ x, int64_t x_row_stride,
                                                                 int8_t *__restrict__ codes, int64_t codes_row_stride,
                                                                 float *__restrict__ xd, int *__restrict__ xs32,
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
    if ((lane & 3) == 0) xs32[(int64_t)r * nsb * 8 + sb * 8 + (lane >> 2)] = s;
    if (lane == 0) xd[(int64_t)r * nsb + sb] = d;
}

// Physical 16-byte chunk of logical chunk c (0..15) of super-block sb in a
// staged activation row: XOR by (2 sb + c/8) & 7, so the eight lanes of a
// quarter-warp (super-blocks p..p+3, both halves) read eight bank groups.
__device__ __forceinline__ uint32_t xchunk_k(int sb, int c) {
    return (uint32_t)(sb * QK + 16 * (c ^ ((2 * sb + (c >> 3)) & 7)));
}

struct Q4kArgs {
    const uint8_t *w;
    const int8_t *xq;
    const float *xd;
    const int *xs32;
    const float *bias;
    void *y;
    int y_dtype, M, nsb;
    int64_t N, xq_row_stride, y_row_stride;
};

__device__ __forceinline__ uint4 ldg_na(const uint8_t *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

template <int MT>
__global__ void __launch_bounds__(256, (MT <= 1) ? 2 : 1) q4k_gemv_kernel(const Q4kArgs a) {
    extern __shared__ __align__(16) uint8_t sm[];
    const int K = a.nsb * QK;
    uint8_t *xs = sm;                                                  // [M][K] codes, swizzled
    float *xd = reinterpret_cast<float *>(sm + (size_t)a.M * K);       // [M][nsb]
    int *x32 = reinterpret_cast<int *>(xd + (size_t)a.M * a.nsb);      // [M][nsb * 8]
    pdl_launch_dependents();
    pdl_wait();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int g = tid; g < a.M * K / 16; g += blockDim.x) {
        const int m = g / (K / 16), c16 = g % (K / 16);
        const uint4 v = *reinterpret_cast<const uint4 *>(a.xq + (int64_t)m * a.xq_row_stride + 16 * c16);
        *reinterpret_cast<uint4 *>(xs + (size_t)m * K + xchunk_k(c16 >> 4, c16 & 15)) = v;
    }
    for (int i = tid; i < a.M * a.nsb; i += blockDim.x) xd[i] = a.xd[i];
    for (int i = tid; i < a.M * a.nsb * 8; i += blockDim.x) x32[i] = a.xs32[i];
    __syncthreads();

    const int h = lane & 1, p = lane >> 1;
    const int64_t rowbytes = (int64_t)a.nsb * QKB;
    const int64_t pairs = (a.N + 1) / 2;
    for (int64_t rp = (int64_t)blockIdx.x * 8 + warp; rp < pairs; rp += (int64_t)gridDim.x * 8) {
        const int64_t r0 = 2 * rp;
        const bool has_b = r0 + 1 < a.N;
        float acc[2][MT];
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int m = 0; m < MT; ++m) acc[r][m] = 0.0f;
        for (int sb = p; sb < a.nsb; sb += 16) {
            uint4 hd[2], qv[2][4];
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const uint8_t *blk = a.w + (r0 + (r == 1 && has_b ? 1 : 0)) * rowbytes + (int64_t)sb * QKB;
                hd[r] = ldg_na(blk);
#pragma unroll
                for (int k = 0; k < 4; ++k) qv[r][k] = ldg_na(blk + 16 + 64 * h + 16 * k);
            }
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                if (r == 1 && !has_b) break;
                const float dw = half_bits_to_f32(hd[r].x & 0xffffu), dmw = half_bits_to_f32(hd[r].x >> 16);
                // get_scale_min_k4 for sub-blocks 4h..4h+3, four at a time on the
                // scale words W0 = bytes 0-3, W1 = 4-7, W2 = 8-11
                const uint32_t W0 = hd[r].y, W1 = hd[r].z, W2 = hd[r].w;
                const uint32_t scw = h ? ((W2 & 0x0f0f0f0fu) | (((W0 >> 6) & 0x03030303u) << 4)) : (W0 & 0x3f3f3f3fu);
                const uint32_t mnw = h ? (((W2 >> 4) & 0x0f0f0f0fu) | (((W1 >> 6) & 0x03030303u) << 4))
                                       : (W1 & 0x3f3f3f3fu);
                int sc[4], mn[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    sc[j] = (int)((scw >> (8 * j)) & 0xffu);
                    mn[j] = (int)((mnw >> (8 * j)) & 0xffu);
                }
                const uint32_t q[16] = {qv[r][0].x, qv[r][0].y, qv[r][0].z, qv[r][0].w, qv[r][1].x, qv[r][1].y,
                                        qv[r][1].z, qv[r][1].w, qv[r][2].x, qv[r][2].y, qv[r][2].z, qv[r][2].w,
                                        qv[r][3].x, qv[r][3].y, qv[r][3].z, qv[r][3].w};
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    if (m >= a.M) break;
                    const uint8_t *xrow = xs + (size_t)m * K;
                    int S = 0;
#pragma unroll
                    for (int cc = 0; cc < 2; ++cc) {  // sub-block pair c = 2h + cc: low nibbles = 2c, high = 2c + 1
                        const int c = 2 * h + cc;
                        const uint4 xl0 = *reinterpret_cast<const uint4 *>(xrow + xchunk_k(sb, 4 * c + 0));
                        const uint4 xl1 = *reinterpret_cast<const uint4 *>(xrow + xchunk_k(sb, 4 * c + 1));
                        const uint4 xh0 = *reinterpret_cast<const uint4 *>(xrow + xchunk_k(sb, 4 * c + 2));
                        const uint4 xh1 = *reinterpret_cast<const uint4 *>(xrow + xchunk_k(sb, 4 * c + 3));
                        const uint32_t xl[8] = {xl0.x, xl0.y, xl0.z, xl0.w, xl1.x, xl1.y, xl1.z, xl1.w};
                        const uint32_t xh[8] = {xh0.x, xh0.y, xh0.z, xh0.w, xh1.x, xh1.y, xh1.z, xh1.w};
                        int il = 0, ih = 0;
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const uint32_t w = q[8 * cc + i];
                            il = __dp4a((int)(w & 0x0F0F0F0Fu), (int)xl[i], il);
                            ih = __dp4a((int)((w >> 4) & 0x0F0F0F0Fu), (int)xh[i], ih);
                        }
                        S += sc[2 * cc] * il + sc[2 * cc + 1] * ih;
                    }
                    const int *s32 = x32 + ((size_t)m * a.nsb + sb) * 8 + 4 * h;
                    const int Mv = mn[0] * s32[0] + mn[1] * s32[1] + mn[2] * s32[2] + mn[3] * s32[3];
                    const float dx = xd[(size_t)m * a.nsb + sb];
                    acc[r][m] = fmaf(dw * dx, (float)S, acc[r][m]);
                    acc[r][m] = fmaf(-(dmw * dx), (float)Mv, acc[r][m]);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                float t = acc[r][m];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
                acc[r][m] = t;
            }
        }
        if (lane < 2 * MT) {
            const int r = lane / MT, m = lane % MT;
            const int64_t n = r0 + r;
            if (m < a.M && (r == 0 || has_b)) {
                float t = 0.0f;
#pragma unroll
                for (int rr = 0; rr < 2; ++rr)
#pragma unroll
                    for (int mm = 0; mm < MT; ++mm)
                        if (rr == r && mm == m) t = acc[rr][mm];
                if (a.bias) t = t + __ldg(a.bias + n);
                store_out(a.y, a.y_dtype, (int64_t)m * a.y_row_stride + n, t);
            }
        }
    }
}

size_t q4k_smem(int M, int nsb) { return (size_t)M * (nsb * QK + nsb * 4 + nsb * 32) + 16; }

template <int MT>
int launch_q4k_gemv(const Q4kArgs &a, cudaStream_t stream, const DeviceFacts &f) {
    const size_t smem = q4k_smem(a.M, a.nsb);
    static int configured_for[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && configured_for[dev] < (int)smem) {
        int st = check_cuda(cudaFuncSetAttribute(q4k_gemv_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)smem),
                            "torch._C._quantized_linear", "cudaFuncSetAttribute (q4_k)");
        if (st) return st;
        configured_for[dev] = (int)smem;
    }
    const int64_t pairs = (a.N + 1) / 2;
    int64_t grid = (int64_t)f.sm_count * 2;
    const int64_t need = (pairs + 7) / 8;
    if (need < grid) grid = need;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int st = check_cuda(cudaLaunchKernelEx(&cfg, q4k_gemv_kernel<MT>, a), "torch._C._quantized_linear",
                        "cudaLaunchKernelEx (q4_k GEMV)");
    if (st) return st;
    __atomic_fetch_add(&counters().q4_gemv_generic, 1ull, __ATOMIC_RELAXED);
    return TN_OK;
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
    tn::q4k_dequantize_kernel<<<(unsigned)((nsb * 4 + threads - 1) / threads), threads, 0, (cudaStream_t)stream>>>(
        static_cast<const uint8_t *>(blob), out, nsb);
    __atomic_fetch_add(&tn::counters().q4_codec_launches, 1ull, __ATOMIC_RELAXED);
    return tn::check_launch(op.c_str());
}

extern "C" int tn_q4_k_linear(const void *x, int x_dtype, int64_t x_row_stride, const void *w_blob, const float *bias,
                              void *y, int y_dtype, int64_t M, int64_t N, int64_t K, int act_mode, void *stream_) {
    const std::string op = "torch._C._quantized_linear";
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
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
    tn::DeviceFacts f{};
    int st = tn::device_facts(&f);
    if (st) return st;
    const int nsb = (int)(K / 256);
    int chunk = 0;
    for (int mt = 16; mt >= 1; mt >>= 1)
        if (tn::q4k_smem(mt, nsb) + 1024 <= (size_t)f.smem_optin) {
            chunk = mt;
            break;
        }
    if (chunk == 0)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": in_features " + std::to_string(K) +
                                                         " is too large for the q4_k kernel's shared memory");
    // Workspace: Q8_K codes [M][K], d [M][K/256], sub-block code sums [M][K/32].
    const size_t codes = ((size_t)M * K + 255) & ~size_t(255), dsz = ((size_t)M * nsb * 4 + 255) & ~size_t(255);
    void *ws = nullptr;
    st = tn::workspace(&ws, codes + dsz + (size_t)M * nsb * 32 + 256, stream, /*slot=*/0);
    if (st) return st;
    int8_t *xq = static_cast<int8_t *>(ws);
    float *xd = reinterpret_cast<float *>(static_cast<uint8_t *>(ws) + codes);
    int *xs32 = reinterpret_cast<int *>(static_cast<uint8_t *>(ws) + codes + dsz);
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
        tn::Q4kArgs a{};
        a.w = static_cast<const uint8_t *>(w_blob);
        a.xq = xq + m0 * K;
        a.xd = xd + m0 * nsb;
        a.xs32 = xs32 + m0 * nsb * 8;
        a.bias = bias;
        a.y = static_cast<uint8_t *>(y) + (size_t)m0 * N * ysz;
        a.y_dtype = y_dtype;
        a.M = (int)((M - m0) < chunk ? (M - m0) : chunk);
        a.nsb = nsb;
        a.N = N;
        a.xq_row_stride = K;
        a.y_row_stride = N;
        if (a.M <= 1) st = tn::launch_q4k_gemv<1>(a, stream, f);
        else if (a.M <= 2) st = tn::launch_q4k_gemv<2>(a, stream, f);
        else if (a.M <= 4) st = tn::launch_q4k_gemv<4>(a, stream, f);
        else if (a.M <= 8) st = tn::launch_q4k_gemv<8>(a, stream, f);
        else st = tn::launch_q4k_gemv<16>(a, stream, f);
        if (st) return st;
    }
    return TN_OK;
}
