// q4_gemm.cu -- the prefill Q4_0 linear (many activation rows) on the 5th
// generation tensor cores.
//
// Arithmetic (the reference's, k_quants.rs:312-330 and 2430-2580): for every
// output y[m, n] = sum over 32-blocks b of (isum_b * d_w[n, b]) * d_x[m, b],
// isum_b = sum of q8 codes times (q4 nibble - 8), an exact integer. The
// tensor core computes isum_b exactly: both operands are small integers held
// in f16 (|q8| <= 127, |q4 - 8| <= 8) and every partial sum stays below 2^15,
// so the f32 accumulator is exact. A block's scales differ per row and per
// column, so each block is its own MMA into TMEM and the epilogue warps apply
// acc = fma(isum_b * d_w, d_x, acc) in f32 -- the reference's two products
// with the final rounding merged into the add.
//
// One CTA = 128 activation rows x 128 weight rows, 14 warps:
//   warp 0      TMA producer: A panels (f16 codes, 64 K-elements, 128-byte
//               swizzle) and raw weight chunks (128 rows x 144 bytes = 8 Q4_0
//               blocks per row, straight from the GGML blob)
//   warp 1      TMEM owner and MMA issuer (one thread): per block 2 MMAs of
//               K = 16, M = N = 128, into one of 4 TMEM accumulators
//   warps 2-5   converters (thread = weight row): raw blocks -> f16 (q - 8)
//               in the swizzled K-major panel layout the MMA reads (the
//               K order within a block permuted as the activation codes
//               are), plus the f32 block scales d_w
//   warps 6-13  epilogue: read each block's isum tile from TMEM, scale and
//               accumulate in registers (thread = one row, 64 columns), then
//               add the bias and store y
// Every wait is bounded; a wait that gives up raises a CTA-wide abort flag so
// the other roles stop too, the producer waits for its copies in flight, the
// MMA issuer for its MMAs, and TMEM is freed.
#include "q4_kernels.cuh"
#include "tc05.cuh"

namespace tn {
namespace {

constexpr int GM = 128, GN = 128;
constexpr int NA = 4, NB = 4, NR = 2, NS = 4;
constexpr int PANEL = 128 * 128;     // 128 rows x 64 f16
constexpr int RAW = GN * 144;        // 128 rows x 8 Q4_0 blocks
constexpr int OFF_A = 0, OFF_B = NA * PANEL, OFF_R = OFF_B + NB * PANEL, OFF_DW = OFF_R + NR * RAW;
constexpr int OFF_BAR = OFF_DW + NB * 2 * GN * 4;
constexpr int NBARS = 2 * NA + 2 * NB + 2 * NR + 2 * NS + 1;
constexpr size_t GEMM_SMEM = OFF_BAR + 256 + 1024;
constexpr int CONV_WARPS = 4, EPI_WARPS = 8, EPI_COLS = GN / (EPI_WARPS / 4);
constexpr int GEMM_THREADS = (2 + CONV_WARPS + EPI_WARPS) * 32;
static_assert(NBARS * 8 + 8 <= 256, "barrier area");

struct GemmArgs {
    const float *xd;  // [M][nb] activation block scales
    const float *bias;
    void *y;
    int y_dtype;
    int64_t y_row_stride;
    int M, N, nb;
    int vec_store;  // rows of y 16-byte aligned and N % 8 == 0
    int *err;
};

__device__ __forceinline__ bool wait_or_abort(uint64_t *bar, uint32_t parity, volatile int *abort, int *err) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long start = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (*abort) return false;
        if (clock64() - start > kWaitBudgetCycles) {
            *abort = 1;
            record_device_error(err, DEV_ERR_WAIT_FULL);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void st_shared_v4(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}

__device__ __forceinline__ void ld_shared_v4(uint32_t a, uint32_t &x, uint32_t &y, uint32_t &z, uint32_t &w) {
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(x), "=r"(y), "=r"(z), "=r"(w) : "r"(a));
}

// Two nibble codes (bits 0-3 and 16-19 of v) -> half2 (code - 8), exact:
// 0x6400 | c is the f16 1024 + c, and 1024 + c - 1032 = c - 8.
__device__ __forceinline__ uint32_t nib2_to_h2(uint32_t v) {
    const uint32_t h = (v & 0x000F000Fu) | 0x64006400u;
    const __half2 r = __hsub2(*reinterpret_cast<const __half2 *>(&h), __halves2half2(__ushort_as_half(0x6408),
                                                                                        __ushort_as_half(0x6408)));
    return *reinterpret_cast<const uint32_t *>(&r);
}

// Packed pairs of f32 (sm_100 f32x2 arithmetic: two lanes per instruction,
// each rounded as the scalar operation would be).
__device__ __forceinline__ void fma2(float &a0, float &a1, float x0, float x1, float y0, float y1) {
    asm("{\n\t.reg .b64 ra, rx, ry;\n\tmov.b64 ra, {%0, %1};\n\tmov.b64 rx, {%2, %3};\n\tmov.b64 ry, {%4, %5};\n\t"
        "fma.rn.f32x2 ra, rx, ry, ra;\n\tmov.b64 {%0, %1}, ra;\n\t}"
        : "+f"(a0), "+f"(a1)
        : "f"(x0), "f"(x1), "f"(y0), "f"(y1));
}
__device__ __forceinline__ void mul2(float &d0, float &d1, float x0, float x1, float y0, float y1) {
    asm("{\n\t.reg .b64 rd, rx, ry;\n\tmov.b64 rx, {%2, %3};\n\tmov.b64 ry, {%4, %5};\n\t"
        "mul.rn.f32x2 rd, rx, ry;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "f"(x0), "f"(x1), "f"(y0), "f"(y1));
}

__global__ void __launch_bounds__(GEMM_THREADS, 1) q4_gemm_kernel(const __grid_constant__ CUtensorMap map_a,
                                                                  const __grid_constant__ CUtensorMap map_w,
                                                                  const GemmArgs g) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sb = smem_u32(base);
    uint64_t *bars = reinterpret_cast<uint64_t *>(base + OFF_BAR);
    uint64_t *a_full = bars, *a_empty = a_full + NA, *b_full = a_empty + NA, *b_empty = b_full + NB,
             *r_full = b_empty + NB, *r_empty = r_full + NR, *s_full = r_empty + NR, *s_empty = s_full + NS,
             *done = s_empty + NS;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
    const float *dwt = reinterpret_cast<const float *>(base + OFF_DW);  // [NB][2][GN]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.x * GM, n0 = blockIdx.y * GN;
    const int nb = g.nb, nchunks = nb / 8;

    if (warp == 1) tc05::alloc(tmem_slot, 512);
    if (tid == 0) {
        for (int i = 0; i < NA; ++i) {
            mbar_init(&a_full[i], 1);
            mbar_init(&a_empty[i], 1);
        }
        for (int i = 0; i < NB; ++i) {
            mbar_init(&b_full[i], CONV_WARPS);
            mbar_init(&b_empty[i], 1 + EPI_WARPS);
        }
        for (int i = 0; i < NR; ++i) {
            mbar_init(&r_full[i], 1);
            mbar_init(&r_empty[i], CONV_WARPS);
        }
        for (int i = 0; i < NS; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&s_empty[i], EPI_WARPS);
        }
        mbar_init(done, 1);
        *abort = 0;
        fence_mbar_init();
        tc05::prefetch_map(&map_a);
        tc05::prefetch_map(&map_w);
    }
    tc05::fence_before();
    __syncthreads();
    tc05::fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();
    pdl_wait();

    if (warp == 0) {
        // ---------------- producer
        if (lane == 0) {
            // A panels, gated by the MMAs. (Raw weight chunks are requested by
            // the converters, NR chunks ahead of their own progress.)
            int a_issued = 0;
            for (int p = 0; p < 4 * nchunks && !*abort; ++p) {
                const int as = p % NA;
                if (p >= NA && !wait_or_abort(&a_empty[as], ((p / NA) - 1) & 1, abort, g.err)) break;
                mbar_arrive_expect_tx(&a_full[as], PANEL);
                tc05::tma_load_2d(sb + OFF_A + as * PANEL, &map_a, p * 64, m0, &a_full[as]);
                ++a_issued;
            }
            // Drain: the last copy issued into each slot has landed.
            for (int p = a_issued > NA ? a_issued - NA : 0; p < a_issued; ++p)
                if (!mbar_wait(&a_full[p % NA], (p / NA) & 1)) record_device_error(g.err, DEV_ERR_DRAIN);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer
        if (lane == 0) {
            const uint32_t idesc = tc05::idesc_f16(false, GM, GN, false);
            for (int b = 0; b < nb; ++b) {
                const int p = b >> 1, h = b & 1, s = b % NS;
                if (h == 0 && (!wait_or_abort(&a_full[p % NA], (p / NA) & 1, abort, g.err) ||
                               !wait_or_abort(&b_full[p % NB], (p / NB) & 1, abort, g.err)))
                    break;
                if (b >= NS && !wait_or_abort(&s_empty[s], ((b / NS) - 1) & 1, abort, g.err)) break;
                tc05::fence_after();
                const uint32_t ab = sb + OFF_A + (p % NA) * PANEL, bb = sb + OFF_B + (p % NB) * PANEL;
#pragma unroll
                for (int kk = 0; kk < 2; ++kk) {
                    const uint32_t off = h * 64 + kk * 32;
                    tc05::mma_ss(tmem + s * GN, tc05::desc_sw128(ab + off, 16, 1024),
                                 tc05::desc_sw128(bb + off, 16, 1024), idesc, kk);
                }
                tc05::commit(&s_full[s]);
                if (h == 1) {
                    tc05::commit(&a_empty[p % NA]);
                    tc05::commit(&b_empty[p % NB]);
                }
            }
            tc05::commit(done);
            if (!mbar_wait(done, 0)) record_device_error(g.err, DEV_ERR_DRAIN);
        }
    } else if (warp < 2 + CONV_WARPS) {
        // ---------------- converters: thread ct owns weight row n0 + ct of the tile
        const int ct = tid - 64;
        const bool loader = ct == 0;
        int r_issued = 0;
        auto load_raw = [&](int c) {
            const int rs = c % NR;
            mbar_arrive_expect_tx(&r_full[rs], RAW);
            tc05::tma_load_2d(sb + OFF_R + rs * RAW, &map_w, c * 144, n0, &r_full[rs]);
            ++r_issued;
        };
        if (loader)
            for (int c = 0; c < NR && c < nchunks; ++c) load_raw(c);
        float *dws = reinterpret_cast<float *>(base + OFF_DW);
        for (int c = 0; c < nchunks; ++c) {
            const int rs = c % NR;
            if (!wait_or_abort(&r_full[rs], (c / NR) & 1, abort, g.err)) break;
            // This row's 8 blocks (144 bytes, 16-byte aligned rows: conflict-free
            // 128-bit loads), in two halves of 80 bytes (blocks 0-3, then 4-7).
            const uint32_t row = sb + OFF_R + rs * RAW + ct * 144;
            bool ok = true;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                uint32_t raw[20];
#pragma unroll
                for (int i = 0; i < 5; ++i)
                    ld_shared_v4(row + 64 * half + 16 * i, raw[4 * i], raw[4 * i + 1], raw[4 * i + 2], raw[4 * i + 3]);
                if (half == 1) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&r_empty[rs]);
                }
#pragma unroll
                for (int qq = 0; qq < 2; ++qq) {
                    const int q = 2 * half + qq, p = 4 * c + q, bs = p % NB;
                    if (p >= NB && !wait_or_abort(&b_empty[bs], ((p / NB) - 1) & 1, abort, g.err)) {
                        ok = false;
                        break;
                    }
                    const uint32_t prow = sb + OFF_B + bs * PANEL + ct * 128;
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int b = 2 * q + h, w0 = (18 * b) / 4 - 16 * half;  // block b starts at byte 18 b
                        uint32_t d, w[4];
                        if ((b & 1) == 0) {  // 4-byte aligned block: d low half, qs 2 bytes in
                            d = raw[w0] & 0xffffu;
#pragma unroll
                            for (int i = 0; i < 4; ++i) w[i] = __funnelshift_r(raw[w0 + i], raw[w0 + i + 1], 16);
                        } else {  // d is the high half of word w0, qs word aligned
                            d = raw[w0] >> 16;
#pragma unroll
                            for (int i = 0; i < 4; ++i) w[i] = raw[w0 + 1 + i];
                        }
                        // word j (qs[4j..4j+3]) -> elements 4j + {0, 2, 16, 18, 1, 3, 17, 19}
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const uint32_t cidx = 4 * h + j;
                            st_shared_v4(prow + ((cidx ^ (ct & 7)) << 4), nib2_to_h2(w[j]), nib2_to_h2(w[j] >> 4),
                                         nib2_to_h2(w[j] >> 8), nib2_to_h2(w[j] >> 12));
                        }
                        dws[(bs * 2 + h) * GN + ct] = half_bits_to_f32(d);
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&b_full[bs]);
                }
                if (!ok) break;
            }
            if (!ok) break;
            // Every converter warp has read chunk c: its raw slot takes chunk c + NR.
            if (loader && c + NR < nchunks) {
                if (!wait_or_abort(&r_empty[rs], (c / NR) & 1, abort, g.err)) break;
                load_raw(c + NR);
            }
        }
        if (loader)  // drain: the last raw copy issued into each slot has landed
            for (int c = r_issued > NR ? r_issued - NR : 0; c < r_issued; ++c)
                if (!mbar_wait(&r_full[c % NR], (c / NR) & 1)) record_device_error(g.err, DEV_ERR_DRAIN);
    } else {
        // ---------------- epilogue: thread = activation row, 64 weight columns
        const int quad = warp & 3, cg = (warp - 2 - CONV_WARPS) >> 2;
        const int mrow = quad * 32 + lane, m = m0 + mrow;
        const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + cg * EPI_COLS;
        const float *xdrow = g.xd + (int64_t)(m < g.M ? m : g.M - 1) * nb;
        float acc[EPI_COLS];
#pragma unroll
        for (int i = 0; i < EPI_COLS; ++i) acc[i] = 0.0f;
        bool ok = true;
        // acc[o .. o + 15] += (v * dw[o ..]) * dx, as packed f32 pairs
        auto scale_add = [&](const float (&v)[16], const float *dw, int o, float dx) {
#pragma unroll
            for (int i = 0; i < 16; i += 4) {
                const float4 w4 = *reinterpret_cast<const float4 *>(dw + o + i);
                float t0, t1, t2, t3;
                mul2(t0, t1, v[i], v[i + 1], w4.x, w4.y);
                mul2(t2, t3, v[i + 2], v[i + 3], w4.z, w4.w);
                fma2(acc[o + i], acc[o + i + 1], t0, t1, dx, dx);
                fma2(acc[o + i + 2], acc[o + i + 3], t2, t3, dx, dx);
            }
        };
        float4 nx0 = reinterpret_cast<const float4 *>(xdrow)[0], nx1 = reinterpret_cast<const float4 *>(xdrow)[1];
        for (int c = 0; c < nchunks && ok; ++c) {
            // the activation scales of the next chunk's 8 blocks are loaded a chunk ahead
            const float dx8[8] = {nx0.x, nx0.y, nx0.z, nx0.w, nx1.x, nx1.y, nx1.z, nx1.w};
            if (c + 1 < nchunks) {
                nx0 = reinterpret_cast<const float4 *>(xdrow + 8 * (c + 1))[0];
                nx1 = reinterpret_cast<const float4 *>(xdrow + 8 * (c + 1))[1];
            }
#pragma unroll
            for (int bi = 0; bi < 8; ++bi) {
                const int b = 8 * c + bi, s = b % NS, p = b >> 1, h = b & 1;
                if (!wait_or_abort(&s_full[s], (b / NS) & 1, abort, g.err)) {
                    ok = false;
                    break;
                }
                if (h == 0 && !wait_or_abort(&b_full[p % NB], (p / NB) & 1, abort, g.err)) {
                    ok = false;
                    break;
                }
                tc05::fence_after();
                const float *dw = dwt + ((p % NB) * 2 + h) * GN + cg * EPI_COLS;
#pragma unroll
                for (int k = 0; k < EPI_COLS / 16; ++k) {
                    float v[16];
                    tc05::ld16(taddr + s * GN + 16 * k, v);
                    tc05::wait_ld();
                    if (k == EPI_COLS / 16 - 1) {
                        tc05::fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&s_empty[s]);
                    }
                    scale_add(v, dw, 16 * k, dx8[bi]);
                }
                if (h == 1) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&b_empty[p % NB]);
                }
            }
        }
        if (ok && m < g.M) {
            const int nc = n0 + cg * EPI_COLS;
            const int64_t yo = (int64_t)m * g.y_row_stride + nc;
#pragma unroll
            for (int i = 0; i < EPI_COLS; ++i)
                if (g.bias && nc + i < g.N) acc[i] += g.bias[nc + i];
            if (g.vec_store && nc + EPI_COLS <= g.N && g.y_dtype != TN_F32) {
                uint4 *dst = reinterpret_cast<uint4 *>(static_cast<uint8_t *>(g.y) + yo * 2);
#pragma unroll
                for (int i = 0; i < EPI_COLS / 8; ++i) {
                    uint32_t w[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float lo = acc[8 * i + 2 * e], hi = acc[8 * i + 2 * e + 1];
                        if (g.y_dtype == TN_BF16) {
                            const __nv_bfloat162 t = __floats2bfloat162_rn(lo, hi);
                            w[e] = *reinterpret_cast<const uint32_t *>(&t);
                        } else {
                            const __half2 t = __floats2half2_rn(lo, hi);
                            w[e] = *reinterpret_cast<const uint32_t *>(&t);
                        }
                    }
                    dst[i] = make_uint4(w[0], w[1], w[2], w[3]);
                }
            } else if (g.vec_store && nc + EPI_COLS <= g.N) {
                float4 *dst = reinterpret_cast<float4 *>(static_cast<float *>(g.y) + yo);
#pragma unroll
                for (int i = 0; i < EPI_COLS / 4; ++i)
                    dst[i] = make_float4(acc[4 * i], acc[4 * i + 1], acc[4 * i + 2], acc[4 * i + 3]);
            } else {
#pragma unroll
                for (int i = 0; i < EPI_COLS; ++i)
                    if (nc + i < g.N) store_out(g.y, g.y_dtype, yo + i, acc[i]);
            }
        }
    }

    tc05::fence_before();
    __syncthreads();
    if (warp == 1) {
        tc05::fence_after();
        tc05::dealloc(tmem, 512);
    }
}

}  // namespace

bool q4_gemm_applies(const void *w_blob, int64_t M, int64_t N, int64_t K) {
    return M > 16 && K % 256 == 0 && K > 0 && N > 0 && (reinterpret_cast<uintptr_t>(w_blob) & 15) == 0 &&
           (M + GM - 1) / GM <= 0x7fffffff && (N + GN - 1) / GN <= 65535;
}

int launch_q4_gemm(const __half *xq, int64_t xq_row_stride, const float *xd, const uint8_t *w, const float *bias,
                   void *y, int y_dtype, int64_t y_row_stride, int64_t M, int64_t N, int64_t K, cudaStream_t stream) {
    const char *op = "torch._C._quantized_linear";
    const int64_t nb = K / 32, rowbytes = nb * 18;
    CUtensorMap ma, mw;
    int st = encode_map_2d(&ma, xq, 2, (uint64_t)K, (uint64_t)M, (uint64_t)xq_row_stride * 2, 64, GM, true);
    if (st) return st;
    st = encode_map_2d(&mw, w, 1, (uint64_t)rowbytes, (uint64_t)N, (uint64_t)rowbytes, 144, GN, false);
    if (st) return st;
    GemmArgs g{};
    g.xd = xd;
    g.bias = bias;
    g.y = y;
    g.y_dtype = y_dtype;
    g.y_row_stride = y_row_stride;
    g.M = (int)M;
    g.N = (int)N;
    g.nb = (int)nb;
    const size_t es = tn_dtype_size(y_dtype);
    g.vec_store = (reinterpret_cast<uintptr_t>(y) % 16 == 0) && ((y_row_stride * (int64_t)es) % 16 == 0);
    g.err = device_error_word();
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        st = check_cuda(cudaFuncSetAttribute(q4_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GEMM_SMEM),
                        op, "cudaFuncSetAttribute");
        if (st) return st;
        configured[dev] = 1;
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((M + GM - 1) / GM), (unsigned)((N + GN - 1) / GN));
    cfg.blockDim = dim3(GEMM_THREADS);
    cfg.dynamicSmemBytes = GEMM_SMEM;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, q4_gemm_kernel, ma, mw, g);
    if (e != cudaSuccess) {
        cudaFuncAttributes fa{};
        cudaFuncGetAttributes(&fa, q4_gemm_kernel);
        return check_cuda(e, op, ("cudaLaunchKernelEx (q4 gemm: " + std::to_string(fa.numRegs) + " registers, " +
                                  std::to_string(fa.maxThreadsPerBlock) + " max threads, " +
                                  std::to_string(GEMM_SMEM) + " B smem)")
                                     .c_str());
    }
    __atomic_fetch_add(&counters().q4_gemm_launches, 1ull, __ATOMIC_RELAXED);
    return TN_OK;
}

}  // namespace tn
