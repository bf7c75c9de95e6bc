// q4_gemv.cu -- decode Q4_0 linear (M <= 16 activation rows), the reference's
// Q8_0-activation arithmetic, streamed from HBM with bulk-async (TMA) copies.
//
// Work split. CTA c of G owns output columns (weight rows) [c*N/G, (c+1)*N/G).
// One producer warp streams those weight rows -- each row is K/32 GGML blocks of
// 18 bytes, i.e. rowbytes = 18*K/32 contiguous bytes -- into a ring of shared
// memory slots with cp.async.bulk (one copy per row, completion counted on the
// slot's mbarrier). Eight consumer warps take rows round-robin; a warp splits
// its row's blocks across its 32 lanes in pairs (36 bytes = 9 words; 9 is odd,
// so the 32 lanes of a warp hit 32 different banks), takes exact integer block
// dots with dp4a against the Q8_0 activation codes held in shared memory, and
// applies the per-block scales in float32. A warp-shuffle tree sums the lanes.
//
// Arithmetic (reference: k_quants.rs:312-330 vec_dot_unopt). Per block b:
//   I_b = sum_j (q4_j - 8) * q8_j                 exact int32
//   t_b = I_b * (d_w * d_x)                        d_w*d_x is exact in f32 (11+11 bits)
// The int -> float step is a magic-number add folded into dp4a's accumulator
// (bits 0x4B400000 + I read as float = 12582912 + I, exact for |I| < 2^22), and
// the "-8" offset is folded into the subtracted constant xc = 12582912 + 8*sum(q8).
// Each lane accumulates its blocks with fmaf (one rounding per block), then a
// 5-level shuffle tree: depth ceil(nb/32) + 5 <= nb + 3, the depth the
// reference's own bound counts (scripts/q4quality/q4_gguf_ref.py:370-405).
#include "q4_kernels.cuh"

namespace tn {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kMaxSlots = 32;
constexpr uint32_t kMagic = 0x4B400000u;  // 12582912.0f

struct GemvParams {
    const uint8_t *w;
    const int8_t *xq;
    const float *xd;
    const float *xc;
    const float *bias;
    void *y;
    int64_t xq_row_stride;
    int64_t y_row_stride;
    int64_t N;
    int y_dtype;
    int M;
    int nb;       // blocks per weight row
    int nbp;      // nb rounded up to even (x staging granularity)
    int rowbytes; // 18 * nb
    int nslots;
    int *err;
};

// Shared-memory layout (dynamic):
//   [0, 16*kMaxSlots)                   full[kMaxSlots], empty[kMaxSlots] mbarriers
//   xs   M * nbp * 32 bytes             activation codes, pair-swizzled (see stage_x)
//   xds  M * nbp floats                 widened activation scales
//   xcs  M * nbp floats                 offset constants
//   slots nslots * rowbytes             weight rows (16-byte aligned)
struct Smem {
    uint64_t *full, *empty;
    uint8_t *xs;
    float *xds, *xcs;
    uint8_t *slots;
};

__device__ __forceinline__ Smem carve(uint8_t *base, const GemvParams &p) {
    Smem s;
    s.full = reinterpret_cast<uint64_t *>(base);
    s.empty = s.full + kMaxSlots;
    size_t off = 16 * kMaxSlots;
    s.xs = base + off;
    off += (size_t)p.M * p.nbp * 32;
    s.xds = reinterpret_cast<float *>(base + off);
    off += (size_t)p.M * p.nbp * 4;
    s.xcs = reinterpret_cast<float *>(base + off);
    off += (size_t)p.M * p.nbp * 4;
    off = (off + 127) & ~size_t(127);
    s.slots = base + off;
    return s;
}

// Byte offset of 16-byte chunk c (0..3) of block pair `pair` inside one
// activation row of the staged codes. Chunks 0/1 are the low/high 16 codes of
// block 2*pair, chunks 2/3 those of block 2*pair+1. The XOR spreads the eight
// lanes of a quarter-warp (which read pairs l..l+7) over all eight 16-byte bank
// groups, so every 128-bit load below is conflict-free.
__device__ __forceinline__ int xchunk(int pair, int c) { return pair * 64 + 16 * (c ^ ((pair >> 1) & 3)); }

template <int MT>
__device__ __forceinline__ void block_dot(uint32_t q0, uint32_t q1, uint32_t q2, uint32_t q3, uint32_t dbits, int b,
                                          const Smem &s, const GemvParams &p, float (&acc)[MT]) {
    const uint32_t lo0 = q0 & 0x0F0F0F0Fu, lo1 = q1 & 0x0F0F0F0Fu, lo2 = q2 & 0x0F0F0F0Fu, lo3 = q3 & 0x0F0F0F0Fu;
    const uint32_t hi0 = (q0 >> 4) & 0x0F0F0F0Fu, hi1 = (q1 >> 4) & 0x0F0F0F0Fu, hi2 = (q2 >> 4) & 0x0F0F0F0Fu,
                   hi3 = (q3 >> 4) & 0x0F0F0F0Fu;
    const float dw = half_bits_to_f32(dbits);
    const int pair = b >> 1, cb = (b & 1) * 2;
    const int off_lo = xchunk(pair, cb), off_hi = xchunk(pair, cb + 1);
    const int xrow = p.nbp * 32;
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        if (m < p.M) {
            const int4 xl = *reinterpret_cast<const int4 *>(s.xs + m * xrow + off_lo);
            const int4 xh = *reinterpret_cast<const int4 *>(s.xs + m * xrow + off_hi);
            int I = (int)kMagic;
            I = __dp4a((int)lo0, xl.x, I);
            I = __dp4a((int)lo1, xl.y, I);
            I = __dp4a((int)lo2, xl.z, I);
            I = __dp4a((int)lo3, xl.w, I);
            I = __dp4a((int)hi0, xh.x, I);
            I = __dp4a((int)hi1, xh.y, I);
            I = __dp4a((int)hi2, xh.z, I);
            I = __dp4a((int)hi3, xh.w, I);
            const float f = __int_as_float(I) - s.xcs[m * p.nbp + b];
            const float sc = dw * s.xds[m * p.nbp + b];
            acc[m] = fmaf(f, sc, acc[m]);
        }
    }
}

// Copy this CTA's activations into shared memory (all consumer threads).
__device__ __forceinline__ void stage_x(const Smem &s, const GemvParams &p, int tid, int nthr) {
    const int chunks_per_row = p.nbp * 2;  // 16-byte chunks
    for (int idx = tid; idx < p.M * chunks_per_row; idx += nthr) {
        const int m = idx / chunks_per_row, g = idx % chunks_per_row;
        const int b = g >> 1, half = g & 1;
        int4 v = make_int4(0, 0, 0, 0);
        if (b < p.nb) v = __ldg(reinterpret_cast<const int4 *>(p.xq + m * p.xq_row_stride + b * 32 + half * 16));
        const int pair = b >> 1, c = (b & 1) * 2 + half;
        *reinterpret_cast<int4 *>(s.xs + m * p.nbp * 32 + xchunk(pair, c)) = v;
    }
    for (int idx = tid; idx < p.M * p.nbp; idx += nthr) {
        const int m = idx / p.nbp, b = idx % p.nbp;
        s.xds[idx] = b < p.nb ? __ldg(p.xd + (int64_t)m * p.nb + b) : 0.0f;
        s.xcs[idx] = b < p.nb ? __ldg(p.xc + (int64_t)m * p.nb + b) : 12582912.0f;
    }
}

template <int MT>
__device__ __forceinline__ void finish_row(float (&acc)[MT], const GemvParams &p, int64_t n, int lane) {
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        float v = acc[m];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        acc[m] = v;
    }
    float mine = 0.0f;
#pragma unroll
    for (int m = 0; m < MT; ++m)
        if (lane == m) mine = acc[m];
    if (lane < p.M) {
        if (p.bias) mine = mine + __ldg(p.bias + n);
        store_out(p.y, p.y_dtype, lane * p.y_row_stride + n, mine);
    }
}

// 16-bit little-endian loads of one 18-byte block from global memory (the
// unstaged path: K % 256 != 0, so rows are not 16-byte multiples).
__device__ __forceinline__ void load_block_global(const uint8_t *blk, uint32_t &d, uint32_t &q0, uint32_t &q1,
                                                  uint32_t &q2, uint32_t &q3) {
    const unsigned short *h = reinterpret_cast<const unsigned short *>(blk);
    uint32_t u[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) u[i] = __ldg(h + i);
    d = u[0];
    q0 = u[1] | (u[2] << 16);
    q1 = u[3] | (u[4] << 16);
    q2 = u[5] | (u[6] << 16);
    q3 = u[7] | (u[8] << 16);
}

template <int MT, bool STAGED>
__global__ void __launch_bounds__(kThreads, 1) q4_gemv_q8_kernel(const GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const Smem s = carve(smem_raw, p);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t G = gridDim.x, c = blockIdx.x;
    const int64_t r0 = c * p.N / G, r1 = (c + 1) * p.N / G;
    const int nrows = (int)(r1 - r0);

    if (STAGED && threadIdx.x == 0) {
        for (int i = 0; i < p.nslots; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ---------------- producer: one lane streams this CTA's weight rows
        if (STAGED && lane == 0) {
            // The weights may have been written by the previous kernel in the
            // stream (a quantise on the device), so wait for it like the
            // consumers do.
            pdl_wait();
            const uint64_t pol = policy_evict_first();
            int issued = 0;
            for (int i = 0; i < nrows; ++i) {
                const int slot = i % p.nslots, use = i / p.nslots;
                if (use > 0 && !mbar_wait(&s.empty[slot], (use - 1) & 1)) {
                    record_device_error(p.err, DEV_ERR_WAIT_EMPTY);
                    break;
                }
                mbar_arrive_expect_tx(&s.full[slot], (uint32_t)p.rowbytes);
                bulk_g2s_hint(s.slots + (size_t)slot * p.rowbytes, p.w + (r0 + i) * (int64_t)p.rowbytes,
                              (uint32_t)p.rowbytes, &s.full[slot], pol);
                issued = i + 1;
            }
            // Drain: every copy issued must have landed before the CTA exits.
            // (On the normal path the consumers already waited for all of them.)
            for (int i = issued > p.nslots ? issued - p.nslots : 0; i < issued; ++i) {
                if (!mbar_wait(&s.full[i % p.nslots], (i / p.nslots) & 1)) {
                    record_device_error(p.err, DEV_ERR_DRAIN);
                    break;
                }
            }
        }
        return;
    }

    // ---------------- consumers
    pdl_wait();  // the activations may come from the previous kernel in the stream
    stage_x(s, p, threadIdx.x, kConsumerWarps * 32);
    asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");

    const int npairs = p.nb >> 1;
    for (int i = warp; i < nrows; i += kConsumerWarps) {
        const int64_t n = r0 + i;
        float acc[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[m] = 0.0f;
        if (STAGED) {
            const int slot = i % p.nslots;
            if (!mbar_wait(&s.full[slot], (i / p.nslots) & 1)) {
                record_device_error(p.err, DEV_ERR_WAIT_FULL);
                return;
            }
            const uint32_t *row = reinterpret_cast<const uint32_t *>(s.slots + (size_t)slot * p.rowbytes);
            for (int pp = lane; pp < npairs; pp += 32) {
                const uint32_t *w9 = row + pp * 9;
                const uint32_t w0 = w9[0], w1 = w9[1], w2 = w9[2], w3 = w9[3], w4 = w9[4];
                const uint32_t w5 = w9[5], w6 = w9[6], w7 = w9[7], w8 = w9[8];
                block_dot<MT>(__funnelshift_r(w0, w1, 16), __funnelshift_r(w1, w2, 16), __funnelshift_r(w2, w3, 16),
                              __funnelshift_r(w3, w4, 16), w0 & 0xffffu, 2 * pp, s, p, acc);
                block_dot<MT>(w5, w6, w7, w8, w4 >> 16, 2 * pp + 1, s, p, acc);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.empty[slot]);
        } else {
            const uint8_t *row = p.w + n * (int64_t)p.rowbytes;
            for (int b = lane; b < p.nb; b += 32) {
                uint32_t d, q0, q1, q2, q3;
                load_block_global(row + b * 18, d, q0, q1, q2, q3);
                block_dot<MT>(q0, q1, q2, q3, d, b, s, p, acc);
            }
        }
        finish_row<MT>(acc, p, n, lane);
    }
}

template <int MT, bool STAGED>
int launch_variant(const GemvParams &p, int grid, size_t smem, cudaStream_t stream) {
    static int configured_for[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && configured_for[dev] < (int)smem) {
        int st = check_cuda(cudaFuncSetAttribute(q4_gemv_q8_kernel<MT, STAGED>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                            "torch._C._quantized_linear", "cudaFuncSetAttribute");
        if (st) return st;
        configured_for[dev] = (int)smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int st = check_cuda(cudaLaunchKernelEx(&cfg, q4_gemv_q8_kernel<MT, STAGED>, p), "torch._C._quantized_linear",
                        "cudaLaunchKernelEx");
    if (st) return st;
    __atomic_fetch_add(STAGED ? &counters().q4_gemv_launches : &counters().q4_gemv_generic, 1ull, __ATOMIC_RELAXED);
    return TN_OK;
}

size_t smem_bytes(int M, int nbp, int nslots, int rowbytes) {
    size_t off = 16 * kMaxSlots + (size_t)M * nbp * 40;
    off = (off + 127) & ~size_t(127);
    return off + (size_t)nslots * rowbytes;
}

}  // namespace

int q4_gemv_max_rows(int64_t K) {
    DeviceFacts f{};
    if (device_facts(&f)) return 0;
    const int nb = (int)(K / 32), nbp = (nb + 1) & ~1, rowbytes = 18 * nb;
    const bool staged = (K % 256 == 0);
    for (int mt = 16; mt >= 1; mt >>= 1)
        if (smem_bytes(mt, nbp, staged ? kConsumerWarps : 0, rowbytes) <= (size_t)f.smem_optin) return mt;
    return 0;
}

int launch_q4_gemv_q8(const uint8_t *w, const int8_t *xq, const float *xd, const float *xc, int64_t xq_row_stride,
                      const float *bias, void *y, int y_dtype, int64_t y_row_stride, int M, int64_t N, int64_t K,
                      cudaStream_t stream) {
    const char *op = "torch._C._quantized_linear";
    DeviceFacts f{};
    int st = device_facts(&f);
    if (st) return st;
    GemvParams p{};
    p.w = w;
    p.xq = xq;
    p.xd = xd;
    p.xc = xc;
    p.bias = bias;
    p.y = y;
    p.xq_row_stride = xq_row_stride;
    p.y_row_stride = y_row_stride;
    p.N = N;
    p.y_dtype = y_dtype;
    p.M = M;
    p.nb = (int)(K / 32);
    p.nbp = (p.nb + 1) & ~1;
    p.rowbytes = 18 * p.nb;
    p.err = device_error_word();
    const bool staged = (K % 256 == 0) && ((reinterpret_cast<uintptr_t>(w) & 15) == 0);
    const size_t budget = (size_t)f.smem_optin;
    int nslots = 0;
    if (staged) {
        const size_t base = smem_bytes(M, p.nbp, 0, p.rowbytes);
        if (base + (size_t)kConsumerWarps * p.rowbytes > budget)
            return set_error(TN_ERR_NOT_IMPLEMENTED, std::string(op) + ": internal: activation tile too large for "
                                                                       "shared memory");
        nslots = (int)((budget - base) / p.rowbytes);
        // ~96 KB in flight per SM covers HBM latency; more only costs occupancy.
        const int want = (int)((96 * 1024 + p.rowbytes - 1) / p.rowbytes);
        nslots = nslots < want ? nslots : want;
        nslots = nslots < kMaxSlots ? nslots : kMaxSlots;
        // A multiple of the consumer-warp count: row i and row i - nslots then
        // belong to the same warp, so no warp ever waits on a slot's barrier
        // more than one phase ahead (parity waits cannot tell phases two apart).
        nslots = (nslots / kConsumerWarps) * kConsumerWarps;
        nslots = nslots > kConsumerWarps ? nslots : kConsumerWarps;
    } else if (smem_bytes(M, p.nbp, 0, 0) > budget) {
        return set_error(TN_ERR_NOT_IMPLEMENTED, std::string(op) + ": internal: activation tile too large for "
                                                                   "shared memory");
    }
    p.nslots = nslots;
    const size_t smem = smem_bytes(M, p.nbp, nslots, p.rowbytes);
    int64_t grid = f.sm_count;
    const int64_t by_rows = (N + kConsumerWarps - 1) / kConsumerWarps;
    if (by_rows < grid) grid = by_rows > 0 ? by_rows : 1;
#define TN_GEMV_CASE(MT)                                                                   \
    if (M <= MT)                                                                           \
        return staged ? launch_variant<MT, true>(p, (int)grid, smem, stream)               \
                      : launch_variant<MT, false>(p, (int)grid, smem, stream);
    TN_GEMV_CASE(1)
    TN_GEMV_CASE(2)
    TN_GEMV_CASE(4)
    TN_GEMV_CASE(8)
    TN_GEMV_CASE(16)
#undef TN_GEMV_CASE
    return set_error(TN_ERR_NOT_IMPLEMENTED, std::string(op) + ": internal: GEMV called with M > 16");
}

}  // namespace tn
