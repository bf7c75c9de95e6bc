// sdpa_decode.cu -- split-KV ("flash-decoding") attention for few query rows
// (decode: L = 1 against a KV cache), all of a KV head's query heads together.
//
// Grid (splits, row_groups * Hkv, B). A CTA owns one KV head of one batch row,
// up to RMAX query rows of that head's group (the rep = Hq/Hkv query heads that
// read it, times L positions) and one contiguous range of keys. K and V are read
// from HBM exactly once per (b, kv head): GQA is an index, not a copy
// (repeat_kv_heads, aten.rs:17106-17130, materialises the copy instead).
//
// Per tile of 32 keys: cp.async brings K and V rows (any t stride, so a
// [B, Hkv, cap, D] cache narrowed to S keys is read in place) into a 3-stage
// ring; scores s = (q . k) * scale (+ causal -inf, upper-left, + additive mask);
// online softmax (running max m, running sum l, rescale by exp(m_old - m_new));
// o += p * v. Arithmetic in f32 for every input dtype, as the reference widens
// f16/bf16 to f32 (aten.rs:10202-10211). A split writes its unnormalised o and
// (m, l); the combine kernel merges splits, normalises, narrows to the input
// dtype and writes lse = m + log(l).
#include <type_traits>

#include "sdpa_common.cuh"

namespace tn {
namespace {

constexpr int kThreads = 128;
constexpr int TK = 32;      // keys per tile
constexpr int NSTAGE = 3;   // cp.async ring depth
constexpr int RMAX = 8;     // query rows per CTA

template <typename T>
struct Elem;
template <>
struct Elem<float> {
    static constexpr int per16 = 4;  // elements per 16-byte chunk
    __device__ static void unpack(const int4 &c, float *o) {
        o[0] = __int_as_float(c.x);
        o[1] = __int_as_float(c.y);
        o[2] = __int_as_float(c.z);
        o[3] = __int_as_float(c.w);
    }
};
template <>
struct Elem<__nv_bfloat16> {
    static constexpr int per16 = 8;
    __device__ static void unpack(const int4 &c, float *o) {
        const uint32_t w[4] = {(uint32_t)c.x, (uint32_t)c.y, (uint32_t)c.z, (uint32_t)c.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            o[2 * i] = __uint_as_float(w[i] << 16);
            o[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
    }
};
template <>
struct Elem<__half> {
    static constexpr int per16 = 8;
    __device__ static void unpack(const int4 &c, float *o) {
        const uint32_t w[4] = {(uint32_t)c.x, (uint32_t)c.y, (uint32_t)c.z, (uint32_t)c.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
            o[2 * i] = f.x;
            o[2 * i + 1] = f.y;
        }
    }
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ float load_mask(const SdpaParams &p, int b, int hq, int l, int t) {
    const int64_t i = b * p.ms[0] + hq * p.ms[1] + l * p.ms[2] + t * p.ms[3];
    switch (p.mask_dtype) {
    case TN_F32: return static_cast<const float *>(p.mask)[i];
    case TN_BF16: return __bfloat162float(static_cast<const __nv_bfloat16 *>(p.mask)[i]);
    default: return __half2float(static_cast<const __half *>(p.mask)[i]);
    }
}

template <typename T, int D>
struct Layout {
    static constexpr int CPR = D * (int)sizeof(T) / 16;  // 16-byte chunks per K/V row
    static constexpr int EPC = Elem<T>::per16;           // elements per chunk
    static constexpr int TILE_BYTES = TK * D * (int)sizeof(T);
    // QK: thread (key j = tid / 4, part p = tid % 4) reads chunks p, p+4, ...
    static constexpr int QK_CHUNKS = CPR / 4;
    // PV: thread (chunk c = tid % CPR, key group g = tid / CPR) handles keys j = g, g + G, ...
    static constexpr int PV_GROUPS = kThreads / CPR;
};

// Physical 16-byte chunk of logical chunk c in K row j: rows j and j+1 share a
// quarter-warp in the QK loop, so odd rows swap the two halves of each 128-byte
// line and the eight lanes of a quarter-warp hit eight different bank groups.
__device__ __forceinline__ int kswz(int j, int c) { return c ^ ((j & 1) << 2); }

template <typename T, int D>
__global__ void __launch_bounds__(kThreads) sdpa_decode_kernel(const SdpaParams p) {
    using LY = Layout<T, D>;
    extern __shared__ __align__(128) uint8_t smem[];
    float *qsm = reinterpret_cast<float *>(smem);          // [RMAX][D] f32 queries
    float *ssm = qsm + RMAX * D;                            // [RMAX][TK] scores -> probabilities
    float *stat = ssm + RMAX * TK;                          // m[RMAX], l[RMAX], alpha[RMAX]
    uint8_t *ring = reinterpret_cast<uint8_t *>(stat + 4 * RMAX);  // NSTAGE x (K tile, V tile)
    float *osm = reinterpret_cast<float *>(ring);  // [PV_GROUPS][RMAX][D] partial o, after the ring is drained
    const uint32_t ring_u32 = smem_u32(ring);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int split = blockIdx.x, rg = blockIdx.y % p.row_groups, kvh = blockIdx.y / p.row_groups, b = blockIdx.z;
    const int R = min(p.rows, p.rep * p.L - rg * p.rows);  // query rows of this CTA

    pdl_launch_dependents();
    pdl_wait();
    // The key count may live on the device (a decode loop replayed as one CUDA
    // graph while the cache grows); splits were planned for the capacity p.S.
    const int S = p.S_dev ? min(*p.S_dev + p.S_add, p.S) : p.S;
    const int t0 = split * p.keys_per_split, t1 = min(S, t0 + p.keys_per_split);
    const int ntiles = t1 > t0 ? (t1 - t0 + TK - 1) / TK : 0;

    // ---- queries (widened to f32) and row state
    for (int idx = tid; idx < RMAX * D; idx += kThreads) {
        const int r = idx / D, d = idx % D;
        float v = 0.0f;
        if (r < R) {
            const int gr = rg * p.rows + r, l = gr / p.rep, hq = kvh * p.rep + gr % p.rep;
            v = to_f32<T>(static_cast<const T *>(p.q)[b * p.qs[0] + hq * p.qs[1] + l * p.qs[2] + d]);
        }
        qsm[idx] = v;
    }
    if (tid < RMAX) {
        stat[tid] = -INFINITY;       // m
        stat[RMAX + tid] = 0.0f;     // l
        stat[2 * RMAX + tid] = 1.0f; // alpha
    }

    const T *kbase = static_cast<const T *>(p.k) + b * p.ks[0] + kvh * p.ks[1];
    const T *vbase = static_cast<const T *>(p.v) + b * p.vs[0] + kvh * p.vs[1];
    auto issue_tile = [&](int tile, int stage) {
        const uint32_t kst = ring_u32 + stage * 2 * LY::TILE_BYTES, vst = kst + LY::TILE_BYTES;
        for (int idx = tid; idx < TK * LY::CPR; idx += kThreads) {
            const int j = idx / LY::CPR, c = idx % LY::CPR;
            const int t = t0 + tile * TK + j;
            const bool ok = t < t1;
            const int ts = ok ? t : t0;
            cp_async16(kst + (j * LY::CPR + kswz(j, c)) * 16, kbase + ts * p.ks[2] + c * LY::EPC, ok ? 16u : 0u);
            cp_async16(vst + (j * LY::CPR + c) * 16, vbase + ts * p.vs[2] + c * LY::EPC, ok ? 16u : 0u);
        }
    };
#pragma unroll
    for (int s = 0; s < NSTAGE - 1; ++s) {
        if (s < ntiles) issue_tile(s, s);
        cp_async_commit();
    }

    // PV ownership: chunk pc of every row, keys pg, pg + G, ...
    const int pc = tid % LY::CPR, pg = tid / LY::CPR;
    float o[RMAX][LY::EPC];
#pragma unroll
    for (int r = 0; r < RMAX; ++r)
#pragma unroll
        for (int e = 0; e < LY::EPC; ++e) o[r][e] = 0.0f;

    const int qk_j = tid >> 2, qk_p = tid & 3;
    for (int tile = 0; tile < ntiles; ++tile) {
        if (tile + NSTAGE - 1 < ntiles) issue_tile(tile + NSTAGE - 1, (tile + NSTAGE - 1) % NSTAGE);
        cp_async_commit();
        cp_async_wait<NSTAGE - 1>();
        __syncthreads();
        const int stage = tile % NSTAGE;
        const uint8_t *kst = ring + stage * 2 * LY::TILE_BYTES;
        const uint8_t *vst = kst + LY::TILE_BYTES;

        // ---- scores: thread (qk_j, qk_p) dots its quarter of key qk_j with every row
        {
            float acc[RMAX];
#pragma unroll
            for (int r = 0; r < RMAX; ++r) acc[r] = 0.0f;
#pragma unroll
            for (int i = 0; i < LY::QK_CHUNKS; ++i) {
                const int c = qk_p + 4 * i;
                const int4 raw = *reinterpret_cast<const int4 *>(kst + (qk_j * LY::CPR + kswz(qk_j, c)) * 16);
                float kv[LY::EPC];
                Elem<T>::unpack(raw, kv);
#pragma unroll
                for (int r = 0; r < RMAX; ++r) {
                    if (r < R) {
                        const float *qr = qsm + r * D + c * LY::EPC;
#pragma unroll
                        for (int e = 0; e < LY::EPC; ++e) acc[r] = fmaf(qr[e], kv[e], acc[r]);
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < RMAX; ++r) {
                acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], 1);
                acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], 2);
            }
            if (qk_p == 0) {
                const int t = t0 + tile * TK + qk_j;
#pragma unroll
                for (int r = 0; r < RMAX; ++r) {
                    if (r < R) {
                        const int gr = rg * p.rows + r, l = gr / p.rep, hq = kvh * p.rep + gr % p.rep;
                        float s = acc[r] * p.scale;
                        const bool masked = t >= t1 || (p.causal && t > l);
                        s = masked ? -INFINITY : s + 0.0f;
                        if (p.mask && t < t1) s = s + load_mask(p, b, hq, l, t);
                        ssm[r * TK + qk_j] = s;
                    }
                }
            }
        }
        __syncthreads();

        // ---- online softmax: warp w handles rows w, w + 4; lane = key
        for (int r = warp; r < R; r += 4) {
            const float s = ssm[r * TK + lane];
            float mx = s;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float m_old = stat[r], m_new = fmaxf(m_old, mx);
            // all keys so far masked: keep everything at zero weight
            const float pj = (m_new == -INFINITY) ? 0.0f : expf(s - m_new);
            float sum = pj;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
            ssm[r * TK + lane] = pj;
            if (lane == 0) {
                const float alpha = (m_old == -INFINITY) ? 0.0f : expf(m_old - m_new);
                stat[r] = m_new;
                stat[RMAX + r] = stat[RMAX + r] * alpha + sum;
                stat[2 * RMAX + r] = alpha;
            }
        }
        __syncthreads();

        // ---- o = o * alpha + p v
#pragma unroll
        for (int r = 0; r < RMAX; ++r) {
            if (r < R) {
                const float a = stat[2 * RMAX + r];
#pragma unroll
                for (int e = 0; e < LY::EPC; ++e) o[r][e] *= a;
            }
        }
        for (int j = pg; j < TK; j += LY::PV_GROUPS) {
            const int4 raw = *reinterpret_cast<const int4 *>(vst + (j * LY::CPR + pc) * 16);
            float vv[LY::EPC];
            Elem<T>::unpack(raw, vv);
#pragma unroll
            for (int r = 0; r < RMAX; ++r) {
                if (r < R) {
                    const float pr = ssm[r * TK + j];
#pragma unroll
                    for (int e = 0; e < LY::EPC; ++e) o[r][e] = fmaf(pr, vv[e], o[r][e]);
                }
            }
        }
        __syncthreads();  // the stage and the probabilities are reused next tile
    }
    cp_async_wait<0>();
    __syncthreads();

    // ---- combine the key groups of this CTA, write the split's partial
#pragma unroll
    for (int r = 0; r < RMAX; ++r)
#pragma unroll
        for (int e = 0; e < LY::EPC; ++e) osm[(pg * RMAX + r) * D + pc * LY::EPC + e] = o[r][e];
    __syncthreads();
    for (int idx = tid; idx < R * D; idx += kThreads) {
        const int r = idx / D, d = idx % D;
        float acc = 0.0f;
        for (int g = 0; g < LY::PV_GROUPS; ++g) acc += osm[(g * RMAX + r) * D + d];
        const int gr = rg * p.rows + r, l = gr / p.rep, hq = kvh * p.rep + gr % p.rep;
        const int64_t row = ((int64_t)b * p.Hq + hq) * p.L + l;
        p.part_o[(row * p.splits + split) * D + d] = acc;
        if (d == 0) {
            p.part_ml[(row * p.splits + split) * 2 + 0] = stat[r];
            p.part_ml[(row * p.splits + split) * 2 + 1] = stat[RMAX + r];
        }
    }
}

// Merge the splits of one output row: M = max m_s, w_s = exp(m_s - M),
// out = sum w_s o_s / sum w_s l_s, lse = M + log(sum w_s l_s). One warp per row.
template <typename T, int D>
__global__ void __launch_bounds__(128) sdpa_combine_kernel(const SdpaParams p) {
    pdl_launch_dependents();
    pdl_wait();
    const int64_t rows = (int64_t)p.B * p.Hq * p.L;
    const int64_t row = blockIdx.x * 4 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float *ml = p.part_ml + row * p.splits * 2;
    float M = -INFINITY;
    for (int s = 0; s < p.splits; ++s) M = fmaxf(M, ml[2 * s]);
    float den = 0.0f;
    constexpr int PER = D / 32;
    float acc[PER];
#pragma unroll
    for (int e = 0; e < PER; ++e) acc[e] = 0.0f;
    for (int s = 0; s < p.splits; ++s) {
        const float m = ml[2 * s];
        const float w = (m == -INFINITY) ? 0.0f : expf(m - M);
        den = fmaf(w, ml[2 * s + 1], den);
        const float *os = p.part_o + (row * p.splits + s) * D;
#pragma unroll
        for (int e = 0; e < PER; ++e) acc[e] = fmaf(w, os[lane + 32 * e], acc[e]);
    }
    // softmax divides each weight by the sum (aten.rs:10406); here the sum is
    // applied once to the accumulated row
    const float inv_den = 1.0f / den;
#pragma unroll
    for (int e = 0; e < PER; ++e) {
        const float v = acc[e] * inv_den;
        const int64_t oi = row * D + lane + 32 * e;
        if (std::is_same<T, float>::value)
            static_cast<float *>(p.out)[oi] = v;
        else if (std::is_same<T, __nv_bfloat16>::value)
            static_cast<__nv_bfloat16 *>(p.out)[oi] = __float2bfloat16_rn(v);
        else
            static_cast<__half *>(p.out)[oi] = __float2half_rn(v);
    }
    if (lane == 0 && p.lse) p.lse[row] = logf(den) + M;
}

template <typename T, int D>
size_t decode_smem() {
    using LY = Layout<T, D>;
    const size_t ring = (size_t)NSTAGE * 2 * LY::TILE_BYTES, o = (size_t)LY::PV_GROUPS * RMAX * D * 4;
    return (size_t)(RMAX * D + RMAX * TK + 4 * RMAX) * 4 + (ring > o ? ring : o) + 128;
}

template <typename T, int D>
int launch_typed(const SdpaParams &p, cudaStream_t stream) {
    const size_t smem = decode_smem<T, D>();
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        int st = check_cuda(cudaFuncSetAttribute(sdpa_decode_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)smem),
                            "aten._scaled_dot_product_flash_attention_for_cpu", "cudaFuncSetAttribute");
        if (st) return st;
        configured[dev] = 1;
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.splits, p.row_groups * p.Hkv, p.B);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int st = check_cuda(cudaLaunchKernelEx(&cfg, sdpa_decode_kernel<T, D>, p),
                        "aten._scaled_dot_product_flash_attention_for_cpu", "cudaLaunchKernelEx (decode)");
    if (st) return st;
    const int64_t rows = (int64_t)p.B * p.Hq * p.L;
    cudaLaunchConfig_t cfg2 = cfg;
    cfg2.gridDim = dim3((unsigned)((rows + 3) / 4));
    cfg2.blockDim = dim3(128);
    cfg2.dynamicSmemBytes = 0;
    st = check_cuda(cudaLaunchKernelEx(&cfg2, sdpa_combine_kernel<T, D>, p),
                    "aten._scaled_dot_product_flash_attention_for_cpu", "cudaLaunchKernelEx (combine)");
    if (st) return st;
    __atomic_fetch_add(&counters().sdpa_decode_launches, 1ull, __ATOMIC_RELAXED);
    return TN_OK;
}

}  // namespace

int plan_sdpa_decode(SdpaParams &p, int sm_count) {
    const int R = p.rep * p.L;
    p.rows = R < RMAX ? R : RMAX;
    p.row_groups = (R + p.rows - 1) / p.rows;
    const int64_t base = (int64_t)p.B * p.Hkv * p.row_groups;
    // enough CTAs for ~4 per SM, but no split shorter than 4 tiles
    int64_t want = (4LL * sm_count + base - 1) / base;
    const int64_t max_splits = (p.S + 4 * TK - 1) / (4 * TK);
    if (want > max_splits) want = max_splits;
    if (want < 1) want = 1;
    int kps = (int)((p.S + want - 1) / want);
    kps = (kps + TK - 1) / TK * TK;
    p.keys_per_split = kps;
    p.splits = (p.S + kps - 1) / kps;
    return TN_OK;
}

size_t sdpa_decode_workspace(const SdpaParams &p) {
    const int64_t rows = (int64_t)p.B * p.Hq * p.L;
    return (size_t)rows * p.splits * (p.D + 2) * 4 + 256;
}

int launch_sdpa_decode(const SdpaParams &p, int dtype, cudaStream_t stream) {
    if (p.D == 128) {
        if (dtype == TN_F32) return launch_typed<float, 128>(p, stream);
        if (dtype == TN_BF16) return launch_typed<__nv_bfloat16, 128>(p, stream);
        return launch_typed<__half, 128>(p, stream);
    }
    if (dtype == TN_F32) return launch_typed<float, 64>(p, stream);
    if (dtype == TN_BF16) return launch_typed<__nv_bfloat16, 64>(p, stream);
    return launch_typed<__half, 64>(p, stream);
}

}  // namespace tn
