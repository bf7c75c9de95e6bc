// sdpa_simt.cu -- flash attention on the FP32 pipes, for the prefill cases the
// tcgen05 kernel does not take: float32 inputs (whose products must stay f32:
// the reference computes q k^T in f32, aten.rs:10327-10360, and a tf32 or bf16
// tensor-core product would not meet its error), head dimension 64, an
// additive attn_mask, or q/k/v whose strides TMA cannot describe.
//
// One CTA = 64 query rows of one (batch, query head); 256 threads. Per 64-key
// tile: K and V rows are read (any strides; f16/bf16 widened exactly) and
// stored transposed-for-broadcast in shared memory; every thread computes a
// 4 x 4 block of S = Q K^T (scale, upper-left causal, key range, + mask), the
// online softmax keeps a running max and sum per row in f32, and each thread
// accumulates a 4-row x (D/16)-column block of O = P V. GQA by indexing.
#include <type_traits>

#include "sdpa_common.cuh"

namespace tn {
namespace {

constexpr int SM_ROWS = 64, SM_KEYS = 64, SM_THREADS = 256;
constexpr int PAD = 68;  // row stride (floats) of the transposed tiles and of P: float4-aligned, few bank conflicts

// Four consecutive elements widened to f32 (p 8-byte aligned for 16-bit types,
// 16-byte aligned for f32).
template <typename T>
__device__ __forceinline__ void load4(const T *p, float (&v)[4]) {
    if constexpr (std::is_same<T, float>::value) {
        const float4 x = *reinterpret_cast<const float4 *>(p);
        v[0] = x.x, v[1] = x.y, v[2] = x.z, v[3] = x.w;
    } else {
        const uint2 x = *reinterpret_cast<const uint2 *>(p);
        const uint32_t w[4] = {x.x & 0xffffu, x.x >> 16, x.y & 0xffffu, x.y >> 16};
#pragma unroll
        for (int i = 0; i < 4; ++i)
            v[i] = std::is_same<T, __nv_bfloat16>::value ? __uint_as_float(w[i] << 16) : half_bits_to_f32(w[i]);
    }
}

template <typename T, int D>
__global__ void __launch_bounds__(SM_THREADS) sdpa_simt_kernel(const SdpaParams p) {
    constexpr int DC = D / 16;  // output dims per thread
    extern __shared__ __align__(16) float sm[];
    float *Qt = sm;                     // [D][PAD] queries, transposed
    float *Kt = Qt + D * PAD;           // [D][PAD] keys, transposed
    float *Vs = Kt + D * PAD;           // [64 keys][D] values
    float *P = Vs + SM_KEYS * D;        // [64 rows][PAD] scores -> probabilities
    float *rowstat = P + SM_ROWS * PAD; // [64] alpha of this tile, then l

    const int tid = threadIdx.x;
    const int qt = blockIdx.x, hq = blockIdx.y, b = blockIdx.z;
    const int hk = hq / p.rep, q0 = qt * SM_ROWS;
    pdl_launch_dependents();
    pdl_wait();

    const T *qb = static_cast<const T *>(p.q) + b * p.qs[0] + hq * p.qs[1];
    const T *kb = static_cast<const T *>(p.k) + b * p.ks[0] + hk * p.ks[1];
    const T *vb = static_cast<const T *>(p.v) + b * p.vs[0] + hk * p.vs[1];
    // q may have any strides: element loads, row index fastest so the
    // transposed stores do not conflict.
    for (int idx = tid; idx < SM_ROWS * D; idx += SM_THREADS) {
        const int r = idx % SM_ROWS, d = idx / SM_ROWS;
        Qt[d * PAD + r] = (q0 + r < p.L) ? to_f32<T>(qb[(int64_t)(q0 + r) * p.qs[2] + d]) : 0.0f;
    }

    // QK and PV ownership: rows 4*(tid/16).., keys 4*(tid%16).. / dims DC*(tid%16)..
    const int ri = (tid >> 4) * 4, kj = (tid & 15) * 4, pd = (tid & 15) * DC;
    // softmax ownership: row tid/4, keys 16*(tid%4)..
    const int sr = tid >> 2, sc = (tid & 3) * 16;
    float o[4][DC];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int e = 0; e < DC; ++e) o[i][e] = 0.0f;
    float m_run = -INFINITY, l_run = 0.0f;  // row sr (each of its 4 threads keeps a copy)

    const int last_key = p.causal ? min(q0 + SM_ROWS - 1, p.S - 1) : p.S - 1;
    const int ntiles = last_key / SM_KEYS + 1;
    for (int j = 0; j < ntiles; ++j) {
        const int t0 = j * SM_KEYS;
        __syncthreads();  // previous tile's K, V, P fully used
        // K: four consecutive dims of one key per thread (16-byte aligned rows),
        // key index fastest; V: row-major, dims fastest.
        for (int idx = tid; idx < SM_KEYS * (D / 4); idx += SM_THREADS) {
            const int r = idx % SM_KEYS, d4 = (idx / SM_KEYS) * 4;
            float v4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            if (t0 + r < p.S) load4<T>(kb + (int64_t)(t0 + r) * p.ks[2] + d4, v4);
#pragma unroll
            for (int e = 0; e < 4; ++e) Kt[(d4 + e) * PAD + r] = v4[e];
        }
        for (int idx = tid; idx < SM_KEYS * (D / 4); idx += SM_THREADS) {
            const int r = idx / (D / 4), d4 = (idx % (D / 4)) * 4;
            float v4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            if (t0 + r < p.S) load4<T>(vb + (int64_t)(t0 + r) * p.vs[2] + d4, v4);
            *reinterpret_cast<float4 *>(Vs + r * D + d4) = make_float4(v4[0], v4[1], v4[2], v4[3]);
        }
        __syncthreads();
        // ---- S block
        float s[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int k = 0; k < 4; ++k) s[i][k] = 0.0f;
#pragma unroll 8
        for (int d = 0; d < D; ++d) {
            const float4 qv = *reinterpret_cast<const float4 *>(Qt + d * PAD + ri);
            const float4 kv = *reinterpret_cast<const float4 *>(Kt + d * PAD + kj);
            const float qa[4] = {qv.x, qv.y, qv.z, qv.w}, ka[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int k = 0; k < 4; ++k) s[i][k] = fmaf(qa[i], ka[k], s[i][k]);
        }
        // scale, masks (the reference's order: s*scale + (-inf | 0.0), then + mask)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int row = q0 + ri + i;
            float w[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int key = t0 + kj + k;
                float v = s[i][k] * p.scale;
                const bool masked = key >= p.S || (p.causal && key > row);
                v = masked ? -INFINITY : v + 0.0f;
                if (p.mask && key < p.S && row < p.L) {
                    const int64_t mi = b * p.ms[0] + hq * p.ms[1] + (int64_t)row * p.ms[2] + (int64_t)key * p.ms[3];
                    const float mv = p.mask_dtype == TN_F32 ? static_cast<const float *>(p.mask)[mi]
                                                            : to_f32<T>(static_cast<const T *>(p.mask)[mi]);
                    v = v + mv;
                }
                w[k] = v;
            }
            *reinterpret_cast<float4 *>(P + (ri + i) * PAD + kj) = make_float4(w[0], w[1], w[2], w[3]);
        }
        __syncthreads();
        // ---- online softmax for row sr over this tile (4 threads per row)
        {
            float *prow = P + sr * PAD + sc;
            float mx = -INFINITY;
#pragma unroll
            for (int c = 0; c < 16; ++c) mx = fmaxf(mx, prow[c]);
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            const float m_new = fmaxf(m_run, mx);
            float sum = 0.0f;
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                const float e = (m_new == -INFINITY) ? 0.0f : expf(prow[c] - m_new);
                prow[c] = e;
                sum += e;
            }
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            const float alpha = (m_run == -INFINITY) ? 0.0f : expf(m_run - m_new);
            l_run = l_run * alpha + sum;
            m_run = m_new;
            if ((tid & 3) == 0) rowstat[sr] = alpha;
        }
        __syncthreads();
        // ---- O = O * alpha + P V
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float a = rowstat[ri + i];
#pragma unroll
            for (int e = 0; e < DC; ++e) o[i][e] *= a;
        }
#pragma unroll 2
        for (int k = 0; k < SM_KEYS; k += 4) {
            float pa[4][4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float4 x = *reinterpret_cast<const float4 *>(P + (ri + i) * PAD + k);
                pa[i][0] = x.x, pa[i][1] = x.y, pa[i][2] = x.z, pa[i][3] = x.w;
            }
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                float vv[DC];
#pragma unroll
                for (int e = 0; e < DC; e += 4) {
                    const float4 v4 = *reinterpret_cast<const float4 *>(Vs + (k + kk) * D + pd + e);
                    vv[e] = v4.x, vv[e + 1] = v4.y, vv[e + 2] = v4.z, vv[e + 3] = v4.w;
                }
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int e = 0; e < DC; ++e) o[i][e] = fmaf(pa[i][kk], vv[e], o[i][e]);
            }
        }
    }
    // ---- out = O / l (the row's l from its softmax owners), lse = m + log l
    __syncthreads();
    if ((tid & 3) == 0) {
        rowstat[sr] = l_run;
        // a row that sees no key (every score -inf) answers zeros and lse 0,
        // as upstream and the reference's blocked kernel do (flash.rs:758-776)
        if (p.lse && q0 + sr < p.L)
            p.lse[((int64_t)b * p.Hq + hq) * p.L + q0 + sr] = (l_run == 0.0f) ? 0.0f : logf(l_run) + m_run;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int row = q0 + ri + i;
        if (row >= p.L) continue;
        const float inv = (rowstat[ri + i] == 0.0f) ? 0.0f : 1.0f / rowstat[ri + i];
        const int64_t oi = (((int64_t)b * p.Hq + hq) * p.L + row) * D + pd;
#pragma unroll
        for (int e = 0; e < DC; ++e) {
            const float v = o[i][e] * inv;
            if constexpr (std::is_same<T, float>::value)
                static_cast<float *>(p.out)[oi + e] = v;
            else if constexpr (std::is_same<T, __nv_bfloat16>::value)
                static_cast<__nv_bfloat16 *>(p.out)[oi + e] = __float2bfloat16_rn(v);
            else
                static_cast<__half *>(p.out)[oi + e] = __float2half_rn(v);
        }
    }
}

template <typename T, int D>
int launch_simt_typed(const SdpaParams &p, cudaStream_t stream) {
    const size_t smem = (size_t)(2 * D * PAD + SM_KEYS * D + SM_ROWS * PAD + SM_ROWS) * 4;
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        int st = check_cuda(cudaFuncSetAttribute(sdpa_simt_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)smem),
                            "aten._scaled_dot_product_flash_attention_for_cpu", "cudaFuncSetAttribute");
        if (st) return st;
        configured[dev] = 1;
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((p.L + SM_ROWS - 1) / SM_ROWS), (unsigned)p.Hq, (unsigned)p.B);
    cfg.blockDim = dim3(SM_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int st = check_cuda(cudaLaunchKernelEx(&cfg, sdpa_simt_kernel<T, D>, p),
                        "aten._scaled_dot_product_flash_attention_for_cpu", "cudaLaunchKernelEx (prefill, fp32 pipes)");
    if (st) return st;
    __atomic_fetch_add(&counters().sdpa_prefill_launches, 1ull, __ATOMIC_RELAXED);
    return TN_OK;
}

}  // namespace

int launch_sdpa_prefill_simt(const SdpaParams &p, int dtype, cudaStream_t stream) {
    if (p.D == 128) {
        if (dtype == TN_F32) return launch_simt_typed<float, 128>(p, stream);
        if (dtype == TN_BF16) return launch_simt_typed<__nv_bfloat16, 128>(p, stream);
        return launch_simt_typed<__half, 128>(p, stream);
    }
    if (dtype == TN_F32) return launch_simt_typed<float, 64>(p, stream);
    if (dtype == TN_BF16) return launch_simt_typed<__nv_bfloat16, 64>(p, stream);
    return launch_simt_typed<__half, 64>(p, stream);
}

}  // namespace tn
