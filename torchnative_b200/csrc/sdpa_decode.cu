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

__device__ __forceinline__ float bfr16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

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

// After a CTA wrote its split's partial: the last CTA of its (b, kv head, row
// group) to finish merges all splits of these rows, in split order:
// M = max m_s, out = sum e^(m_s - M) o_s / sum e^(m_s - M) l_s, lse = M + log(den).
// `scratch` is `scratch_bytes` of drained shared memory. When the rows'
// partial outputs fit there next to the merge weights, one bulk copy per row
// brings them in (a single memory latency for the whole merge); otherwise
// each thread streams its dimensions through L2.
template <typename T, int D>
__device__ __forceinline__ void merge_if_last(const SdpaParams &p, int b, int kvh, int rg, int R, int tid,
                                              float *scratch, size_t scratch_bytes) {
    __shared__ int last;
    __shared__ __align__(8) uint64_t staged_bar;
    // One thread publishes the CTA's partial: the barrier orders every
    // thread's stores before its release fence and ticket; the last CTA's
    // acquire fence (same thread) orders the other splits' partials before the
    // barrier that releases its readers.
    __syncthreads();
    int *counter = p.counters + ((int64_t)b * p.Hkv + kvh) * p.row_groups + rg;
    if (tid == 0) {
        __threadfence();
        last = (atomicAdd(counter, 1) == p.splits - 1);
        if (last) __threadfence();
    }
    __syncthreads();
    if (!last) return;
    float *wsm = scratch;                 // [R][splits] m_s, then weights e^(m_s - M)
    float *lsp = wsm + RMAX * p.splits;   // [R][splits] l_s
    float *lsm = lsp + RMAX * p.splits;   // [R] sum of weighted l_s
    const size_t ml_bytes = ((size_t)(2 * RMAX * p.splits + RMAX) * 4 + 127) & ~size_t(127);
    const size_t row_bytes = (size_t)p.splits * D * 4;
    float *pos_ = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(scratch) + ml_bytes);
    const bool staged = ml_bytes + (size_t)R * row_bytes <= scratch_bytes;
    const int64_t row0 = ((int64_t)b * p.Hq + kvh * p.rep) * p.L;  // R consecutive rows (L = 1 or one head)
    const bool contiguous = p.L == 1 && rg == 0;
    bool have = false;
    if (staged && contiguous) {
        if (tid == 0) {
            mbar_init(&staged_bar, 1);
            fence_mbar_init();
            // the partials were written through the generic proxy by other CTAs
            asm volatile("fence.proxy.async.global;" ::: "memory");
            mbar_arrive_expect_tx(&staged_bar, (uint32_t)(R * row_bytes));
            bulk_g2s(pos_, p.part_o + row0 * p.splits * D, (uint32_t)(R * row_bytes), &staged_bar);
        }
        have = true;
    }
    for (int idx = tid; idx < R * p.splits; idx += kThreads) {
        const int r = idx / p.splits, sp = idx % p.splits;
        const int64_t row = ((int64_t)b * p.Hq + kvh * p.rep + r) * p.L;
        const float2 ml = __ldcg(reinterpret_cast<const float2 *>(p.part_ml + (row * p.splits + sp) * 2));
        wsm[idx] = ml.x;
        lsp[idx] = ml.y;
    }
    __syncthreads();
    // one warp per row: the splits' maximum, weights and weighted sum across lanes
    {
        const int warp = tid >> 5, lane = tid & 31;
        for (int r = warp; r < R; r += kThreads / 32) {
            const int64_t row = ((int64_t)b * p.Hq + kvh * p.rep + r) * p.L;
            float M = -INFINITY;
            for (int sp = lane; sp < p.splits; sp += 32) M = fmaxf(M, wsm[r * p.splits + sp]);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
            float den = 0.0f;
            for (int sp = lane; sp < p.splits; sp += 32) {
                const float m = wsm[r * p.splits + sp];
                const float w = (m == -INFINITY) ? 0.0f : expf(m - M);
                wsm[r * p.splits + sp] = w;
                den = fmaf(w, lsp[r * p.splits + sp], den);
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) den += __shfl_xor_sync(0xffffffffu, den, off);
            if (lane == 0) {
                lsm[r] = den;
                // no key seen by any split: zeros and lse 0 (flash.rs:758-776)
                if (p.lse) p.lse[row] = (den == 0.0f) ? 0.0f : logf(den) + M;
            }
        }
    }
    bool ok = true;
    if (have) ok = mbar_wait(&staged_bar, 0);
    if (have && !ok) record_device_error(p.err, DEV_ERR_WAIT_FULL);
    __syncthreads();
    for (int idx = tid; idx < R * (D / 4); idx += kThreads) {
        const int r = idx / (D / 4), d4 = idx % (D / 4);
        const int64_t row = ((int64_t)b * p.Hq + kvh * p.rep + r) * p.L;
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (have) {
            const float4 *po = reinterpret_cast<const float4 *>(pos_ + (size_t)r * p.splits * D) + d4;
#pragma unroll 8
            for (int sp = 0; sp < p.splits; ++sp) {
                const float w = wsm[r * p.splits + sp];
                const float4 o = po[(int64_t)sp * (D / 4)];
                acc.x = fmaf(w, o.x, acc.x);
                acc.y = fmaf(w, o.y, acc.y);
                acc.z = fmaf(w, o.z, acc.z);
                acc.w = fmaf(w, o.w, acc.w);
            }
        } else {
            const float4 *po = reinterpret_cast<const float4 *>(p.part_o + row * p.splits * D) + d4;
#pragma unroll 8
            for (int sp = 0; sp < p.splits; ++sp) {
                const float w = wsm[r * p.splits + sp];
                const float4 o = __ldcg(po + (int64_t)sp * (D / 4));
                acc.x = fmaf(w, o.x, acc.x);
                acc.y = fmaf(w, o.y, acc.y);
                acc.z = fmaf(w, o.z, acc.z);
                acc.w = fmaf(w, o.w, acc.w);
            }
        }
        const float inv = (lsm[r] == 0.0f) ? 0.0f : 1.0f / lsm[r];
        const float v4[4] = {acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int64_t oi = row * D + d4 * 4 + e;
            if (std::is_same<T, float>::value)
                static_cast<float *>(p.out)[oi] = v4[e];
            else if (std::is_same<T, __nv_bfloat16>::value)
                static_cast<__nv_bfloat16 *>(p.out)[oi] = __float2bfloat16_rn(v4[e]);
            else
                static_cast<__half *>(p.out)[oi] = __float2half_rn(v4[e]);
        }
        if constexpr (std::is_same<T, __nv_bfloat16>::value) {
            if (p.q8_codes) {
                // Planar Q8_0 of the bf16 output (k_quants.rs:676-706): the 8 lanes
                // holding one 32-element block (consecutive d4) share its maximum
                // and code sum.
                const int lane = tid & 31;
                const unsigned gm = 0xffu << (lane & ~7);
                float q[4], amax = 0.0f;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    q[e] = __bfloat162float(__float2bfloat16_rn(v4[e]));
                    amax = fmaxf(amax, fabsf(q[e]));
                }
#pragma unroll
                for (int off = 1; off < 8; off <<= 1) amax = fmaxf(amax, __shfl_xor_sync(gm, amax, off));
                const float dq = __fdiv_rn(amax, 127.0f);
                const float id = (dq != 0.0f) ? __fdiv_rn(1.0f, dq) : 0.0f;
                uint32_t word = 0;
                int sum = 0;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float t = roundf(__fmul_rn(q[e], id));
                    const int c = !(t == t) ? 0 : (t <= -128.0f ? -128 : (t >= 127.0f ? 127 : __float2int_rz(t)));
                    sum += c;
                    word |= (uint32_t)(c & 0xff) << (8 * e);
                }
#pragma unroll
                for (int off = 1; off < 8; off <<= 1) sum += __shfl_xor_sync(gm, sum, off);
                const int hq = kvh * p.rep + r, K = p.Hq * D;
                const int64_t e0 = (int64_t)b * K + hq * D + d4 * 4;
                *reinterpret_cast<uint32_t *>(p.q8_codes + e0) = word;
                if ((lane & 7) == 0) {
                    p.q8_scales[e0 / 32] = __half2float(__float2half_rn(dq));
                    p.q8_offs[e0 / 32] = 12582912.0f + 8.0f * (float)sum;
                }
            }
        }
    }
    if (tid == 0) *counter = 0;
}

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
    if (p.qkv) {
        // Fused step: rotate q (rotate_half convention, cos/sin rounded to bf16
        // as transformers does) from the projection row; the CTA whose key
        // range holds slot S - 1 also appends the rotated k and v there.
        const int pos = S - 1, half = D / 2, W = (p.Hq + 2 * p.Hkv) * D;
        const __nv_bfloat16 *row = p.qkv + (int64_t)b * W;
        // cos/sin of inv_freq[i] * pos, rounded to bf16, once per CTA (in the
        // score scratch, which is not used before the first tile)
        float *cs = ssm, *sn_t = ssm + half;
        for (int i = tid; i < half; i += kThreads) {
            const float f = p.inv_freq[i] * (float)pos;
            cs[i] = bfr16(cosf(f));
            sn_t[i] = bfr16(sinf(f));
        }
        __syncthreads();
        for (int idx = tid; idx < RMAX * D; idx += kThreads) {
            const int r = idx / D, d = idx % D;
            float v = 0.0f;
            if (r < R) {
                const int hq = kvh * p.rep + r;
                const int i = d % half;
                const float c = cs[i], sn = sn_t[i];
                const float x1 = __bfloat162float(row[hq * D + i]), x2 = __bfloat162float(row[hq * D + i + half]);
                v = d < half ? bfr16(bfr16(x1 * c) + bfr16(-x2 * sn)) : bfr16(bfr16(x2 * c) + bfr16(x1 * sn));
            }
            qsm[idx] = v;
        }
        if (t0 <= pos && pos < t1 && rg == 0) {
            __nv_bfloat16 *kc = (__nv_bfloat16 *)p.k + b * p.ks[0] + kvh * p.ks[1] + (int64_t)pos * p.ks[2];
            __nv_bfloat16 *vc = (__nv_bfloat16 *)p.v + b * p.vs[0] + kvh * p.vs[1] + (int64_t)pos * p.vs[2];
            const __nv_bfloat16 *kr = row + (p.Hq + kvh) * D, *vr = row + (p.Hq + p.Hkv + kvh) * D;
            for (int i = tid; i < half; i += kThreads) {
                const float c = cs[i], sn = sn_t[i];
                const float x1 = __bfloat162float(kr[i]), x2 = __bfloat162float(kr[i + half]);
                kc[i] = __float2bfloat16_rn(bfr16(x1 * c) + bfr16(-x2 * sn));
                kc[i + half] = __float2bfloat16_rn(bfr16(x2 * c) + bfr16(x1 * sn));
                vc[i] = vr[i];
                vc[i + half] = vr[i + half];
            }
        }
        __syncthreads();  // the appended slot is written before any tile copy reads it
    } else {
        for (int idx = tid; idx < RMAX * D; idx += kThreads) {
            const int r = idx / D, d = idx % D;
            float v = 0.0f;
            if (r < R) {
                const int gr = rg * p.rows + r, l = gr / p.rep, hq = kvh * p.rep + gr % p.rep;
                v = to_f32<T>(static_cast<const T *>(p.q)[b * p.qs[0] + hq * p.qs[1] + l * p.qs[2] + d]);
            }
            qsm[idx] = v;
        }
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
    if (!p.counters) return;
    {
        const size_t ring_b = (size_t)NSTAGE * 2 * LY::TILE_BYTES, o_b = (size_t)LY::PV_GROUPS * RMAX * D * 4;
        merge_if_last<T, D>(p, b, kvh, rg, R, tid, reinterpret_cast<float *>(ring), ring_b > o_b ? ring_b : o_b);
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
    const float inv_den = (den == 0.0f) ? 0.0f : 1.0f / den;  // no key seen: zeros (flash.rs:758-776)
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
    if (lane == 0 && p.lse) p.lse[row] = (den == 0.0f) ? 0.0f : logf(den) + M;
}

// ---------------------------------------------------------------------------
// Tensor-core variant for bf16 / f16 (the decode path of the model): the same
// split-KV algorithm with QK^T and PV on mma.sync.m16n8k16 (f32 accumulate).
// The query rows of the CTA (rep heads of one KV head, <= 16) are the MMA's
// M = 16 rows; each of the 4 warps walks its own 16-key tiles through its own
// 3-stage cp.async ring with no CTA-wide barrier per tile (FlashAttention-2's
// register layout: the score fragment is re-used as the PV A fragment). The
// probabilities enter PV rounded to the input dtype; scores, the softmax and
// every sum stay f32. Warps merge their (m, l, o) in shared memory; the CTA
// writes the split's partial and the last CTA merges the splits, as above.
// ---------------------------------------------------------------------------

constexpr int TKM = 16;     // keys per warp tile
constexpr int NST = 3;      // per-warp ring depth
constexpr int MMA_WARPS = 4;

template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                        uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
    const __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&v);
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// Byte offset of 16-byte chunk c of row j in a [rows][D] 16-bit tile: chunks
// XOR-swizzled by the row's low 3 bits, so the 8 rows an ldmatrix phase reads
// at one column land in 8 different bank groups.
template <int D>
__device__ __forceinline__ uint32_t tile_off(int j, int c) {
    return (uint32_t)(j * (D * 2) + ((c ^ (j & 7)) * 16));
}

template <typename T, int D>
__global__ void __launch_bounds__(MMA_WARPS * 32) sdpa_decode_mma_kernel(const SdpaParams p) {
    constexpr int CPR = D * 2 / 16;                // 16-byte chunks per row
    constexpr int TILE = TKM * D * 2;              // bytes of one K (or V) tile
    constexpr int NT = D / 8;                      // output n-tiles
    constexpr int KS = D / 16;                     // k-steps of QK^T
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *qb = smem;                                            // [16][D] T, swizzled
    uint8_t *rings = smem + 16 * D * 2 + D * 4;                    // MMA_WARPS x NST x (K, V)
    float *cmb = reinterpret_cast<float *>(rings);                 // after the rings drain: warp merge

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t4 = lane & 3;
    const int split = blockIdx.x, rg = blockIdx.y % p.row_groups, kvh = blockIdx.y / p.row_groups, b = blockIdx.z;
    const int R = min(p.rows, p.rep * p.L - rg * p.rows);

    pdl_launch_dependents();
    pdl_wait();
    const int S = p.S_dev ? min(*p.S_dev + p.S_add, p.S) : p.S;
    const int t0 = split * p.keys_per_split, t1 = min(S, t0 + p.keys_per_split);
    const int pos = S - 1;
    // the one CTA per (b, kv head) whose keys include the appended slot writes it first
    const bool appends = p.qkv && t0 <= pos && pos < t1 && rg == 0;

    // ---- per-warp K/V tiles: w, w + 4, ... of the split's 16-key tiles. The
    // first ones are requested before the query rows are prepared (their HBM
    // latency overlaps that work), except in the CTA that appends the new key.
    const int ntiles = t1 > t0 ? (t1 - t0 + TKM - 1) / TKM : 0;
    const T *kbase = static_cast<const T *>(p.k) + b * p.ks[0] + kvh * p.ks[1];
    const T *vbase = static_cast<const T *>(p.v) + b * p.vs[0] + kvh * p.vs[1];
    const uint32_t ring_u = smem_u32(rings) + warp * NST * 2 * TILE;
    auto issue = [&](int tile, int stage) {
        const uint32_t kst = ring_u + stage * 2 * TILE, vst = kst + TILE;
        for (int idx = lane; idx < TKM * CPR; idx += 32) {
            const int j = idx / CPR, c = idx % CPR;
            const int t = t0 + tile * TKM + j;
            const bool ok = t < t1;
            const int ts = ok ? t : t0;
            cp_async16(kst + tile_off<D>(j, c), kbase + (int64_t)ts * p.ks[2] + c * 8, ok ? 16u : 0u);
            cp_async16(vst + tile_off<D>(j, c), vbase + (int64_t)ts * p.vs[2] + c * 8, ok ? 16u : 0u);
        }
    };
    auto prime = [&]() {
#pragma unroll
        for (int s2 = 0; s2 < NST - 1; ++s2) {
            const int tile = warp + s2 * MMA_WARPS;
            if (tile < ntiles) issue(tile, s2);
            cp_async_commit();
        }
    };
    // ---- query rows -> qb (16-bit, rows >= R zero), with the fused RoPE/append
    if (p.qkv) {
        constexpr int half = D / 2, NTH = MMA_WARPS * 32;
        static_assert(NTH % half == 0, "a thread keeps one rotation frequency");
        constexpr int RPP = NTH / half, PER = 16 / RPP;  // rows per pass, passes over the 16 MMA rows
        const int W = (p.Hq + 2 * p.Hkv) * D;
        const __nv_bfloat16 *row = p.qkv + (int64_t)b * W;
        // thread: frequency i = tid % half of rows r0, r0 + RPP, ... Every load
        // is issued first -- the query rows (and, in the appending CTA, the new
        // key and value) ahead of the K/V ring, so that they do not queue behind
        // it -- then the ring, then the arithmetic.
        const int i = tid % half, r0 = tid / half;
        const bool kv_lane = appends && tid < half;
        const float fq = r0 < R ? p.inv_freq[i] : 0.0f;
        float x1[PER], x2[PER];
#pragma unroll
        for (int k = 0; k < PER; ++k) {
            const int r = r0 + k * RPP;
            x1[k] = x2[k] = 0.0f;
            if (r < R) {
                const int hq = kvh * p.rep + r;
                x1[k] = __bfloat162float(row[hq * D + i]);
                x2[k] = __bfloat162float(row[hq * D + i + half]);
            }
        }
        const __nv_bfloat16 *kr = row + (p.Hq + kvh) * D, *vr = row + (p.Hq + p.Hkv + kvh) * D;
        float y1 = 0.0f, y2 = 0.0f;
        __nv_bfloat16 v1 = __float2bfloat16_rn(0.0f), v2 = v1;
        if (kv_lane) {
            y1 = __bfloat162float(kr[i]);
            y2 = __bfloat162float(kr[i + half]);
            v1 = vr[i];
            v2 = vr[i + half];
        }
        if (!appends) prime();
        float c = 0.0f, sn = 0.0f;
        if (r0 < R) {
            const float f = fq * (float)pos;
            c = bfr16(cosf(f));
            sn = bfr16(sinf(f));
        }
#pragma unroll
        for (int k = 0; k < PER; ++k) {
            const int r = r0 + k * RPP;
            float lo = 0.0f, hi = 0.0f;
            if (r < R) {
                lo = bfr16(bfr16(x1[k] * c) + bfr16(-x2[k] * sn));
                hi = bfr16(bfr16(x2[k] * c) + bfr16(x1[k] * sn));
            }
            reinterpret_cast<T *>(qb + tile_off<D>(r, i / 8))[i % 8] = (T)lo;
            reinterpret_cast<T *>(qb + tile_off<D>(r, (i + half) / 8))[(i + half) % 8] = (T)hi;
        }
        if (kv_lane) {
            __nv_bfloat16 *kc = (__nv_bfloat16 *)p.k + b * p.ks[0] + kvh * p.ks[1] + (int64_t)pos * p.ks[2];
            __nv_bfloat16 *vc = (__nv_bfloat16 *)p.v + b * p.vs[0] + kvh * p.vs[1] + (int64_t)pos * p.vs[2];
            kc[i] = __float2bfloat16_rn(bfr16(y1 * c) + bfr16(-y2 * sn));
            kc[i + half] = __float2bfloat16_rn(bfr16(y2 * c) + bfr16(y1 * sn));
            vc[i] = v1;
            vc[i + half] = v2;
        }
    } else {
        if (!appends) prime();
        for (int idx = tid; idx < 16 * D; idx += MMA_WARPS * 32) {
            const int r = idx / D, d = idx % D;
            T v = (T)0.0f;
            if (r < R) {
                const int gr = rg * p.rows + r, l = gr / p.rep, hq = kvh * p.rep + gr % p.rep;
                v = static_cast<const T *>(p.q)[b * p.qs[0] + hq * p.qs[1] + l * p.qs[2] + d];
            }
            reinterpret_cast<T *>(qb + tile_off<D>(r, d / 8))[d % 8] = v;
        }
    }
    __syncthreads();  // qb complete; the appended slot is written before any tile copy reads it
    if (appends) prime();

    // Q fragments (A operand, rows g / g+8, all k-steps), loaded once
    uint32_t qa[KS][4];
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
        const int c0 = 2 * kk, c1 = 2 * kk + 1;
        qa[kk][0] = *reinterpret_cast<const uint32_t *>(qb + tile_off<D>(g, c0) + 4 * t4);
        qa[kk][1] = *reinterpret_cast<const uint32_t *>(qb + tile_off<D>(g + 8, c0) + 4 * t4);
        qa[kk][2] = *reinterpret_cast<const uint32_t *>(qb + tile_off<D>(g, c1) + 4 * t4);
        qa[kk][3] = *reinterpret_cast<const uint32_t *>(qb + tile_off<D>(g + 8, c1) + 4 * t4);
    }
    int lrow[2];  // query position of rows g, g+8 (causal masking)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int gr = rg * p.rows + g + 8 * h;
        lrow[h] = gr / p.rep;
    }

    float o[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f};

    int it = 0;
    for (int tile = warp; tile < ntiles; tile += MMA_WARPS, ++it) {
        {   // keep NST - 1 tiles ahead
            const int nxt = tile + (NST - 1) * MMA_WARPS;
            if (nxt < ntiles) issue(nxt, (it + NST - 1) % NST);
            cp_async_commit();
        }
        cp_async_wait<NST - 1>();
        __syncwarp();
        const int stage = it % NST;
        const uint32_t kst = ring_u + stage * 2 * TILE, vst = kst + TILE;

        // S = Q K^T for 16 keys: n-tiles 0 (keys 0-7) and 1 (keys 8-15)
        float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
            const int mat = lane >> 3, rr = lane & 7;
            const int key = rr + ((mat & 2) ? 8 : 0), c = 2 * kk + (mat & 1);
            uint32_t b0, b1, b2, b3;
            ldsm_x4(kst + tile_off<D>(key, c), b0, b1, b2, b3);
            mma16816<T>(sc[0], qa[kk], b0, b1);
            mma16816<T>(sc[1], qa[kk], b2, b3);
        }
        // scale, mask, online softmax for rows g (h = 0) and g + 8 (h = 1)
        const int tb = t0 + tile * TKM;
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int n = 0; n < 2; ++n) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int h = e >> 1, key = tb + 8 * n + 2 * t4 + (e & 1);
                float v = sc[n][e] * p.scale;
                const bool masked = key >= t1 || (p.causal && key > lrow[h]);
                v = masked ? -INFINITY : v + 0.0f;
                sc[n][e] = v;
                mx[h] = fmaxf(mx[h], v);
            }
        }
        float alpha[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
            mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
            const float m_new = fmaxf(m_run[h], mx[h]);
            alpha[h] = (m_run[h] == -INFINITY) ? 0.0f : expf(m_run[h] - m_new);
            m_run[h] = m_new;
        }
        float ps[2][4];
#pragma unroll
        for (int n = 0; n < 2; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int h = e >> 1;
                ps[n][e] = (m_run[h] == -INFINITY) ? 0.0f : expf(sc[n][e] - m_run[h]);
            }
#pragma unroll
        for (int h = 0; h < 2; ++h)
            l_run[h] = l_run[h] * alpha[h] + ps[0][2 * h] + ps[0][2 * h + 1] + ps[1][2 * h] + ps[1][2 * h + 1];
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            o[n][0] *= alpha[0];
            o[n][1] *= alpha[0];
            o[n][2] *= alpha[1];
            o[n][3] *= alpha[1];
        }
        // O += P V: P as the A fragment (keys 0-15 = k), V through ldmatrix.trans
        uint32_t pa[4];
        pa[0] = pack2<T>(ps[0][0], ps[0][1]);
        pa[1] = pack2<T>(ps[0][2], ps[0][3]);
        pa[2] = pack2<T>(ps[1][0], ps[1][1]);
        pa[3] = pack2<T>(ps[1][2], ps[1][3]);
#pragma unroll
        for (int n2 = 0; n2 < NT / 2; ++n2) {
            const int mat = lane >> 3, rr = lane & 7;
            const int key = rr + ((mat & 1) ? 8 : 0), c = 2 * n2 + (mat >> 1);
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(vst + tile_off<D>(key, c), b0, b1, b2, b3);
            mma16816<T>(o[2 * n2], pa, b0, b1);
            mma16816<T>(o[2 * n2 + 1], pa, b2, b3);
        }
        __syncwarp();  // this stage is refilled NST - 1 tiles later
    }
    cp_async_wait<0>();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 1);
        l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 2);
    }
    __syncthreads();  // every warp's ring is drained: reuse it for the warp merge

    // ---- merge the 4 warps: cmb = [warp][16] m, [warp][16] l, [warp][16][WOS] o
    // (rows padded by 4 floats: the 8 row groups g of a fragment store land in
    // 8 different bank quads)
    constexpr int WOS = D + 4;
    float *wm = cmb, *wl = cmb + MMA_WARPS * 16, *wo = cmb + 2 * MMA_WARPS * 16;
    if (t4 == 0) {
        wm[warp * 16 + g] = m_run[0];
        wm[warp * 16 + g + 8] = m_run[1];
        wl[warp * 16 + g] = l_run[0];
        wl[warp * 16 + g + 8] = l_run[1];
    }
#pragma unroll
    for (int n = 0; n < NT; ++n) {
        float *r0p = wo + (warp * 16 + g) * WOS + 8 * n + 2 * t4, *r1p = r0p + 8 * WOS;
        *reinterpret_cast<float2 *>(r0p) = make_float2(o[n][0], o[n][1]);
        *reinterpret_cast<float2 *>(r1p) = make_float2(o[n][2], o[n][3]);
    }
    __syncthreads();
    // the warps' weights e^(m_w - M) once per (warp, row), then one float4 of a
    // row per thread
    __shared__ float wa[MMA_WARPS * 16], wml[16][2];
    if (tid < R) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < MMA_WARPS; ++w) M = fmaxf(M, wm[w * 16 + tid]);
        float l = 0.0f;
#pragma unroll
        for (int w = 0; w < MMA_WARPS; ++w) {
            const float mw = wm[w * 16 + tid];
            const float a = (mw == -INFINITY) ? 0.0f : expf(mw - M);
            wa[w * 16 + tid] = a;
            l = fmaf(a, wl[w * 16 + tid], l);
        }
        wml[tid][0] = M;
        wml[tid][1] = l;
    }
    __syncthreads();
    for (int idx = tid; idx < R * (D / 4); idx += MMA_WARPS * 32) {
        const int r = idx / (D / 4), d4 = idx % (D / 4);
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
        for (int w = 0; w < MMA_WARPS; ++w) {
            const float a = wa[w * 16 + r];
            const float4 o4 = *reinterpret_cast<const float4 *>(wo + (w * 16 + r) * WOS + 4 * d4);
            acc.x = fmaf(a, o4.x, acc.x);
            acc.y = fmaf(a, o4.y, acc.y);
            acc.z = fmaf(a, o4.z, acc.z);
            acc.w = fmaf(a, o4.w, acc.w);
        }
        const int gr = rg * p.rows + r, lq = gr / p.rep, hq = kvh * p.rep + gr % p.rep;
        const int64_t row = ((int64_t)b * p.Hq + hq) * p.L + lq;
        *reinterpret_cast<float4 *>(p.part_o + (row * p.splits + split) * D + 4 * d4) = acc;
        if (d4 == 0)
            *reinterpret_cast<float2 *>(p.part_ml + (row * p.splits + split) * 2) = make_float2(wml[r][0], wml[r][1]);
    }
    if (!p.counters) return;
    {
        const size_t rings_b = (size_t)MMA_WARPS * NST * 2 * TKM * D * 2;
        const size_t merge_b = (size_t)(2 * MMA_WARPS * 16 + MMA_WARPS * 16 * WOS) * 4;
        merge_if_last<T, D>(p, b, kvh, rg, R, tid, cmb, rings_b > merge_b ? rings_b : merge_b);
    }
}

template <int D>
size_t decode_mma_smem() {
    const size_t rings = (size_t)MMA_WARPS * NST * 2 * TKM * D * 2;
    const size_t merge = (size_t)(2 * MMA_WARPS * 16 + MMA_WARPS * 16 * (D + 4)) * 4;
    return 16 * D * 2 + D * 4 + (rings > merge ? rings : merge) + 128;
}

template <typename T, int D>
size_t decode_smem() {
    using LY = Layout<T, D>;
    const size_t ring = (size_t)NSTAGE * 2 * LY::TILE_BYTES, o = (size_t)LY::PV_GROUPS * RMAX * D * 4;
    return (size_t)(RMAX * D + RMAX * TK + 4 * RMAX) * 4 + (ring > o ? ring : o) + 128;
}

template <typename T, int D, bool MMA>
int launch_typed(const SdpaParams &p, cudaStream_t stream) {
    size_t smem;
    void (*kernel)(const SdpaParams);
    if constexpr (MMA) {
        smem = decode_mma_smem<D>();
        kernel = sdpa_decode_mma_kernel<T, D>;
    } else {
        smem = decode_smem<T, D>();
        kernel = sdpa_decode_kernel<T, D>;
    }
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        int st = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                            "aten._scaled_dot_product_flash_attention_for_cpu", "cudaFuncSetAttribute");
        if (st) return st;
        configured[dev] = 1;
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.splits, p.row_groups * p.Hkv, p.B);
    cfg.blockDim = dim3(MMA ? MMA_WARPS * 32 : kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int st = check_cuda(cudaLaunchKernelEx(&cfg, kernel, p), "aten._scaled_dot_product_flash_attention_for_cpu",
                        "cudaLaunchKernelEx (decode)");
    if (st) return st;
    __atomic_fetch_add(&counters().sdpa_decode_launches, 1ull, __ATOMIC_RELAXED);
    if (p.counters) return TN_OK;
    const int64_t rows = (int64_t)p.B * p.Hq * p.L;
    cudaLaunchConfig_t cfg2 = cfg;
    cfg2.gridDim = dim3((unsigned)((rows + 3) / 4));
    cfg2.blockDim = dim3(128);
    cfg2.dynamicSmemBytes = 0;
    return check_cuda(cudaLaunchKernelEx(&cfg2, sdpa_combine_kernel<T, D>, p),
                      "aten._scaled_dot_product_flash_attention_for_cpu", "cudaLaunchKernelEx (combine)");
}

}  // namespace

int plan_sdpa_decode(SdpaParams &p, int sm_count, int dtype) {
    const int R = p.rep * p.L;
    p.rows = R < RMAX ? R : RMAX;
    p.row_groups = (R + p.rows - 1) / p.rows;
    const int64_t base = (int64_t)p.B * p.Hkv * p.row_groups;
    // About two CTAs per SM when few (b, kv head) pairs share the GPU, one
    // otherwise, and no split shorter than one 16-key tile per warp (tensor-core
    // kernel) or 4 tiles of 32 keys (SIMT kernel): the last CTA's merge grows
    // with the split count (measured on B200: batch 1, 8 KV heads, 2049 keys:
    // 37 splits 11.5 us, 19 splits 12.0 us; batch 4: 5 splits 18.5 us, 10
    // splits 23.3 us).
    const bool mma = dtype != TN_F32 && !p.mask;
    const int min_keys = mma ? MMA_WARPS * TKM : 4 * TK;
    const int64_t per_sm = base <= 8 ? 2 : 1;
    int64_t want = (per_sm * sm_count + base - 1) / base;
    const int64_t max_splits = (p.S + min_keys - 1) / min_keys;
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
    // bf16 / f16 without an additive mask: tensor cores; f32 (whose products
    // must stay f32) and masked calls: the SIMT kernel.
    const bool mma = dtype != TN_F32 && !p.mask;
    if (p.D == 128) {
        if (dtype == TN_F32) return launch_typed<float, 128, false>(p, stream);
        if (dtype == TN_BF16)
            return mma ? launch_typed<__nv_bfloat16, 128, true>(p, stream)
                       : launch_typed<__nv_bfloat16, 128, false>(p, stream);
        return mma ? launch_typed<__half, 128, true>(p, stream) : launch_typed<__half, 128, false>(p, stream);
    }
    if (dtype == TN_F32) return launch_typed<float, 64, false>(p, stream);
    if (dtype == TN_BF16)
        return mma ? launch_typed<__nv_bfloat16, 64, true>(p, stream) : launch_typed<__nv_bfloat16, 64, false>(p, stream);
    return mma ? launch_typed<__half, 64, true>(p, stream) : launch_typed<__half, 64, false>(p, stream);
}

}  // namespace tn
