// sdpa_prefill2.cu -- flash attention for many query rows on tcgen05, two
// query tiles per CTA (each with its own softmax warpgroup), so one tile's
// softmax runs while the tensor core works on the other's products.
//
// One CTA = 256 query rows (tiles Q0, Q1 of 128) of one (batch, query head),
// 12 warps:
//   warps 0-3   softmax of Q0: thread r owns row r (TMEM lane r) and all 64
//               columns of a key tile -- no exchange between warpgroups
//   warps 4-7   softmax of Q1, the same
//   warp 8      TMA producer: Q0 and Q1 once, then K and V tiles of 64 keys
//               (128-byte swizzle) into separate 3-stage rings
//   warp 9      MMA issuer (one thread): S_k = Q_k K_j^T into TMEM (double
//               buffered per tile), then O_k += P_k V_{j-1} one tile behind
//   warp 10     TMEM owner (512 columns: S0[2], S1[2], O0, O1)
// Softmax per tile: raw scores, masks only on tiles that reach the diagonal or
// the key-range end, the row maximum kept in log2 units; the maximum used in
// the exponent moves only when the new maximum exceeds it by more than 8 (P
// then stays below 2^8), and only then is O rescaled in TMEM -- out = O / l
// is exact for any choice of that maximum. P (input dtype) goes to shared
// memory in the swizzled K-major layout the PV MMA reads.
// Every wait is bounded; a wait that gives up raises a CTA-wide abort flag,
// the producer and the MMA issuer wait (bounded) for their copies and MMAs,
// TMEM is freed.
#include "sdpa_common.cuh"
#include "tc05.cuh"

namespace tn {
namespace {

constexpr int BM = 128, NQT = 2, BN = 64, HD = 128;
constexpr int NK = 3, NV = 3;
constexpr int QPANEL = BM * 128;           // 128 rows x 64 columns of 16-bit
constexpr int QTILE = 2 * QPANEL;          // 128 x 128
constexpr int KPANEL = BN * 128;           // 64 rows x 64 columns
constexpr int KTILE = 2 * KPANEL;          // 64 x 128
constexpr int PTILE = BM * 128;            // 128 rows x 64 keys
constexpr int OFF_Q = 0, OFF_K = NQT * QTILE, OFF_V = OFF_K + NK * KTILE, OFF_P = OFF_V + NV * KTILE;
constexpr int OFF_BAR = OFF_P + NQT * PTILE;
constexpr size_t PREFILL2_SMEM = OFF_BAR + 256 + 1024;
constexpr int THREADS = 12 * 32;

struct Args {
    int B, Hq, Hkv, L, S, rep, causal, bf16;
    float scale;
    void *out;
    float *lse;
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

__device__ __forceinline__ uint32_t pack_t(float lo, float hi, int bf16) {
    if (bf16) {
        const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<const uint32_t *>(&v);
    }
    const __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&v);
}

// Packed f32 pairs (sm_100 f32x2: two lanes per instruction, each rounded as
// the scalar operation) on 64-bit pair registers, so loop-invariant pairs are
// packed once; the MUFU base-2 exponential; a three-input maximum.
__device__ __forceinline__ uint64_t pk2(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void upk2(uint64_t r, float &a, float &b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t fma2p(uint64_t x, uint64_t y, uint64_t z) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(x), "l"(y), "l"(z));
    return d;
}
__device__ __forceinline__ uint64_t add2p(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
    float y;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(y) : "f"(a), "f"(b), "f"(c));
    return y;
}
__device__ __forceinline__ float ex2a(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Key tiles of query tile k (rows q0 + 128 k ...): none past the sequence,
// and up to its diagonal when causal.
__device__ __forceinline__ int tiles_of(const Args &a, int q0, int k) {
    const int r0 = q0 + BM * k;
    if (r0 >= a.L) return 0;
    const int last_key = a.causal ? min(r0 + BM - 1, a.S - 1) : a.S - 1;
    return last_key < 0 ? 0 : last_key / BN + 1;
}

__global__ void __launch_bounds__(THREADS, 1) sdpa_prefill2_kernel(const __grid_constant__ CUtensorMap mq,
                                                                   const __grid_constant__ CUtensorMap mk,
                                                                   const __grid_constant__ CUtensorMap mv,
                                                                   const Args a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sb = smem_u32(base);
    uint64_t *bars = reinterpret_cast<uint64_t *>(base + OFF_BAR);
    uint64_t *q_full = bars, *k_full = q_full + 1, *k_empty = k_full + NK, *v_full = k_empty + NK,
             *v_empty = v_full + NV, *s_full = v_empty + NV /*[2][2]*/, *s_free = s_full + 4 /*[2][2]*/,
             *p_full = s_free + 4 /*[2]*/, *o_done = p_full + 2 /*[2]*/, *mma_done = o_done + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // One linear grid, query-tile major. Under a causal mask the work of a
    // tile grows with its index, so the last tiles go out first (longest
    // job first) and the short ones fill the tail of the last wave.
    const int heads = a.Hq * a.B, slot = (int)blockIdx.x / heads, rest = (int)blockIdx.x % heads;
    const int nqt = (int)gridDim.x / heads;
    const int qt = a.causal ? nqt - 1 - slot : slot, hq = rest % a.Hq, b = rest / a.Hq;
    const int hkv = hq / a.rep, q0 = qt * (NQT * BM);
    const int nt0 = tiles_of(a, q0, 0), nt1 = tiles_of(a, q0, 1);
    const int ntm = nt0 > nt1 ? nt0 : nt1;

    if (warp == 10) tc05::alloc(tmem_slot, 512);
    if (tid == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < NK; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
        }
        for (int i = 0; i < NV; ++i) {
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
        }
        for (int i = 0; i < 4; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&s_free[i], 4);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&p_full[i], 4);
            mbar_init(&o_done[i], 1);
        }
        mbar_init(mma_done, 1);
        *abort = 0;
        fence_mbar_init();
        tc05::prefetch_map(&mq);
        tc05::prefetch_map(&mk);
        tc05::prefetch_map(&mv);
    }
    tc05::fence_before();
    __syncthreads();
    tc05::fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();
    pdl_wait();

    if (warp == 8) {
        // ---------------- TMA producer
        if (lane == 0) {
            mbar_arrive_expect_tx(q_full, NQT * QTILE);
            for (int k = 0; k < NQT; ++k)
                for (int p = 0; p < 2; ++p)
                    tc05::tma_load_4d(sb + OFF_Q + k * QTILE + p * QPANEL, &mq, p * 64, q0 + BM * k, hq, b, q_full);
            int kis = 0, vis = 0;
            for (int j = 0; j < ntm && !*abort; ++j) {
                const int ks = j % NK, vs = j % NV;
                if (j >= NK && !wait_or_abort(&k_empty[ks], ((j / NK) - 1) & 1, abort, a.err)) break;
                mbar_arrive_expect_tx(&k_full[ks], KTILE);
                for (int p = 0; p < 2; ++p)
                    tc05::tma_load_4d(sb + OFF_K + ks * KTILE + p * KPANEL, &mk, p * 64, j * BN, hkv, b, &k_full[ks]);
                ++kis;
                if (j >= NV && !wait_or_abort(&v_empty[vs], ((j / NV) - 1) & 1, abort, a.err)) break;
                mbar_arrive_expect_tx(&v_full[vs], KTILE);
                for (int p = 0; p < 2; ++p)
                    tc05::tma_load_4d(sb + OFF_V + vs * KTILE + p * KPANEL, &mv, p * 64, j * BN, hkv, b, &v_full[vs]);
                ++vis;
            }
            // drain: the last copy issued into each stage has landed
            if (!mbar_wait(q_full, 0)) record_device_error(a.err, DEV_ERR_DRAIN);
            for (int j = kis > NK ? kis - NK : 0; j < kis; ++j)
                if (!mbar_wait(&k_full[j % NK], (j / NK) & 1)) record_device_error(a.err, DEV_ERR_DRAIN);
            for (int j = vis > NV ? vis - NV : 0; j < vis; ++j)
                if (!mbar_wait(&v_full[j % NV], (j / NV) & 1)) record_device_error(a.err, DEV_ERR_DRAIN);
        }
    } else if (warp == 9) {
        // ---------------- MMA issuer
        if (lane == 0) {
            const uint32_t id_qk = tc05::idesc_f16(a.bf16 != 0, BM, BN, false);
            const uint32_t id_pv = tc05::idesc_f16(a.bf16 != 0, BM, HD, true);
            const int nt[2] = {nt0, nt1};
            bool ok = wait_or_abort(q_full, 0, abort, a.err);
            auto pv = [&](int t) -> bool {
                const int vs = t % NV;
                if (!wait_or_abort(&v_full[vs], (t / NV) & 1, abort, a.err)) return false;
                for (int k = 0; k < NQT; ++k) {
                    if (t >= nt[k]) continue;
                    if (!wait_or_abort(&p_full[k], t & 1, abort, a.err)) return false;
                    tc05::fence_after();
                    const uint32_t pb = sb + OFF_P + k * PTILE, vb = sb + OFF_V + vs * KTILE;
#pragma unroll
                    for (int kk = 0; kk < BN / 16; ++kk)
                        tc05::mma_ss(tmem + 256 + k * 128, tc05::desc_sw128(pb + kk * 32, 16, 1024),
                                     tc05::desc_sw128(vb + kk * 2048, KPANEL, 1024), id_pv, (t > 0 || kk > 0) ? 1u : 0u);
                    tc05::commit(&o_done[k]);
                }
                tc05::commit(&v_empty[vs]);
                return true;
            };
            for (int j = 0; j < ntm && ok; ++j) {
                const int ks = j % NK, buf = j & 1;
                if (!wait_or_abort(&k_full[ks], (j / NK) & 1, abort, a.err)) break;
                for (int k = 0; k < NQT && ok; ++k) {
                    if (j >= nt[k]) continue;
                    if (j >= 2 && !wait_or_abort(&s_free[k * 2 + buf], ((j >> 1) - 1) & 1, abort, a.err)) {
                        ok = false;
                        break;
                    }
                    tc05::fence_after();
                    const uint32_t qb = sb + OFF_Q + k * QTILE, kb = sb + OFF_K + ks * KTILE;
#pragma unroll
                    for (int kk = 0; kk < HD / 16; ++kk) {
                        const uint32_t qo = (kk >> 2) * QPANEL + (kk & 3) * 32, ko = (kk >> 2) * KPANEL + (kk & 3) * 32;
                        tc05::mma_ss(tmem + (k * 2 + buf) * BN, tc05::desc_sw128(qb + qo, 16, 1024),
                                     tc05::desc_sw128(kb + ko, 16, 1024), id_qk, kk > 0);
                    }
                    tc05::commit(&s_full[k * 2 + buf]);
                }
                tc05::commit(&k_empty[ks]);
                if (ok && j >= 1) ok = pv(j - 1);
            }
            if (ok && ntm > 0) pv(ntm - 1);
            tc05::commit(mma_done);
            if (!mbar_wait(mma_done, 0)) record_device_error(a.err, DEV_ERR_DRAIN);
        }
    } else if (warp < 8) {
        // ---------------- softmax of query tile k: thread r owns row q0 + 128 k + r
        const int k = warp >> 2, r = tid & 127;
        const int row = q0 + BM * k + r, row0 = q0 + BM * k;
        const int nt = k == 0 ? nt0 : nt1;
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t tO = tmem + lane_off + 256 + k * 128;
        const float c2 = a.scale * 1.4426950408889634f;  // p = 2^(s * c2 - m)
        float m_used = -INFINITY, l = 0.0f;
        bool ok = true;
        for (int t = 0; t < nt; ++t) {
            const int buf = t & 1;
            if (!wait_or_abort(&s_full[k * 2 + buf], (t >> 1) & 1, abort, a.err)) {
                ok = false;
                break;
            }
            tc05::fence_after();
            float sv[64];
            {
                float v[32];
                const uint32_t tS = tmem + lane_off + (k * 2 + buf) * BN;
                tc05::ld32(tS, v);
                tc05::wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) sv[i] = v[i];
                tc05::ld32(tS + 32, v);
                tc05::wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) sv[32 + i] = v[i];
            }
            tc05::fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_free[k * 2 + buf]);
            const bool full = (t + 1) * BN <= a.S && (!a.causal || (t + 1) * BN - 1 <= row0);
            // four independent maxima (short dependency chains), two new
            // values per three-input max, then one
            float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
            if (!full) {
#pragma unroll
                for (int c = 0; c < 64; ++c) {
                    const int key = t * BN + c;
                    const bool masked = key >= a.S || (a.causal && key > row);
                    sv[c] = masked ? -INFINITY : sv[c];
                }
            }
#pragma unroll
            for (int c = 0; c < 64; c += 2) mq[(c >> 1) & 3] = max3(mq[(c >> 1) & 3], sv[c], sv[c + 1]);
            float mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
            mx *= c2;
            // the exponent's maximum moves only by more than 2^8
            float alpha = 1.0f;
            if (mx > m_used + 8.0f) {
                alpha = (m_used == -INFINITY) ? 0.0f : exp2f(m_used - mx);
                m_used = mx;
            }
            float sum = 0.0f;
            if (m_used == -INFINITY) {
#pragma unroll
                for (int c = 0; c < 64; ++c) sv[c] = 0.0f;
            } else {
                // p = 2^(s c2 - m): packed exponent arguments, MUFU ex2, two
                // packed partial sums
                const uint64_t c2p = pk2(c2, c2), nmp = pk2(-m_used, -m_used);
                uint64_t sp = pk2(0.0f, 0.0f);
#pragma unroll
                for (int c = 0; c < 64; c += 2) {
                    float e0, e1;
                    upk2(fma2p(pk2(sv[c], sv[c + 1]), c2p, nmp), e0, e1);
                    const float p0 = ex2a(e0), p1 = ex2a(e1);
                    sv[c] = p0;
                    sv[c + 1] = p1;
                    sp = add2p(sp, pk2(p0, p1));
                }
                float s0, s1;
                upk2(sp, s0, s1);
                sum = s0 + s1;
            }
            l = l * alpha + sum;
            // PV_{t-1} has read P and written O: P may be rewritten, O rescaled
            if (t > 0) {
                if (!wait_or_abort(&o_done[k], (t - 1) & 1, abort, a.err)) {
                    ok = false;
                    break;
                }
                tc05::fence_after();
                if (__any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        float v[32];
                        tc05::ld32(tO + c * 32, v);
                        tc05::wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] *= alpha;
                        tc05::st32(tO + c * 32, v);
                    }
                    tc05::wait_st();
                }
            }
            {
                const uint32_t prow = sb + OFF_P + k * PTILE + r * 128;
#pragma unroll
                for (int cc = 0; cc < 8; ++cc)
                    st_shared_v4(prow + ((cc ^ (r & 7)) << 4), pack_t(sv[cc * 8 + 0], sv[cc * 8 + 1], a.bf16),
                                 pack_t(sv[cc * 8 + 2], sv[cc * 8 + 3], a.bf16),
                                 pack_t(sv[cc * 8 + 4], sv[cc * 8 + 5], a.bf16),
                                 pack_t(sv[cc * 8 + 6], sv[cc * 8 + 7], a.bf16));
            }
            fence_proxy_async_smem();
            tc05::fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[k]);
        }
        // ---- out = O / l, lse = m ln 2 + ln l
        if (ok && nt > 0 && wait_or_abort(&o_done[k], (nt - 1) & 1, abort, a.err)) {
            tc05::fence_after();
            const float inv = 1.0f / l;
            const int64_t orow = ((int64_t)b * a.Hq + hq) * a.L + row;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                float v[32];
                tc05::ld32(tO + c * 32, v);
                tc05::wait_ld();
                if (row < a.L) {
                    uint32_t w[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) w[i] = pack_t(v[2 * i] * inv, v[2 * i + 1] * inv, a.bf16);
                    int4 *dst = reinterpret_cast<int4 *>(static_cast<uint8_t *>(a.out) + (orow * HD + c * 32) * 2);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        dst[i] = make_int4((int)w[4 * i], (int)w[4 * i + 1], (int)w[4 * i + 2], (int)w[4 * i + 3]);
                }
            }
            if (row < a.L && a.lse) a.lse[orow] = m_used * 0.6931471805599453f + logf(l);
        }
    }

    tc05::fence_before();
    __syncthreads();
    if (warp == 10) {
        tc05::fence_after();
        tc05::dealloc(tmem, 512);
    }
}

}  // namespace

// Host: q/k/v bf16 or f16, D = 128, no mask; strides in elements [b, h, t, d].
int launch_sdpa_prefill2(const SdpaParams &p, int dtype, cudaStream_t stream) {
    const char *op = "aten._scaled_dot_product_flash_attention_for_cpu";
    CUtensorMap mq, mk, mv;
    const uint64_t es = 2;
    {
        const uint64_t dims[4] = {(uint64_t)p.D, (uint64_t)p.L, (uint64_t)p.Hq, (uint64_t)p.B};
        const uint64_t str[3] = {(uint64_t)p.qs[2] * es, (uint64_t)p.qs[1] * es, (uint64_t)p.qs[0] * es};
        int st = encode_map_4d_b16(&mq, p.q, dims, str, BM);
        if (st) return st;
    }
    {
        const uint64_t dims[4] = {(uint64_t)p.D, (uint64_t)p.S, (uint64_t)p.Hkv, (uint64_t)p.B};
        const uint64_t ks[3] = {(uint64_t)p.ks[2] * es, (uint64_t)p.ks[1] * es, (uint64_t)p.ks[0] * es};
        const uint64_t vs[3] = {(uint64_t)p.vs[2] * es, (uint64_t)p.vs[1] * es, (uint64_t)p.vs[0] * es};
        int st = encode_map_4d_b16(&mk, p.k, dims, ks, BN);
        if (st) return st;
        st = encode_map_4d_b16(&mv, p.v, dims, vs, BN);
        if (st) return st;
    }
    Args a{};
    a.B = p.B;
    a.Hq = p.Hq;
    a.Hkv = p.Hkv;
    a.L = p.L;
    a.S = p.S;
    a.rep = p.rep;
    a.causal = p.causal;
    a.bf16 = dtype == TN_BF16;
    a.scale = p.scale;
    a.out = p.out;
    a.lse = p.lse;
    a.err = p.err;
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        int st = check_cuda(cudaFuncSetAttribute(sdpa_prefill2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)PREFILL2_SMEM),
                            op, "cudaFuncSetAttribute");
        if (st) return st;
        configured[dev] = 1;
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    const long long nqt = (p.L + NQT * BM - 1) / (NQT * BM);
    const long long ctas = nqt * p.Hq * p.B;
    if (ctas > 0x7fffffffLL) return set_error(TN_ERR_SHAPE, std::string(op) + ": too many query tiles for one grid");
    cfg.gridDim = dim3((unsigned)ctas);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = PREFILL2_SMEM;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int st = check_cuda(cudaLaunchKernelEx(&cfg, sdpa_prefill2_kernel, mq, mk, mv, a), op,
                        "cudaLaunchKernelEx (prefill, two query tiles)");
    if (st) return st;
    __atomic_fetch_add(&counters().sdpa_prefill_launches, 1ull, __ATOMIC_RELAXED);
    return TN_OK;
}

}  // namespace tn
