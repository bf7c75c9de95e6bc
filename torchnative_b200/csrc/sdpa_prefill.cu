// sdpa_prefill.cu -- flash attention for many query rows (prefill) on the 5th
// generation tensor cores: tcgen05.mma with both products accumulated in TMEM,
// Q/K/V tiles brought by TMA (128-byte swizzle), online softmax in registers.
//
// One CTA = one (batch, query head, 128 query rows) tile, 4 warps; thread t
// owns query row t, which is TMEM lane t. Per 128-key tile j:
//   S = Q K_j^T       (8 MMAs of K = 16 into TMEM columns [0, 128))
//   softmax: s * scale, upper-left causal / key-range mask, running max m and
//            sum l per row in f32 (the reference's arithmetic, aten.rs:10327-10420,
//            reorganised as FlashAttention's online softmax), O rescaled in TMEM
//   P (bf16 / f16, the input dtype) -> shared memory in the swizzled K-major layout
//   O += P V_j        (8 MMAs into TMEM columns [128, 256); V read MN-major)
// K/V tiles are double-buffered; the tile after next is requested as soon as
// the PV product that read a stage has completed. GQA by indexing: the K/V
// coordinates use kv head hq / (Hq / Hkv). out = O / l, lse = m + log l.
#include "sdpa_common.cuh"
#include "tc05.cuh"

namespace tn {
namespace {

constexpr int BM = 128;                 // query rows per CTA
constexpr int BN = 128;                 // keys per tile
constexpr int HD = 128;                 // head dimension
constexpr int PANEL = BM * 128;         // one 64-column panel of a 128-row tile (bytes)
constexpr int TILE = 2 * PANEL;         // a 128 x 128 16-bit tile
constexpr int OFF_Q = 0, OFF_K0 = TILE, OFF_V0 = 2 * TILE, OFF_K1 = 3 * TILE, OFF_V1 = 4 * TILE, OFF_P = 5 * TILE;
constexpr int OFF_BAR = 6 * TILE;
constexpr size_t PREFILL_SMEM = 6 * TILE + 64 + 2 * 128 * 4 + 1024;  // + barriers, exchange, alignment

struct PrefillArgs {
    int B, Hq, Hkv, L, S, rep, causal, bf16;
    float scale;
    void *out;
    float *lse;
    int *err;
};

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

__global__ void __launch_bounds__(256, 1) sdpa_prefill_kernel(const __grid_constant__ CUtensorMap mq,
                                                              const __grid_constant__ CUtensorMap mk,
                                                              const __grid_constant__ CUtensorMap mv,
                                                              const PrefillArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sb = smem_u32(base);
    uint64_t *bars = reinterpret_cast<uint64_t *>(base + OFF_BAR);
    uint64_t *q_full = bars, *k_full = bars + 1 /*[2]*/, *v_full = bars + 3 /*[2]*/, *s_done = bars + 5,
             *o_done = bars + 6;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 7);
    float *xch = reinterpret_cast<float *>(base + OFF_BAR + 64);  // [2][128] row partials between the warpgroups

    // Two warpgroups: both own every query row (thread r of a warpgroup owns
    // TMEM lane r = row q0 + r); warpgroup 0 works on key/dim columns 0-63,
    // warpgroup 1 on 64-127, and they trade row maxima and sums through `xch`.
    const int tid = threadIdx.x, warp = tid >> 5, wg = tid >> 7, r = tid & 127;
    const int qt = blockIdx.x, hq = blockIdx.y, b = blockIdx.z;
    const int hkv = hq / a.rep, q0 = qt * BM;
    const int row = q0 + r;
    const int last_key = a.causal ? min(q0 + BM - 1, a.S - 1) : a.S - 1;
    const int ntiles = last_key / BN + 1;
    const float c2 = a.scale * 1.4426950408889634f;  // scale * log2(e): p = 2^(s*c2 - m2)

    if (warp == 0) tc05::alloc(tmem_slot, 256);
    if (tid == 0) {
        for (int i = 0; i < 7; ++i) mbar_init(&bars[i], 1);
        fence_mbar_init();
        tc05::prefetch_map(&mq);
        tc05::prefetch_map(&mk);
        tc05::prefetch_map(&mv);
    }
    tc05::fence_before();
    __syncthreads();
    tc05::fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_off + wg * 64, tO = tmem + 128 + lane_off + wg * 64;

    pdl_launch_dependents();
    pdl_wait();

    // K and V rings of two stages each, tracked separately: K_{j+2} may replace
    // K_j once S_j is computed, V_{j+1} replaces V_{j-1} once PV_{j-1} is done.
    int k_issued = 0, v_issued = 0;  // tiles requested (thread 0)
    auto load_k = [&](int j) {
        const int st = j & 1;
        const uint32_t kd = sb + (st ? OFF_K1 : OFF_K0);
        mbar_arrive_expect_tx(&k_full[st], TILE);
        for (int p = 0; p < 2; ++p) tc05::tma_load_4d(kd + p * PANEL, &mk, p * 64, j * BN, hkv, b, &k_full[st]);
    };
    auto load_v = [&](int j) {
        const int st = j & 1;
        const uint32_t vd = sb + (st ? OFF_V1 : OFF_V0);
        mbar_arrive_expect_tx(&v_full[st], TILE);
        for (int p = 0; p < 2; ++p) tc05::tma_load_4d(vd + p * PANEL, &mv, p * 64, j * BN, hkv, b, &v_full[st]);
    };
    const uint32_t id_qk = tc05::idesc_f16(a.bf16 != 0, BM, BN, false);
    const uint32_t id_pv = tc05::idesc_f16(a.bf16 != 0, BM, HD, true);
    bool bad = false, aborted = false;
    // S_j = Q K_j^T into TMEM columns [0, 128), by thread 0.
    auto issue_qk = [&](int j) {
        const int st = j & 1;
        bool ok = !bad && (j > 0 || mbar_wait(q_full, 0)) && mbar_wait(&k_full[st], (j >> 1) & 1);
        if (!ok) {
            record_device_error(a.err, DEV_ERR_WAIT_FULL);
            bad = true;
        } else {
            tc05::fence_after();
            const uint32_t kb = sb + (st ? OFF_K1 : OFF_K0);
#pragma unroll
            for (int kk = 0; kk < HD / 16; ++kk) {
                const uint32_t off = (kk >> 2) * PANEL + (kk & 3) * 32;
                tc05::mma_ss(tmem, tc05::desc_sw128(sb + OFF_Q + off, 16, 1024), tc05::desc_sw128(kb + off, 16, 1024),
                             id_qk, kk > 0);
            }
        }
        tc05::commit(s_done);  // arrives even if nothing was issued
    };
    if (tid == 0) {
        mbar_arrive_expect_tx(q_full, TILE);
        for (int p = 0; p < 2; ++p) tc05::tma_load_4d(sb + OFF_Q + p * PANEL, &mq, p * 64, q0, hq, b, q_full);
        for (int j = 0; j < 2 && j < ntiles; ++j) {
            load_k(j);
            load_v(j);
        }
        k_issued = v_issued = ntiles < 2 ? ntiles : 2;
        issue_qk(0);
    }

    float m2 = -INFINITY, l_part = 0.0f;  // running max (log2 units, scaled) and this half's sum
    for (int j = 0; j < ntiles; ++j) {
        // ---- S_j, this warpgroup's 64 keys of row r
        if (!mbar_wait(s_done, j & 1)) {
            record_device_error(a.err, DEV_ERR_WAIT_FULL);
            bad = true;
        }
        tc05::fence_after();
        if (tid == 0 && k_issued < ntiles && k_issued == j + 2 && !bad) {  // S_j done: K stage j&1 is free
            load_k(k_issued);
            ++k_issued;
        }
        float sv[64];
        {
            float v[32];
            tc05::ld32(tS, v);
            tc05::wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) sv[i] = v[i];
            tc05::ld32(tS + 32, v);
            tc05::wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) sv[32 + i] = v[i];
        }
        // Raw scores here; the scale is applied inside the exponent (c2 > 0, so
        // the maximum of the raw scores scales to the maximum of the scaled).
        // Only tiles that reach the diagonal or the key range end need masks.
        float mx = -INFINITY;
        const int kbase = j * BN + wg * 64;
        const bool full = (j + 1) * BN <= a.S && (!a.causal || (j + 1) * BN - 1 <= q0);
        if (full) {
#pragma unroll
            for (int c = 0; c < 64; ++c) mx = fmaxf(mx, sv[c]);
        } else {
#pragma unroll
            for (int c = 0; c < 64; ++c) {
                const int key = kbase + c;
                const bool masked = key >= a.S || (a.causal && key > row);
                sv[c] = masked ? -INFINITY : sv[c];
                mx = fmaxf(mx, sv[c]);
            }
        }
        mx = mx * c2;
        xch[wg * 128 + r] = mx;
        tc05::fence_before();
        asm volatile("bar.sync 1, 256;" ::: "memory");
        // S_j is in registers everywhere: the tensor core may overwrite it with S_{j+1}
        if (tid == 0 && j + 1 < ntiles) {
            tc05::fence_after();
            issue_qk(j + 1);
        }
        mx = fmaxf(mx, xch[(wg ^ 1) * 128 + r]);
        const float m_new = fmaxf(m2, mx);
        const float alpha = (m2 == -INFINITY) ? 0.0f : exp2f(m2 - m_new);
        float sum = 0.0f;
        if (m_new == -INFINITY) {
#pragma unroll
            for (int c = 0; c < 64; ++c) sv[c] = 0.0f;
        } else {
#pragma unroll
            for (int c = 0; c < 64; ++c) {
                const float p = exp2f(fmaf(sv[c], c2, -m_new));
                sv[c] = p;
                sum += p;
            }
        }
        l_part = l_part * alpha + sum;
        m2 = m_new;

        // ---- PV_{j-1} finished: its K/V stage is free, O can be rescaled, P rewritten
        if (j > 0) {
            if (!mbar_wait(o_done, (j - 1) & 1)) {
                record_device_error(a.err, DEV_ERR_WAIT_FULL);
                bad = true;
            }
            tc05::fence_after();
            if (tid == 0 && v_issued < ntiles && v_issued == j + 1 && !bad) {  // PV_{j-1} done: V stage free
                load_v(v_issued);
                ++v_issued;
            }
            if (__any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll
                for (int c = 0; c < 2; ++c) {
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
        // P (this warpgroup's 64 keys = one panel) -> shared memory, swizzled K-major
        {
            const uint32_t prow = sb + OFF_P + wg * PANEL + r * 128;
#pragma unroll
            for (int cc = 0; cc < 8; ++cc) {
                const uint32_t addr = prow + ((cc ^ (r & 7)) << 4);
                st_shared_v4(addr, pack_t(sv[cc * 8 + 0], sv[cc * 8 + 1], a.bf16),
                             pack_t(sv[cc * 8 + 2], sv[cc * 8 + 3], a.bf16), pack_t(sv[cc * 8 + 4], sv[cc * 8 + 5], a.bf16),
                             pack_t(sv[cc * 8 + 6], sv[cc * 8 + 7], a.bf16));
            }
        }
        fence_proxy_async_smem();
        tc05::fence_before();
        if (__syncthreads_or(bad)) {
            aborted = true;
            break;
        }
        // ---- O += P V_j
        if (tid == 0) {
            tc05::fence_after();
            const int st = j & 1;
            const uint32_t vb = sb + (st ? OFF_V1 : OFF_V0);
            if (!mbar_wait(&v_full[st], (j >> 1) & 1)) {
                record_device_error(a.err, DEV_ERR_WAIT_FULL);
                bad = true;
            }
            tc05::fence_after();
#pragma unroll
            for (int kk = 0; kk < BN / 16; ++kk) {
                const uint32_t poff = (kk >> 2) * PANEL + (kk & 3) * 32;
                tc05::mma_ss(tmem + 128, tc05::desc_sw128(sb + OFF_P + poff, 16, 1024),
                             tc05::desc_sw128(vb + kk * 2048, PANEL, 1024), id_pv, (j > 0 || kk > 0) ? 1u : 0u);
            }
            tc05::commit(o_done);
        }
    }

    // ---- out = O / l, lse = m + log l (the two halves' sums added)
    xch[wg * 128 + r] = l_part;
    asm volatile("bar.sync 1, 256;" ::: "memory");
    const float l_run = l_part + xch[(wg ^ 1) * 128 + r];
    if (!aborted && mbar_wait(o_done, (ntiles - 1) & 1)) {
        tc05::fence_after();
        const float inv = 1.0f / l_run;
        const int64_t orow = ((int64_t)b * a.Hq + hq) * a.L + row;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            float v[32];
            tc05::ld32(tO + c * 32, v);
            tc05::wait_ld();
            if (row < a.L) {
                uint32_t w[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) w[i] = pack_t(v[2 * i] * inv, v[2 * i + 1] * inv, a.bf16);
                int4 *dst = reinterpret_cast<int4 *>(static_cast<uint8_t *>(a.out) + (orow * HD + wg * 64 + c * 32) * 2);
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    dst[i] = make_int4((int)w[4 * i], (int)w[4 * i + 1], (int)w[4 * i + 2], (int)w[4 * i + 3]);
            }
        }
        if (row < a.L && a.lse && wg == 0) a.lse[orow] = m2 * 0.6931471805599453f + logf(l_run);
    } else if (!aborted) {
        record_device_error(a.err, DEV_ERR_WAIT_FULL);
    }
    // Drain: no TMA copy may still be writing this CTA's shared memory.
    if (tid == 0) {
        for (int j = k_issued > 2 ? k_issued - 2 : 0; j < k_issued; ++j)
            if (!mbar_wait(&k_full[j & 1], (j >> 1) & 1)) {
                record_device_error(a.err, DEV_ERR_DRAIN);
                break;
            }
        for (int j = v_issued > 2 ? v_issued - 2 : 0; j < v_issued; ++j)
            if (!mbar_wait(&v_full[j & 1], (j >> 1) & 1)) {
                record_device_error(a.err, DEV_ERR_DRAIN);
                break;
            }
    }
    tc05::fence_before();
    __syncthreads();
    if (warp == 0) {
        tc05::fence_after();
        tc05::dealloc(tmem, 256);
    }
}

}  // namespace

// Host: q/k/v bf16 or f16, D = 128, no mask; strides in elements [b, h, t, d].
int launch_sdpa_prefill(const SdpaParams &p, int dtype, cudaStream_t stream) {
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
    PrefillArgs a{};
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
        int st = check_cuda(cudaFuncSetAttribute(sdpa_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)PREFILL_SMEM),
                            op, "cudaFuncSetAttribute");
        if (st) return st;
        configured[dev] = 1;
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((p.L + BM - 1) / BM), (unsigned)p.Hq, (unsigned)p.B);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = PREFILL_SMEM;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int st = check_cuda(cudaLaunchKernelEx(&cfg, sdpa_prefill_kernel, mq, mk, mv, a), op, "cudaLaunchKernelEx (prefill)");
    if (st) return st;
    __atomic_fetch_add(&counters().sdpa_prefill_launches, 1ull, __ATOMIC_RELAXED);
    return TN_OK;
}

}  // namespace tn
