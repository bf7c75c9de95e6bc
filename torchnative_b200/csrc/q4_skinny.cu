// q4_skinny.cu -- the Q4_0 linear for a few activation rows (batched decode:
// 9 <= M <= 32) on the 5th generation tensor cores, weights on the MMA's
// 128-row side and the activation rows as its N (16 or 32).
//
// Arithmetic (the reference's, k_quants.rs:312-330): y[m, n] = sum over
// 32-blocks b of (isum_b * d_w[n, b]) * d_x[m, b], isum_b = sum of q8 codes
// times (nibble - 8). `tcgen05.mma kind::i8` forms D = sum nibble * q8 exactly
// in s32 (unsigned nibbles 0..15 against signed codes), so the weights are
// never converted beyond splitting bytes into nibbles, and
// isum_b = D - 8 * sum(q8): the planar offset of the block (12582912 +
// 8 * sum(q8)) minus 12582912. Every block is its own MMA into one of NS TMEM
// accumulators (its scales differ per row and column); the epilogue warps
// apply acc = fma(isum * d_w, d_x, acc) in f32, block by block.
//
// One CTA = 128 weight rows x all activation rows x one range of K (a split;
// splits > 1 when the weight has too few 128-row tiles to fill the GPU in one
// wave of two CTAs per SM), 14 warps:
//   warp 0      TMA producer: per 256-wide chunk of K, the activation code
//               panels (NP rows x 128 int8 codes, 128-byte swizzle) with the
//               chunk's activation scales and offsets (NP rows x 8 blocks of
//               f32), and the raw weight chunk (128 rows x 144 bytes = 8 Q4_0
//               blocks per row, straight from the GGML blob)
//   warp 1      TMEM owner and MMA issuer (one thread): one K = 32 MMA per
//               block, M = 128, N = NP
//   warps 2-5   converters (thread = weight row): raw blocks -> nibble bytes in
//               K order in the swizzled K-major panel the MMA reads, and the
//               f32 block scales d_w
//   warps 6-13  epilogue (thread = weight row = TMEM lane; the two warps of a
//               lane quarter take half of the activation rows each): TMEM
//               loads of a group of blocks per wait, then the
//               scale-and-accumulate for each of its activation rows
// With splits, each CTA stores its partial sums; the last CTA of a tile (an
// atomic ticket) adds them in split order and writes y. Every wait is
// bounded; a wait that gives up raises a CTA-wide abort flag so the other
// roles stop too, the producer waits for its copies in flight, the MMA issuer
// for its MMAs, and TMEM is freed.
#include "q4_kernels.cuh"
#include "tc05.cuh"

namespace tn {
namespace {

constexpr int SN = 128;           // weight rows per tile
constexpr int NR = 2, NA = 3, ND = 4;
constexpr int RAW = SN * 144;     // 8 Q4_0 blocks x 128 rows
constexpr int WPANEL = SN * 128;  // 128 rows x 128 nibble bytes (4 blocks)
constexpr int CONV_WARPS = 4, EPI_WARPS = 8;
constexpr int SK_THREADS = (2 + CONV_WARPS + EPI_WARPS) * 32;
constexpr uint32_t kMagicBits = 0x4B400000u;  // 12582912.0f

template <int NP>
struct Layout {
    static constexpr int NB = NP == 16 ? 3 : 2;  // weight panels in the ring
    static constexpr int NS = NP == 16 ? 16 : 8; // TMEM accumulators
    static constexpr int EW = NP / 2;             // activation rows per epilogue warp
    static constexpr int EB = NP == 16 ? 4 : 2;   // blocks per epilogue TMEM wait
    static constexpr int APANEL = NP * 128;       // NP rows x 128 codes
    static constexpr int XT = NP * 8 * 4;         // NP rows x 8 blocks of f32
    static constexpr int ASLOT = 2 * APANEL + 2 * XT;  // codes, scales, offsets of one chunk
    static constexpr int OFF_W = 0;
    static constexpr int OFF_A = OFF_W + NB * WPANEL;
    static constexpr int OFF_R = OFF_A + NA * ASLOT;
    static constexpr int OFF_DW = OFF_R + NR * RAW;  // ND x 4 blocks x 128 rows f32
    static constexpr int OFF_BAR = OFF_DW + ND * 4 * SN * 4;
    static constexpr int NBARS = 2 * NR + 2 * NA + 2 * NB + 2 * ND + 2 * NS + 1;
    static constexpr size_t SMEM = OFF_BAR + NBARS * 8 + 64 + 1024;
    static constexpr int TMEM_COLS = NS * NP;
    static_assert(ASLOT % 1024 == 0 && OFF_R % 128 == 0, "TMA destinations");
    static_assert(TMEM_COLS == 256, "two CTAs per SM share the 512 TMEM columns");
    static_assert(NS % EB == 0 && 4 % EB == 0, "epilogue groups of EB blocks in consecutive accumulators");
};

struct SkinnyArgs {
    const float *bias;
    void *y;
    int y_dtype;
    int64_t y_row_stride;
    int M, N, nb;
    int splits, tiles;
    int pairs;     // SiLU * up of interleaved (gate, up) rows: y column n / 2
    float *part;   // [splits][M][N] partial sums (splits > 1)
    int *tickets;  // [tiles], zero between launches
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

__device__ __forceinline__ float bfr(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Instruction descriptor of kind::i8 with s32 accumulation: bits 4-5 D format
// (2 = s32), 7-9 A format and 10-12 B format (0 = unsigned 8-bit, 1 = signed),
// 15 / 16 A / B major (0 = K), 17-22 N >> 3, 24-28 M >> 4.
constexpr uint32_t idesc_i8(int M, int N, bool a_signed, bool b_signed) {
    return (2u << 4) | ((a_signed ? 1u : 0u) << 7) | ((b_signed ? 1u : 0u) << 10) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

// D[tmem] = A[smem] * B[smem]^T (no accumulation: every block starts fresh),
// issued by one thread.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, 0, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc)
        : "memory");
}

// W consecutive TMEM columns of this warp's 32 lanes (raw 32-bit words).
template <int W>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&r)[W]);
template <>
__device__ __forceinline__ void tmem_ld<8>(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

template <int NP>
__global__ void __launch_bounds__(SK_THREADS, 2) q4_skinny_kernel(const __grid_constant__ CUtensorMap map_a,
                                                                  const __grid_constant__ CUtensorMap map_w,
                                                                  const __grid_constant__ CUtensorMap map_xd,
                                                                  const __grid_constant__ CUtensorMap map_xc,
                                                                  const SkinnyArgs g) {
    using L = Layout<NP>;
    constexpr int NB = L::NB, NS = L::NS, EW = L::EW, EB = L::EB;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sb = smem_u32(base);
    uint64_t *bars = reinterpret_cast<uint64_t *>(base + L::OFF_BAR);
    uint64_t *r_full = bars, *r_empty = r_full + NR, *a_full = r_empty + NR, *a_empty = a_full + NA,
             *b_full = a_empty + NA, *b_empty = b_full + NB, *d_full = b_empty + NB, *d_empty = d_full + ND,
             *s_full = d_empty + ND, *s_empty = s_full + NS, *done = s_empty + NS;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
    volatile int *last_flag = abort + 1;
    float *dws = reinterpret_cast<float *>(base + L::OFF_DW);  // [ND][4][SN]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tile = blockIdx.x % g.tiles, split = blockIdx.x / g.tiles;
    const int n0 = tile * SN;
    const int nchunks = g.nb / 8;
    const int c0 = (int)((int64_t)split * nchunks / g.splits), c1 = (int)((int64_t)(split + 1) * nchunks / g.splits);
    const int nch = c1 - c0;

    if (warp == 1) tc05::alloc(tmem_slot, L::TMEM_COLS);
    if (tid == 0) {
        for (int i = 0; i < NR; ++i) {
            mbar_init(&r_full[i], 1);
            mbar_init(&r_empty[i], CONV_WARPS);
        }
        for (int i = 0; i < NA; ++i) {
            mbar_init(&a_full[i], 1);
            mbar_init(&a_empty[i], 1 + EPI_WARPS);  // the chunk's MMAs, and its scales read
        }
        for (int i = 0; i < NB; ++i) {
            mbar_init(&b_full[i], CONV_WARPS);
            mbar_init(&b_empty[i], 1);
        }
        for (int i = 0; i < ND; ++i) {
            mbar_init(&d_full[i], CONV_WARPS);
            mbar_init(&d_empty[i], EPI_WARPS);
        }
        for (int i = 0; i < NS; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&s_empty[i], EPI_WARPS);
        }
        mbar_init(done, 1);
        *abort = 0;
        *last_flag = 0;
        fence_mbar_init();
        tc05::prefetch_map(&map_a);
        tc05::prefetch_map(&map_w);
        tc05::prefetch_map(&map_xd);
        tc05::prefetch_map(&map_xc);
    }
    tc05::fence_before();
    __syncthreads();
    tc05::fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();
    pdl_wait();

    if (warp == 0) {
        // ---------------- producer: activation codes, scales and offsets, raw weight chunks
        if (lane == 0) {
            int a_issued = 0, r_issued = 0;
            for (int c = 0; c < nch && !*abort; ++c) {
                const int as = c % NA, rs = c % NR, k0 = (c0 + c) * 256;
                if (c >= NA && !wait_or_abort(&a_empty[as], ((c / NA) - 1) & 1, abort, g.err)) break;
                const uint32_t slot = sb + L::OFF_A + as * L::ASLOT;
                mbar_arrive_expect_tx(&a_full[as], L::ASLOT);
                tc05::tma_load_2d(slot, &map_a, k0, 0, &a_full[as]);
                tc05::tma_load_2d(slot + L::APANEL, &map_a, k0 + 128, 0, &a_full[as]);
                tc05::tma_load_2d(slot + 2 * L::APANEL, &map_xd, (c0 + c) * 8, 0, &a_full[as]);
                tc05::tma_load_2d(slot + 2 * L::APANEL + L::XT, &map_xc, (c0 + c) * 8, 0, &a_full[as]);
                ++a_issued;
                if (c >= NR && !wait_or_abort(&r_empty[rs], ((c / NR) - 1) & 1, abort, g.err)) break;
                mbar_arrive_expect_tx(&r_full[rs], RAW);
                tc05::tma_load_2d(sb + L::OFF_R + rs * RAW, &map_w, (c0 + c) * 144, n0, &r_full[rs]);
                ++r_issued;
            }
            // Drain: the last copy issued into each slot has landed.
            for (int c = a_issued > NA ? a_issued - NA : 0; c < a_issued; ++c)
                if (!mbar_wait(&a_full[c % NA], (c / NA) & 1)) record_device_error(g.err, DEV_ERR_DRAIN);
            for (int c = r_issued > NR ? r_issued - NR : 0; c < r_issued; ++c)
                if (!mbar_wait(&r_full[c % NR], (c / NR) & 1)) record_device_error(g.err, DEV_ERR_DRAIN);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_i8(SN, NP, false, true);
            bool ok = true;
            for (int c = 0; c < nch && ok; ++c) {
                if (!wait_or_abort(&a_full[c % NA], (c / NA) & 1, abort, g.err)) break;
                for (int q = 0; q < 2 && ok; ++q) {
                    const int p = 2 * c + q;
                    if (!wait_or_abort(&b_full[p % NB], (p / NB) & 1, abort, g.err)) {
                        ok = false;
                        break;
                    }
                    const uint32_t wb = sb + L::OFF_W + (p % NB) * WPANEL;
                    const uint32_t ab = sb + L::OFF_A + (c % NA) * L::ASLOT + q * L::APANEL;
                    for (int h = 0; h < 4; ++h) {
                        const int i = 4 * p + h, s = i % NS;
                        // EB consecutive blocks form one epilogue group in EB
                        // consecutive accumulators: the group's slots are free
                        // once its last one is released, and its MMAs are done
                        // once the last one's commit lands (one issuing thread:
                        // a commit tracks every earlier MMA of it)
                        const int il = i + EB - 1;
                        if (i % EB == 0 && i >= NS &&
                            !wait_or_abort(&s_empty[il % NS], ((il / NS) - 1) & 1, abort, g.err)) {
                            ok = false;
                            break;
                        }
                        tc05::fence_after();
                        mma_i8(tmem + s * NP, tc05::desc_sw128(wb + 32 * h, 16, 1024),
                               tc05::desc_sw128(ab + 32 * h, 16, 1024), idesc);
                        if (i % EB == EB - 1) tc05::commit(&s_full[s]);
                    }
                    if (!ok) break;
                    tc05::commit(&b_empty[p % NB]);
                }
                if (ok) tc05::commit(&a_empty[c % NA]);
            }
            tc05::commit(done);
            if (!mbar_wait(done, 0)) record_device_error(g.err, DEV_ERR_DRAIN);
        }
    } else if (warp < 2 + CONV_WARPS) {
        // ---------------- converters: thread ct owns weight row n0 + ct of the tile
        const int ct = tid - 64;
        bool ok = true;
        for (int c = 0; c < nch && ok; ++c) {
            const int rs = c % NR;
            if (!__all_sync(0xffffffffu, wait_or_abort(&r_full[rs], (c / NR) & 1, abort, g.err))) break;
            // the row's 8 blocks: 144 bytes, 16-byte aligned rows
            uint32_t raw[36];
            const uint32_t row = sb + L::OFF_R + rs * RAW + ct * 144;
#pragma unroll
            for (int i = 0; i < 9; ++i)
                ld_shared_v4(row + 16 * i, raw[4 * i], raw[4 * i + 1], raw[4 * i + 2], raw[4 * i + 3]);
            __syncwarp();
            if (lane == 0) mbar_arrive(&r_empty[rs]);
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const int p = 2 * c + q;
                ok = __all_sync(0xffffffffu,
                                (p < NB || wait_or_abort(&b_empty[p % NB], ((p / NB) - 1) & 1, abort, g.err)) &&
                                    (p < ND || wait_or_abort(&d_empty[p % ND], ((p / ND) - 1) & 1, abort, g.err)));
                if (!ok) break;
                const uint32_t prow = sb + L::OFF_W + (p % NB) * WPANEL + ct * 128;
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    const int b = 4 * q + h, w0 = (18 * b) / 4;  // block b starts at byte 18 b
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
                    // byte j of qs: element j in the low nibble, element j + 16
                    // in the high one; 16-byte chunks 2h (elements 0-15) and
                    // 2h + 1 (16-31) of the row, swizzled
                    st_shared_v4(prow + (((2 * h) ^ (ct & 7)) << 4), w[0] & 0x0F0F0F0Fu, w[1] & 0x0F0F0F0Fu,
                                 w[2] & 0x0F0F0F0Fu, w[3] & 0x0F0F0F0Fu);
                    st_shared_v4(prow + (((2 * h + 1) ^ (ct & 7)) << 4), (w[0] >> 4) & 0x0F0F0F0Fu,
                                 (w[1] >> 4) & 0x0F0F0F0Fu, (w[2] >> 4) & 0x0F0F0F0Fu, (w[3] >> 4) & 0x0F0F0F0Fu);
                    dws[((p % ND) * 4 + h) * SN + ct] = half_bits_to_f32(d);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&b_full[p % NB]);
                    mbar_arrive(&d_full[p % ND]);
                }
            }
        }
    } else {
        // ---------------- epilogue: thread = weight row = TMEM lane; the two
        // warps of a lane quarter take half of the activation rows each
        const int ew = warp - (2 + CONV_WARPS), quad = warp & 3, half = ew >> 2;
        const int r = quad * 32 + lane, col0 = half * EW;
        const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + col0;
        const int M = g.M;
        float acc[EW];
#pragma unroll
        for (int j = 0; j < EW; ++j) acc[j] = 0.0f;
        bool ok = true;
        for (int c = 0; c < nch && ok; ++c) {
            ok = __all_sync(0xffffffffu, wait_or_abort(&a_full[c % NA], (c / NA) & 1, abort, g.err));
            if (!ok) break;
            // the chunk's activation scales and offsets, [NP rows][8 blocks]
            const float *xdt = reinterpret_cast<const float *>(base + L::OFF_A + (c % NA) * L::ASLOT + 2 * L::APANEL);
            const float *xct = xdt + NP * 8;
            for (int q = 0; q < 2 && ok; ++q) {
                const int p = 2 * c + q;
                ok = __all_sync(0xffffffffu, wait_or_abort(&d_full[p % ND], (p / ND) & 1, abort, g.err));
                if (!ok) break;
                for (int hb = 0; hb < 4; hb += EB) {
                    // one wait for the group (its last block's commit covers the
                    // group's earlier MMAs) and one release (the issuer waits on
                    // the group's last slot before reusing any of its slots)
                    const int il = 4 * p + hb + EB - 1;
                    ok = __all_sync(0xffffffffu, wait_or_abort(&s_full[il % NS], (il / NS) & 1, abort, g.err));
                    if (!ok) break;
                    tc05::fence_after();
                    uint32_t dv[EB][EW];
#pragma unroll
                    for (int e = 0; e < EB; ++e) tmem_ld<EW>(taddr + ((4 * p + hb + e) % NS) * NP, dv[e]);
                    tc05::wait_ld();
                    tc05::fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&s_empty[il % NS]);
                    float dw[EB];
#pragma unroll
                    for (int e = 0; e < EB; ++e) dw[e] = dws[((p % ND) * 4 + hb + e) * SN + r];
                    const int b0 = 4 * q + hb;  // first block of this group within the chunk
#pragma unroll
                    for (int j = 0; j < EW; ++j) {
                        if (col0 + j >= M) break;
                        float xd[EB], xc[EB];
                        if constexpr (EB == 4) {
                            const float4 a = *reinterpret_cast<const float4 *>(xdt + (col0 + j) * 8 + b0);
                            const float4 o = *reinterpret_cast<const float4 *>(xct + (col0 + j) * 8 + b0);
                            xd[0] = a.x, xd[1] = a.y, xd[2] = a.z, xd[3] = a.w;
                            xc[0] = o.x, xc[1] = o.y, xc[2] = o.z, xc[3] = o.w;
                        } else {
                            const float2 a = *reinterpret_cast<const float2 *>(xdt + (col0 + j) * 8 + b0);
                            const float2 o = *reinterpret_cast<const float2 *>(xct + (col0 + j) * 8 + b0);
                            xd[0] = a.x, xd[1] = a.y;
                            xc[0] = o.x, xc[1] = o.y;
                        }
#pragma unroll
                        for (int e = 0; e < EB; ++e) {
                            // D is an exact s32 of magnitude below 2^16: its bits
                            // added to 12582912's give 12582912 + D exactly, and
                            // minus the offset 12582912 + 8 sum(q8) leaves isum
                            const float isum = __uint_as_float(dv[e][j] + kMagicBits) - xc[e];
                            acc[j] = fmaf(isum * dw[e], xd[e], acc[j]);
                        }
                    }
                }
                if (!ok) break;
                __syncwarp();
                if (lane == 0) mbar_arrive(&d_empty[p % ND]);
            }
            if (!ok) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(&a_empty[c % NA]);
        }
        // ---------------- output
        const int n = n0 + r;
        bool write = ok;
        if (g.splits > 1) {
            // every epilogue thread reaches both barriers, whatever happened above
            if (ok && n < g.N) {
#pragma unroll
                for (int j = 0; j < EW; ++j) {
                    if (col0 + j >= M) break;
                    g.part[((int64_t)split * M + col0 + j) * g.N + n] = acc[j];
                }
            }
            __threadfence();
            asm volatile("bar.sync 2, %0;" ::"r"(EPI_WARPS * 32) : "memory");
            if (ew == 0 && lane == 0) {
                __threadfence();
                const int t = atomicAdd(&g.tickets[tile], 1);
                const int last = (t == g.splits - 1) ? 1 : 0;
                if (last) {
                    g.tickets[tile] = 0;  // ready for the next launch
                    __threadfence();
                }
                *last_flag = last;
            }
            asm volatile("bar.sync 2, %0;" ::"r"(EPI_WARPS * 32) : "memory");
            write = *last_flag != 0;
            if (write && n < g.N) {
#pragma unroll
                for (int j = 0; j < EW; ++j) {
                    if (col0 + j >= M) break;
                    float v = 0.0f;
                    for (int sp = 0; sp < g.splits; ++sp)
                        v += __ldcg(g.part + ((int64_t)sp * M + col0 + j) * g.N + n);
                    acc[j] = v;
                }
            }
        }
        if (write) {
            if (g.pairs) {
                // rows n (gate, even) and n + 1 (up) sit in lanes 2i and 2i + 1:
                // each projection rounded to bf16 as nn.Linear's output would
                // be, then LlamaMLP's act = bf16(bf16(silu(gate)) * up) to
                // column n / 2
                const float bn = (g.bias && n < g.N) ? __ldg(g.bias + n) : 0.0f;
#pragma unroll
                for (int j = 0; j < EW; ++j) {
                    if (col0 + j >= M) break;
                    const float t = acc[j] + bn;
                    const float u = __shfl_xor_sync(0xffffffffu, t, 1);
                    if ((lane & 1) == 0 && n < g.N) {
                        const float gg = bfr(t), up = bfr(u);
                        const float a = bfr(bfr(gg / (1.0f + expf(-gg))) * up);
                        store_out(g.y, g.y_dtype, (col0 + j) * g.y_row_stride + (n >> 1), a);
                    }
                }
            } else if (n < g.N) {
                const float bn = g.bias ? __ldg(g.bias + n) : 0.0f;
#pragma unroll
                for (int j = 0; j < EW; ++j) {
                    if (col0 + j >= M) break;
                    store_out(g.y, g.y_dtype, (col0 + j) * g.y_row_stride + n, acc[j] + bn);
                }
            }
        }
    }

    tc05::fence_before();
    __syncthreads();
    if (warp == 1) {
        tc05::fence_after();
        tc05::dealloc(tmem, L::TMEM_COLS);
    }
}

template <int NP>
int launch_np(const CUtensorMap (&maps)[4], const SkinnyArgs &g, int grid, cudaStream_t stream) {
    const char *op = "torch._C._quantized_linear";
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    const size_t smem = Layout<NP>::SMEM;
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        int st = check_cuda(cudaFuncSetAttribute(q4_skinny_kernel<NP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)smem),
                            op, "cudaFuncSetAttribute");
        if (st) return st;
        configured[dev] = 1;
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(SK_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return check_cuda(cudaLaunchKernelEx(&cfg, q4_skinny_kernel<NP>, maps[0], maps[1], maps[2], maps[3], g), op,
                      "cudaLaunchKernelEx (q4 skinny)");
}

}  // namespace

bool q4_skinny_applies(const void *w_blob, const float *xd, const float *xc, int64_t M, int64_t N, int64_t K,
                       int flags) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(w_blob) | reinterpret_cast<uintptr_t>(xd) |
                        reinterpret_cast<uintptr_t>(xc);
    return M >= kQ4SkinnyMinRows && M <= kQ4SkinnyMaxRows && K % 256 == 0 && K > 0 && N > 0 && (a & 15) == 0 &&
           (N + SN - 1) / SN <= (1 << 24) && (!(flags & TN_EPILOGUE_SILU_MUL_PAIRS) || N % 2 == 0);
}

int launch_q4_skinny(const int8_t *xq, int64_t xq_row_stride, const float *xd, const float *xc, const uint8_t *w,
                     const float *bias, void *y, int y_dtype, int64_t y_row_stride, int M, int64_t N, int64_t K,
                     int flags, cudaStream_t stream) {
    const char *op = "torch._C._quantized_linear";
    DeviceFacts f{};
    int st = device_facts(&f);
    if (st) return st;
    const int64_t nb = K / 32, rowbytes = nb * 18;
    const int NP = M <= 16 ? 16 : 32;
    // codes (NP rows x 128, swizzled), raw weight rows (128 x 144 bytes), and
    // the activation scales and offsets (NP rows x 8 blocks of f32)
    CUtensorMap maps[4];
    st = encode_map_2d(&maps[0], xq, 1, (uint64_t)K, (uint64_t)M, (uint64_t)xq_row_stride, 128, (uint32_t)NP, true);
    if (st) return st;
    st = encode_map_2d(&maps[1], w, 1, (uint64_t)rowbytes, (uint64_t)N, (uint64_t)rowbytes, 144, SN, false);
    if (st) return st;
    st = encode_map_2d(&maps[2], xd, 4, (uint64_t)nb, (uint64_t)M, (uint64_t)nb * 4, 8, (uint32_t)NP, false);
    if (st) return st;
    st = encode_map_2d(&maps[3], xc, 4, (uint64_t)nb, (uint64_t)M, (uint64_t)nb * 4, 8, (uint32_t)NP, false);
    if (st) return st;
    SkinnyArgs g{};
    g.bias = bias;
    g.y = y;
    g.y_dtype = y_dtype;
    g.y_row_stride = y_row_stride;
    g.M = M;
    g.N = (int)N;
    g.nb = (int)nb;
    g.pairs = (flags & TN_EPILOGUE_SILU_MUL_PAIRS) ? 1 : 0;
    g.err = device_error_word();
    g.tiles = (int)((N + SN - 1) / SN);
    // Splits of K so that up to two CTAs per SM stream weights in one wave
    // (each split at least one 256-wide chunk).
    const int nchunks = (int)(K / 256);
    int splits = (2 * f.sm_count) / g.tiles;
    if (splits > nchunks) splits = nchunks;
    if (splits < 1) splits = 1;
    g.splits = splits;
    if (splits > 1) {
        void *ws = nullptr;
        st = workspace(&ws, (size_t)splits * M * N * sizeof(float) + 256, stream, /*slot=*/4);
        if (st) return st;
        g.part = static_cast<float *>(ws);
        void *cnt = nullptr;
        st = workspace_zeroed(&cnt, (size_t)g.tiles * sizeof(int) + 256, stream, /*slot=*/5);
        if (st) return st;
        g.tickets = static_cast<int *>(cnt);
    }
    const int64_t grid = (int64_t)g.tiles * splits;
    if (grid > 0x7fffffff) return set_error(TN_ERR_SHAPE, std::string(op) + ": too many output rows");
    st = NP == 16 ? launch_np<16>(maps, g, (int)grid, stream) : launch_np<32>(maps, g, (int)grid, stream);
    if (st) return st;
    __atomic_fetch_add(&counters().q4_skinny_launches, 1ull, __ATOMIC_RELAXED);
    return TN_OK;
}

}  // namespace tn
