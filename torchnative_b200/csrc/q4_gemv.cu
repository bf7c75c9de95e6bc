// q4_gemv.cu -- decode Q4_0 linear (M <= 16 activation rows), the reference's
// Q8_0-activation arithmetic, streamed from HBM with bulk-async (TMA) copies.
//
// Work split. CTA c of G owns output columns (weight rows) [c*N/G, (c+1)*N/G).
// One producer lane streams those weight rows -- each row is K/32 GGML blocks
// of 18 bytes, rowbytes = 18*K/32 contiguous bytes -- into a ring of shared
// memory slots with cp.async.bulk (one copy per row, completion counted on the
// slot's mbarrier). Eight consumer warps take rows two at a time (rows 2q and
// 2q+1 for q = warp, warp+8, ...): two independent accumulation chains per
// lane, and every activation load serves both rows. A warp splits a row's
// blocks across its 32 lanes in pairs (36 bytes = 9 words; 9 is odd, so the 32
// lanes hit 32 different banks), takes exact integer block dots with dp4a
// against the Q8_0 activation codes held in shared memory, and applies the
// per-block scales in float32. A reduce-scatter shuffle butterfly sums lanes.
//
// Arithmetic (reference: k_quants.rs:312-330 vec_dot_unopt). Per block b:
//   I_b = sum_j (q4_j - 8) * q8_j                 exact int32
//   t_b = I_b * (d_w * d_x)                        d_w*d_x is exact in f32 (11+11 bits)
// The int -> float step is a magic-number add folded into dp4a's accumulator
// (bits 0x4B400000 + I read as float = 12582912 + I, exact for |I| < 2^22), and
// the "-8" offset is folded into the subtracted constant xc = 12582912 + 8*sum(q8).
// Each lane accumulates its blocks with fmaf (one rounding per block), then a
// 5-level shuffle tree: depth ceil(nb/64)*2 + 5 <= nb + 3 for nb >= 2, the
// depth the reference's own bound counts (scripts/q4quality/q4_gguf_ref.py:370-405).
#include "q4_kernels.cuh"

namespace tn {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kMaxSlots = 32;
constexpr uint32_t kMagic = 0x4B400000u;           // 12582912.0f
// Shared memory per CTA when two CTAs share an SM (228 KB per SM, 1 KB of it
// reserved per CTA).
constexpr size_t kTwoCtaBudget = 112 * 1024;
// Output columns a CTA may hold for the planar Q8_0 epilogue (whole 32-column
// blocks), per activation row.
constexpr int kYCap = 128;

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
    int rowbytes; // 18 * nb (Q4_0 weights) or 34 * nb (Q8_0 weights)
    int wpc;      // consumer warps per chunk (a chunk is rpw * wpc rows)
    int rpw;      // weight rows per consumer warp in a chunk: 2, or 1 for rows too long to stage two per warp
    int slot_bytes;
    int nslots;
    int flags;
    int *err;
    // Activation source (x_mode): X_PLANAR reads xq/xd/xc; the others build the
    // planar Q8_0 tile in shared memory from bf16 rows (M <= 4), every CTA the
    // same bytes from the same inputs.
    int x_mode;
    const __nv_bfloat16 *xb;     // X_BF16: x; X_NORM: h; X_SILU: [gate | up] rows
    const __nv_bfloat16 *xdelta; // X_NORM: residual delta (or null)
    __nv_bfloat16 *xh_out;       // X_NORM: h + delta is written here by CTA 0 (never == xb)
    const __nv_bfloat16 *xw;     // X_NORM: RMSNorm weight
    float eps;
    int64_t xb_row_stride;       // elements
    // Tensor parallelism (tn_tp_link): scatter the output into every rank's
    // exchange region (tp_slot >= 0) and/or wait for a gathered input.
    // tp_reduce: row-parallel linear, the all-reduce of its f32 partials
    // fused in (every CTA stores its columns' partials into every rank's
    // region, then sums the same columns of every rank's partials into y).
    int tp_world, tp_rank, tp_slot, tp_wait, tp_reduce;
    int64_t tp_dst_off, tp_dst_row, tp_cols;
    uint8_t *tp_bases[kTpMaxRanks];
    // Planar Q8_0 of y (oq != null): every CTA owns whole 32-column blocks of
    // y, keeps its bf16 outputs in shared memory and quantises them after its
    // last row.
    int8_t *oq;
    float *od, *oc;
    int64_t oq_row_stride;
    int wfmt;  // weight format: 0 = Q4_0 (18-byte blocks), 1 = Q8_0 (34-byte blocks), 2 = Q4_K (144 per 256)
};

// Shared-memory layout (dynamic), as 32-bit shared-window addresses:
//   bars  full[kMaxSlots], empty[kMaxSlots] mbarriers
//   xs    M * nbp * 32 bytes      activation codes, pair-swizzled (xchunk)
//   xds   M * nbp floats          widened activation scales
//   xcs   M * nbp floats          offset constants
//   ys    M * kYCap floats        this CTA's outputs (planar Q8_0 epilogue only)
//   slots nslots * slot_bytes     chunks of 2*wpc weight rows (16-byte aligned)
struct Smem {
    uint64_t *full, *empty;
    uint32_t xs, xds, xcs, ys, slots;
};

__device__ __forceinline__ Smem carve(uint8_t *base, const GemvParams &p) {
    Smem s;
    s.full = reinterpret_cast<uint64_t *>(base);
    s.empty = s.full + kMaxSlots;
    const uint32_t b = smem_u32(base);
    uint32_t off = 16 * kMaxSlots;
    s.xs = b + off;
    off += (uint32_t)p.M * p.nbp * 32;
    s.xds = b + off;
    off += (uint32_t)p.M * p.nbp * 4;
    s.xcs = b + off;
    off += (uint32_t)p.M * p.nbp * 4;
    s.ys = b + off;
    if (p.oq) off += (uint32_t)p.M * kYCap * 4;
    off = (off + 127) & ~127u;
    s.slots = b + off;
    return s;
}

__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ int4 lds128(uint32_t a) {
    int4 v;
    asm volatile("ld.shared.v4.s32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ float2 lds64f(uint32_t a) {
    float2 v;
    asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ float ldsf(uint32_t a) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ void sts128(uint32_t a, int4 v) {
    asm volatile("st.shared.v4.s32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}
__device__ __forceinline__ void stsf(uint32_t a, float v) {
    asm volatile("st.shared.f32 [%0], %1;" ::"r"(a), "f"(v) : "memory");
}

// Byte offset of 16-byte chunk c (0..3) of block pair `pair` inside one
// activation row of the staged codes. Chunks 0/1 are the low/high 16 codes of
// block 2*pair, chunks 2/3 those of block 2*pair+1. The XOR spreads the eight
// lanes of a quarter-warp (which read pairs l..l+7) over all eight 16-byte bank
// groups, so every 128-bit load below is conflict-free.
__device__ __forceinline__ uint32_t xchunk(int pair, int c) {
    return (uint32_t)(pair * 64 + 16 * (c ^ ((pair >> 1) & 3)));
}

// One Q4_0 block, unpacked: low and high nibbles of its 16 code bytes (values
// 0..15, element j and element j+16 of the block), and its f16 scale.
struct Blk {
    uint32_t lo[4], hi[4];
    float d;
};

__device__ __forceinline__ Blk unpack(uint32_t q0, uint32_t q1, uint32_t q2, uint32_t q3, uint32_t dbits) {
    Blk b;
    const uint32_t q[4] = {q0, q1, q2, q3};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        b.lo[i] = q[i] & 0x0F0F0F0Fu;
        b.hi[i] = (q[i] >> 4) & 0x0F0F0F0Fu;
    }
    b.d = half_bits_to_f32(dbits);
    return b;
}

// 12582912 + sum_j nibble_j * x_j, exactly, as float bits.
__device__ __forceinline__ float magic_dot(const Blk &w, int4 xl, int4 xh) {
    int I = (int)kMagic;
    I = __dp4a((int)w.lo[0], xl.x, I);
    I = __dp4a((int)w.lo[1], xl.y, I);
    I = __dp4a((int)w.lo[2], xl.z, I);
    I = __dp4a((int)w.lo[3], xl.w, I);
    I = __dp4a((int)w.hi[0], xh.x, I);
    I = __dp4a((int)w.hi[1], xh.y, I);
    I = __dp4a((int)w.hi[2], xh.z, I);
    I = __dp4a((int)w.hi[3], xh.w, I);
    return __int_as_float(I);
}

// Accumulate blocks b0 = 2*pair and b1 = 2*pair + 1 of up to two rows (A, B)
// against every activation row m < M.
template <int MT, bool TWO>
__device__ __forceinline__ void pair_dot(const Blk &a0, const Blk &a1, const Blk &b0, const Blk &b1, int pair,
                                         const Smem &s, const GemvParams &p, float (&acc)[2][MT]) {
    const uint32_t xrow = (uint32_t)p.nbp * 32;
    const uint32_t c0 = xchunk(pair, 0), c1 = xchunk(pair, 1), c2 = xchunk(pair, 2), c3 = xchunk(pair, 3);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        if (m < p.M) {
            const uint32_t xb = s.xs + m * xrow;
            const int4 x0 = lds128(xb + c0), x1 = lds128(xb + c1), x2 = lds128(xb + c2), x3 = lds128(xb + c3);
            const uint32_t so = (uint32_t)(m * p.nbp + 2 * pair) * 4;
            const float2 xd = lds64f(s.xds + so), xc = lds64f(s.xcs + so);
            acc[0][m] = fmaf(magic_dot(a0, x0, x1) - xc.x, a0.d * xd.x, acc[0][m]);
            acc[0][m] = fmaf(magic_dot(a1, x2, x3) - xc.y, a1.d * xd.y, acc[0][m]);
            if (TWO) {
                acc[1][m] = fmaf(magic_dot(b0, x0, x1) - xc.x, b0.d * xd.x, acc[1][m]);
                acc[1][m] = fmaf(magic_dot(b1, x2, x3) - xc.y, b1.d * xd.y, acc[1][m]);
            }
        }
    }
}

// Single-block variant for the unstaged path (block b of rows A and B).
template <int MT, bool TWO>
__device__ __forceinline__ void single_dot(const Blk &a, const Blk &bb, int b, const Smem &s, const GemvParams &p,
                                           float (&acc)[2][MT]) {
    const uint32_t xrow = (uint32_t)p.nbp * 32;
    const int pair = b >> 1, cb = (b & 1) * 2;
    const uint32_t cl = xchunk(pair, cb), ch = xchunk(pair, cb + 1);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        if (m < p.M) {
            const uint32_t xb = s.xs + m * xrow;
            const int4 xl = lds128(xb + cl), xh = lds128(xb + ch);
            const uint32_t so = (uint32_t)(m * p.nbp + b) * 4;
            const float xd = ldsf(s.xds + so), xc = ldsf(s.xcs + so);
            acc[0][m] = fmaf(magic_dot(a, xl, xh) - xc, a.d * xd, acc[0][m]);
            if (TWO) acc[1][m] = fmaf(magic_dot(bb, xl, xh) - xc, bb.d * xd, acc[1][m]);
        }
    }
}

// Q8_0 weights (BlockQ8_0, k_quants.rs:652-756): 32 signed codes and an f16
// scale per block. The block dot is the same exact integer as for Q4_0 (signed
// dp4a, |sum| <= 32 * 127 * 127 < 2^22, so the magic-number sum is exact) and
// needs no code-sum offset: subtract the magic constant itself.
struct Blk8 {
    uint32_t c[8];  // codes 0-15 in c[0..3], codes 16-31 in c[4..7]
    float d;
};
constexpr float kMagicF = 12582912.0f;

__device__ __forceinline__ float magic_dot8(const Blk8 &w, int4 xl, int4 xh) {
    int I = (int)kMagic;
    I = __dp4a((int)w.c[0], xl.x, I);
    I = __dp4a((int)w.c[1], xl.y, I);
    I = __dp4a((int)w.c[2], xl.z, I);
    I = __dp4a((int)w.c[3], xl.w, I);
    I = __dp4a((int)w.c[4], xh.x, I);
    I = __dp4a((int)w.c[5], xh.y, I);
    I = __dp4a((int)w.c[6], xh.z, I);
    I = __dp4a((int)w.c[7], xh.w, I);
    return __int_as_float(I);
}

template <int MT, bool TWO>
__device__ __forceinline__ void pair_dot8(const Blk8 &a0, const Blk8 &a1, const Blk8 &b0, const Blk8 &b1, int pair,
                                          const Smem &s, const GemvParams &p, float (&acc)[2][MT]) {
    const uint32_t xrow = (uint32_t)p.nbp * 32;
    const uint32_t c0 = xchunk(pair, 0), c1 = xchunk(pair, 1), c2 = xchunk(pair, 2), c3 = xchunk(pair, 3);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        if (m < p.M) {
            const uint32_t xb = s.xs + m * xrow;
            const int4 x0 = lds128(xb + c0), x1 = lds128(xb + c1), x2 = lds128(xb + c2), x3 = lds128(xb + c3);
            const float2 xd = lds64f(s.xds + (uint32_t)(m * p.nbp + 2 * pair) * 4);
            acc[0][m] = fmaf(magic_dot8(a0, x0, x1) - kMagicF, a0.d * xd.x, acc[0][m]);
            acc[0][m] = fmaf(magic_dot8(a1, x2, x3) - kMagicF, a1.d * xd.y, acc[0][m]);
            if (TWO) {
                acc[1][m] = fmaf(magic_dot8(b0, x0, x1) - kMagicF, b0.d * xd.x, acc[1][m]);
                acc[1][m] = fmaf(magic_dot8(b1, x2, x3) - kMagicF, b1.d * xd.y, acc[1][m]);
            }
        }
    }
}

template <int MT, bool TWO>
__device__ __forceinline__ void single_dot8(const Blk8 &a, const Blk8 &bb, int b, const Smem &s, const GemvParams &p,
                                            float (&acc)[2][MT]) {
    const uint32_t xrow = (uint32_t)p.nbp * 32;
    const int pair = b >> 1, cb = (b & 1) * 2;
    const uint32_t cl = xchunk(pair, cb), ch = xchunk(pair, cb + 1);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        if (m < p.M) {
            const uint32_t xb = s.xs + m * xrow;
            const int4 xl = lds128(xb + cl), xh = lds128(xb + ch);
            const float xd = ldsf(s.xds + (uint32_t)(m * p.nbp + b) * 4);
            acc[0][m] = fmaf(magic_dot8(a, xl, xh) - kMagicF, a.d * xd, acc[0][m]);
            if (TWO) acc[1][m] = fmaf(magic_dot8(bb, xl, xh) - kMagicF, bb.d * xd, acc[1][m]);
        }
    }
}

__device__ __forceinline__ float bfr(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ int sat_i8r(float v) {
    if (!(v == v)) return 0;
    if (v <= -128.0f) return -128;
    if (v >= 127.0f) return 127;
    return __float2int_rz(v);
}

// One Q8_0 block (k_quants.rs:676-706) quantised by two adjacent lanes (lane
// pair 2i, 2i + 1), each holding 16 of its values (`half` 0: elements 0-15,
// 1: 16-31), written into the staged planar tile (codes as two 16-byte chunks
// in the pair-swizzled layout, then the widened scale and the offset
// constant). The block maximum and the code sum cross the pair by shuffles.
__device__ __forceinline__ void q8_half_block_to_smem(const float (&v)[16], int m, int b, int half, const Smem &s,
                                                      const GemvParams &p, int lane) {
    const unsigned pm = 3u << (lane & ~1);
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(v[j]));
    amax = fmaxf(amax, __shfl_xor_sync(pm, amax, 1));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = (d != 0.0f) ? __fdiv_rn(1.0f, d) : 0.0f;
    uint32_t w[4];
    int sum = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        uint32_t word = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int q = sat_i8r(roundf(__fmul_rn(v[4 * k + e], id)));
            sum += q;
            word |= (uint32_t)(q & 0xff) << (8 * e);
        }
        w[k] = word;
    }
    sum += __shfl_xor_sync(pm, sum, 1);
    const int pair = b >> 1, c = (b & 1) * 2 + half;
    const uint32_t row = s.xs + (uint32_t)m * p.nbp * 32;
    sts128(row + xchunk(pair, c), make_int4((int)w[0], (int)w[1], (int)w[2], (int)w[3]));
    if (half == 0) {
        stsf(s.xds + (uint32_t)(m * p.nbp + b) * 4, __half2float(__float2half_rn(d)));
        stsf(s.xcs + (uint32_t)(m * p.nbp + b) * 4, 12582912.0f + 8.0f * (float)sum);
    }
}

// 8 consecutive bf16 values (one 16-byte load; rows are 16-byte aligned) as f32.
__device__ __forceinline__ void load8_bf16(const __nv_bfloat16 *src, float *v) {
    const int4 r = __ldg(reinterpret_cast<const int4 *>(src));
    const uint32_t u[4] = {(uint32_t)r.x, (uint32_t)r.y, (uint32_t)r.z, (uint32_t)r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        v[2 * i] = __uint_as_float(u[i] << 16);
        v[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
    }
}

// Packed bf16 pairs (element 2i in the low half of word i, 2i+1 in the high).
__device__ __forceinline__ uint32_t bf2_bits(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t *>(&v); }
__device__ __forceinline__ __nv_bfloat162 bf2_of(uint32_t u) { return *reinterpret_cast<__nv_bfloat162 *>(&u); }
__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

// q8_half_block_to_smem for 16 values that are bf16 already (as 8 packed
// pairs): the same codes, scale and offset, with the block maximum taken on
// the packed magnitudes (exact), the codes packed by byte permutes and their
// sum by one dp4a per word.
__device__ __forceinline__ void q8_half_block_bf16_to_smem(const uint32_t (&v)[8], int m, int b, int half,
                                                           const Smem &s, const GemvParams &p, int lane) {
    const unsigned pm = 3u << (lane & ~1);
    __nv_bfloat162 mx = bf2_of(v[0] & 0x7fff7fffu);
#pragma unroll
    for (int i = 1; i < 8; ++i) mx = __hmax2(mx, bf2_of(v[i] & 0x7fff7fffu));
    const uint32_t mb = bf2_bits(mx);
    float amax = fmaxf(bf_lo(mb), bf_hi(mb));
    amax = fmaxf(amax, __shfl_xor_sync(pm, amax, 1));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = (d != 0.0f) ? __fdiv_rn(1.0f, d) : 0.0f;
    uint32_t w[4];
    int sum = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int q0 = sat_i8r(roundf(__fmul_rn(bf_lo(v[2 * k]), id)));
        const int q1 = sat_i8r(roundf(__fmul_rn(bf_hi(v[2 * k]), id)));
        const int q2 = sat_i8r(roundf(__fmul_rn(bf_lo(v[2 * k + 1]), id)));
        const int q3 = sat_i8r(roundf(__fmul_rn(bf_hi(v[2 * k + 1]), id)));
        w[k] = __byte_perm(__byte_perm((uint32_t)q0, (uint32_t)q1, 0x0040), __byte_perm((uint32_t)q2, (uint32_t)q3, 0x0040),
                           0x5410);
        sum = __dp4a((int)w[k], 0x01010101, sum);
    }
    sum += __shfl_xor_sync(pm, sum, 1);
    const int pair = b >> 1, c = (b & 1) * 2 + half;
    const uint32_t row = s.xs + (uint32_t)m * p.nbp * 32;
    sts128(row + xchunk(pair, c), make_int4((int)w[0], (int)w[1], (int)w[2], (int)w[3]));
    if (half == 0) {
        stsf(s.xds + (uint32_t)(m * p.nbp + b) * 4, __half2float(__float2half_rn(d)));
        stsf(s.xcs + (uint32_t)(m * p.nbp + b) * 4, 12582912.0f + 8.0f * (float)sum);
    }
}

enum : int { X_PLANAR = 0, X_BF16 = 1, X_NORM = 2, X_SILU = 3 };
constexpr int kMaxFusedRows = 4;

// Build the planar Q8_0 tile from bf16 rows, one 32-element block per thread:
// x itself (X_BF16), transformers' RMSNorm of h + delta (X_NORM: w * bf16(x *
// rsqrt(mean(x^2) + eps)), x = bf16(h + delta)), or bf16(bf16(silu(g)) * u)
// (X_SILU). Consumer threads only; `red` is kMaxFusedRows * kConsumerWarps
// floats of shared scratch.
template <int MT, int XM>
__device__ __forceinline__ void stage_x_fused(const Smem &s, const GemvParams &p, int tid, int warp, int lane,
                                              float *red) {
    const int K = p.nb * 32, nthr = kConsumerWarps * 32;
    if (XM == X_NORM && 2 * p.nb <= nthr) {
        // The decode case (K <= 16 x consumer threads): half a block per
        // thread and row (lanes 2i, 2i + 1 share block i). Every load of
        // every row is issued before the first use and the values stay in
        // registers across the CTA-wide reduction, so the prologue costs one
        // L2 round trip whatever the row count.
        // h = bf16(x + delta) as packed pairs: a correctly rounded bf16 sum is
        // the f32 sum rounded to bf16 (the exact sum of two bf16 values either
        // fits in f32 or differs from the larger by less than a quarter bf16
        // ulp), so __hadd2 gives transformers' bits
        constexpr int R = MT < kMaxFusedRows ? MT : kMaxFusedRows;
        const int b = tid >> 1, hf = tid & 1, e0 = b * 32 + 16 * hf;
        uint32_t hb[R][8], wp[8];
        float ss[R];
#pragma unroll
        for (int m = 0; m < R; ++m) ss[m] = 0.0f;
        if (b < p.nb) {
            int4 xr[R][2], dr[R][2], wr[2];
#pragma unroll
            for (int c = 0; c < 2; ++c) wr[c] = __ldg(reinterpret_cast<const int4 *>(p.xw + e0) + c);
#pragma unroll
            for (int m = 0; m < R; ++m) {
                if (m >= p.M) continue;
                const int64_t o = m * p.xb_row_stride + e0;
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    xr[m][c] = __ldg(reinterpret_cast<const int4 *>(p.xb + o) + c);
                    dr[m][c] = p.xdelta ? __ldg(reinterpret_cast<const int4 *>(p.xdelta + o) + c)
                                        : make_int4(0, 0, 0, 0);
                }
            }
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                wp[4 * c] = (uint32_t)wr[c].x;
                wp[4 * c + 1] = (uint32_t)wr[c].y;
                wp[4 * c + 2] = (uint32_t)wr[c].z;
                wp[4 * c + 3] = (uint32_t)wr[c].w;
            }
#pragma unroll
            for (int m = 0; m < R; ++m) {
                if (m >= p.M) continue;
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const uint32_t xu[4] = {(uint32_t)xr[m][c].x, (uint32_t)xr[m][c].y, (uint32_t)xr[m][c].z,
                                            (uint32_t)xr[m][c].w};
                    const uint32_t du[4] = {(uint32_t)dr[m][c].x, (uint32_t)dr[m][c].y, (uint32_t)dr[m][c].z,
                                            (uint32_t)dr[m][c].w};
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        hb[m][4 * c + i] = p.xdelta ? bf2_bits(__hadd2(bf2_of(xu[i]), bf2_of(du[i]))) : xu[i];
                }
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float lo = bf_lo(hb[m][i]), hi = bf_hi(hb[m][i]);
                    ss[m] = fmaf(lo, lo, ss[m]);
                    ss[m] = fmaf(hi, hi, ss[m]);
                }
            }
        }
#pragma unroll
        for (int m = 0; m < R; ++m) {
            if (m >= p.M) continue;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) ss[m] += __shfl_xor_sync(0xffffffffu, ss[m], off);
            if (lane == 0) red[m * kConsumerWarps + warp] = ss[m];
        }
        asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
        float r[R];
#pragma unroll
        for (int m = 0; m < R; ++m) {
            float t = 0.0f;
            if (m < p.M)
#pragma unroll
                for (int w = 0; w < kConsumerWarps; ++w) t += red[m * kConsumerWarps + w];
            r[m] = rsqrtf(t / (float)K + p.eps);
        }
        if (b < p.nb) {
#pragma unroll
            for (int m = 0; m < R; ++m) {
                if (m >= p.M) continue;
                if (p.xh_out && blockIdx.x == 0) {
                    int4 *dst = reinterpret_cast<int4 *>(p.xh_out + m * p.xb_row_stride + e0);
#pragma unroll
                    for (int c = 0; c < 2; ++c)
                        dst[c] = make_int4((int)hb[m][4 * c], (int)hb[m][4 * c + 1], (int)hb[m][4 * c + 2],
                                           (int)hb[m][4 * c + 3]);
                }
                // w * bf16(h * r): the f32 products rounded to bf16 in one
                // packed convert, then one correctly rounded bf16 product per
                // pair (a product of two bf16 values is exact in f32, so it
                // equals bf16(f32 product))
                uint32_t v[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const __nv_bfloat162 hr = __floats2bfloat162_rn(bf_lo(hb[m][i]) * r[m], bf_hi(hb[m][i]) * r[m]);
                    v[i] = bf2_bits(__hmul2(bf2_of(wp[i]), hr));
                }
                q8_half_block_bf16_to_smem(v, m, b, hf, s, p, lane);
            }
        } else if (b < p.nbp) {
            float z[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) z[j] = 0.0f;
#pragma unroll
            for (int m = 0; m < R; ++m)
                if (m < p.M) q8_half_block_to_smem(z, m, b, hf, s, p, lane);
        }
        return;
    }
    float rinv[kMaxFusedRows] = {1.0f, 1.0f, 1.0f, 1.0f};
    if constexpr (XM == X_NORM) {
        float ss[kMaxFusedRows] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int m = 0; m < kMaxFusedRows; ++m) {
            if (m < p.M) {
                for (int b = tid; b < p.nb; b += nthr) {
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        float x[8], dl[8];
                        load8_bf16(p.xb + m * p.xb_row_stride + b * 32 + 8 * c, x);
                        if (p.xdelta) load8_bf16(p.xdelta + m * p.xb_row_stride + b * 32 + 8 * c, dl);
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const float h = p.xdelta ? bfr(x[j] + dl[j]) : x[j];
                            ss[m] = fmaf(h, h, ss[m]);
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int m = 0; m < kMaxFusedRows; ++m) {
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) ss[m] += __shfl_xor_sync(0xffffffffu, ss[m], off);
            if (lane == 0) red[m * kConsumerWarps + warp] = ss[m];
        }
        asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
#pragma unroll
        for (int m = 0; m < kMaxFusedRows; ++m) {
            float t = 0.0f;
            for (int w = 0; w < kConsumerWarps; ++w) t += red[m * kConsumerWarps + w];
            rinv[m] = rsqrtf(t / (float)K + p.eps);
        }
    }
    // half a block per task: (b, hf) = (t / 2, t % 2); lane pairs hold one
    // block. One loop per mode, every load of a task issued before its math.
#pragma unroll
    for (int m = 0; m < kMaxFusedRows; ++m) {
        if (m >= p.M) continue;
        const __nv_bfloat16 *xrow = p.xb + m * p.xb_row_stride;
        for (int t = tid; t < 2 * p.nbp; t += nthr) {
            const int b = t >> 1, hf = t & 1, e0 = b * 32 + 16 * hf;
            float v[16];
            if (b >= p.nb) {  // padding block of an odd block count
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = 0.0f;
            } else if constexpr (XM == X_BF16) {
                load8_bf16(xrow + e0, v);
                load8_bf16(xrow + e0 + 8, v + 8);
            } else if constexpr (XM == X_NORM) {
                float dl[16], w[16];
                load8_bf16(xrow + e0, v);
                load8_bf16(xrow + e0 + 8, v + 8);
                if (p.xdelta) {
                    load8_bf16(p.xdelta + m * p.xb_row_stride + e0, dl);
                    load8_bf16(p.xdelta + m * p.xb_row_stride + e0 + 8, dl + 8);
                }
                load8_bf16(p.xw + e0, w);
                load8_bf16(p.xw + e0 + 8, w + 8);
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const float h = p.xdelta ? bfr(v[j] + dl[j]) : v[j];
                    if (p.xh_out && blockIdx.x == 0) p.xh_out[m * p.xb_row_stride + e0 + j] = __float2bfloat16_rn(h);
                    v[j] = bfr(w[j] * bfr(h * rinv[m]));
                }
            } else {  // X_SILU: rows are [gate (K) | up (K)]
                float u[16];
                load8_bf16(xrow + e0, v);
                load8_bf16(xrow + e0 + 8, v + 8);
                load8_bf16(xrow + K + e0, u);
                load8_bf16(xrow + K + e0 + 8, u + 8);
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = bfr(bfr(v[j] / (1.0f + expf(-v[j]))) * u[j]);
            }
            q8_half_block_to_smem(v, m, b, hf, s, p, lane);
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
        sts128(s.xs + (uint32_t)m * p.nbp * 32 + xchunk(pair, c), v);
    }
    for (int idx = tid; idx < p.M * p.nbp; idx += nthr) {
        const int m = idx / p.nbp, b = idx % p.nbp;
        stsf(s.xds + idx * 4, b < p.nb ? __ldg(p.xd + (int64_t)m * p.nb + b) : 0.0f);
        stsf(s.xcs + idx * 4, b < p.nb ? __ldg(p.xc + (int64_t)m * p.nb + b) : 12582912.0f);
    }
}

// The tag of this launch's row-parallel reduction (epoch * 256 + slot + 1):
// set by consumer thread 0 before the main loop, read by every store and
// every poll of the reduction.
__shared__ uint32_t g_red_tag;

__device__ __forceinline__ void st_relaxed_sys_u64(uint8_t *p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint8_t *p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Output column n of row m: into y, or (tensor-parallel producer) into this
// rank's columns of the gathered buffer in its exchange region.
__device__ __forceinline__ void store_y(const GemvParams &p, int m, int64_t n, float v) {
    if (p.tp_slot < 0) {
        store_out(p.y, p.y_dtype, m * p.y_row_stride + n, v);
        return;
    }
    if (p.tp_reduce) {
        // this rank's f32 partial with its use tag in one 8-byte word, straight
        // into every rank's region (peer stores over NVLink): a reader that
        // sees the tag sees the value, so no fence and no separate signal
        const int64_t off = kTpDataOff + p.tp_dst_off + (m * p.tp_dst_row + (int64_t)p.tp_rank * p.tp_cols + n) * 8;
        const uint64_t word = ((uint64_t)g_red_tag << 32) | __float_as_uint(v);
        for (int g = 0; g < p.tp_world; ++g) st_relaxed_sys_u64(p.tp_bases[g] + off, word);
        return;
    }
    // this rank's own region only; the launch's last CTA pushes the finished
    // slice to the other ranks in 16-byte pieces
    const int64_t idx = m * p.tp_dst_row + (int64_t)p.tp_rank * p.tp_cols + n;
    store_out(p.tp_bases[p.tp_rank] + kTpDataOff + p.tp_dst_off, p.y_dtype, idx, v);
}

// Reduce-scatter across the warp: V = 2*MT values per lane (row r, column m at
// index r*MT + m). After log2(V) butterfly levels each lane holds a partial of
// one value, index lane >> (5 - log2 V); the remaining levels finish the sum.
template <int MT>
__device__ __forceinline__ void finish_rows(float (&acc)[2][MT], const GemvParams &p, int64_t n0, bool has_b,
                                            int lane, const Smem &s, int64_t ycol0) {
    constexpr int V = 2 * MT;
    constexpr int LOGV = (V == 2) ? 1 : (V == 4) ? 2 : (V == 8) ? 3 : (V == 16) ? 4 : 5;
    float v[V];
#pragma unroll
    for (int i = 0; i < V; ++i) v[i] = acc[i / MT][i % MT];
#pragma unroll
    for (int k = 0; k < LOGV; ++k) {
        const int off = 16 >> k;
        const bool upper = (lane & off) != 0;
        const int half = V >> (k + 1);
#pragma unroll
        for (int i = 0; i < half; ++i) {
            const float send = upper ? v[i] : v[i + half];
            const float keep = upper ? v[i + half] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
    }
    float t = v[0];
#pragma unroll
    for (int off = 16 >> LOGV; off > 0; off >>= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
    const int idx = lane >> (5 - LOGV);
    const int r = idx / MT, m = idx % MT;
    if (p.flags & TN_EPILOGUE_SILU_MUL_PAIRS) {
        // Rows n0 (gate) and n0 + 1 (up) of an interleaved gate/up weight: the
        // lanes holding up's totals sit 16 above gate's. Each projection is
        // rounded to bf16 as nn.Linear's output would be, then LlamaMLP's
        // act = bf16(bf16(silu(gate)) * up) goes to column n0 / 2.
        if (p.bias) t = t + __ldg(p.bias + n0 + r);
        const float u = __shfl_down_sync(0xffffffffu, t, 16);
        if ((lane & ((1 << (5 - LOGV)) - 1)) == 0 && r == 0 && m < p.M) {
            const float g = bfr(t), up = bfr(u);
            const float a = bfr(bfr(g / (1.0f + expf(-g))) * up);
            store_y(p, m, n0 >> 1, a);
            if (p.oq) stsf(s.ys + (uint32_t)(m * kYCap + ((n0 >> 1) - ycol0)) * 4, a);
        }
        return;
    }
    if ((lane & ((1 << (5 - LOGV)) - 1)) == 0 && m < p.M && (r == 0 || has_b)) {
        const int64_t n = n0 + r;
        if (p.bias) t = t + __ldg(p.bias + n);
        store_y(p, m, n, t);
        if (p.oq) stsf(s.ys + (uint32_t)(m * kYCap + (n - ycol0)) * 4, bfr(t));
    }
}

// 16-bit little-endian loads of one 18-byte block from global memory (the
// unstaged path: K % 256 != 0, so rows are not 16-byte multiples).
__device__ __forceinline__ Blk load_block_global(const uint8_t *blk) {
    const unsigned short *h = reinterpret_cast<const unsigned short *>(blk);
    uint32_t u[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) u[i] = __ldg(h + i);
    return unpack(u[1] | (u[2] << 16), u[3] | (u[4] << 16), u[5] | (u[6] << 16), u[7] | (u[8] << 16), u[0]);
}

// One 34-byte Q8_0 block from global memory, as 17 little-endian halves.
__device__ __forceinline__ Blk8 load_block8_global(const uint8_t *blk) {
    const unsigned short *h = reinterpret_cast<const unsigned short *>(blk);
    uint32_t u[17];
#pragma unroll
    for (int i = 0; i < 17; ++i) u[i] = __ldg(h + i);
    Blk8 b;
#pragma unroll
    for (int i = 0; i < 8; ++i) b.c[i] = u[1 + 2 * i] | (u[2 + 2 * i] << 16);
    b.d = half_bits_to_f32(u[0]);
    return b;
}

// Staged Q8_0 rows: a pair of blocks is 68 bytes = 17 aligned words. Block
// 2*pair: scale in the low half of word 0, codes straddling words 0..8 (funnel
// shifts); block 2*pair+1: scale in the high half of word 8, codes in words
// 9..16.
__device__ __forceinline__ void unpack8_pair(const uint32_t (&w)[17], Blk8 &b0, Blk8 &b1) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        b0.c[i] = __funnelshift_r(w[i], w[i + 1], 16);
        b1.c[i] = w[9 + i];
    }
    b0.d = half_bits_to_f32(w[0] & 0xffffu);
    b1.d = half_bits_to_f32(w[8] >> 16);
}

template <int MT, bool TWO>
__device__ __forceinline__ void staged_rows8(const Smem &s, const GemvParams &p, uint32_t rowA, uint32_t rowB,
                                             int lane, float (&acc)[2][MT]) {
    const int npairs = p.nb >> 1;
    for (int pp = lane; pp < npairs; pp += 32) {
        const uint32_t a = rowA + pp * 68, b = rowB + pp * 68;
        uint32_t wa[17], wb[17];
#pragma unroll
        for (int i = 0; i < 17; ++i) wa[i] = lds32(a + 4 * i);
        if (TWO) {
#pragma unroll
            for (int i = 0; i < 17; ++i) wb[i] = lds32(b + 4 * i);
        }
        Blk8 a0, a1, b0, b1;
        unpack8_pair(wa, a0, a1);
        if (TWO) {
            unpack8_pair(wb, b0, b1);
        } else {
            b0 = a0;
            b1 = a1;
        }
        pair_dot8<MT, TWO>(a0, a1, b0, b1, pp, s, p, acc);
    }
}

template <int MT, bool TWO>
__device__ __forceinline__ void global_rows8(const Smem &s, const GemvParams &p, const uint8_t *rowA,
                                             const uint8_t *rowB, int lane, float (&acc)[2][MT]) {
    for (int b = lane; b < p.nb; b += 32) {
        const Blk8 a = load_block8_global(rowA + b * 34);
        const Blk8 bb = TWO ? load_block8_global(rowB + b * 34) : a;
        single_dot8<MT, TWO>(a, bb, b, s, p, acc);
    }
}

// Q4_K weights (BlockQ4K, k_quants.rs:153-159; dot product :1478-1544): a lane
// takes sub-block pair c (64 elements) of super-block sb at a time -- the
// super-block's 16-byte header (f16 d, f16 dmin, 6-bit scales/mins) and its
// 32 nibble bytes -- against the staged Q8_K codes of 32-blocks 8 sb + 2c and
// + 1 (the same block pair the Q4_0 path reads), whose staged scale is the
// super-block's d and whose "offset" slot holds the block's code sum. Per
// pair: acc += (d_w d_x) * (sc0 i0 + sc1 i1) - (dmin_w d_x) * (m0 s0 + m1 s1),
// both integer sums exact in f32.
template <int MT, bool TWO>
__device__ __forceinline__ void staged_rows_k(const Smem &s, const GemvParams &p, uint32_t rowA, uint32_t rowB,
                                              int lane, float (&acc)[2][MT]) {
    const int nsp = p.nb >> 1;  // sub-block pairs per row
    const uint32_t xrow = (uint32_t)p.nbp * 32;
    for (int sp = lane; sp < nsp; sp += 32) {
        const int sb = sp >> 2, c = sp & 3;
        int4 hdr[2], qa[2], qb[2];
#pragma unroll
        for (int r = 0; r < (TWO ? 2 : 1); ++r) {
            const uint32_t base = (r ? rowB : rowA) + (uint32_t)sb * 144u;
            hdr[r] = lds128(base);
            qa[r] = lds128(base + 16u + 32u * c);
            qb[r] = lds128(base + 32u + 32u * c);
        }
        const uint32_t c0 = xchunk(sp, 0), c1 = xchunk(sp, 1), c2 = xchunk(sp, 2), c3 = xchunk(sp, 3);
#pragma unroll
        for (int r = 0; r < (TWO ? 2 : 1); ++r) {
            const uint32_t W0 = (uint32_t)hdr[r].y, W1 = (uint32_t)hdr[r].z, W2 = (uint32_t)hdr[r].w;
            const float dw = half_bits_to_f32((uint32_t)hdr[r].x & 0xffffu), dmw = half_bits_to_f32((uint32_t)hdr[r].x >> 16);
            // get_scale_min_k4 (quantized/utils.rs:50-60) for sub-blocks j0 = 2c, j1 = 2c + 1
            const bool hi = c >= 2;
            const uint32_t scw = hi ? ((W2 & 0x0f0f0f0fu) | (((W0 >> 6) & 0x03030303u) << 4)) : (W0 & 0x3f3f3f3fu);
            const uint32_t mnw = hi ? (((W2 >> 4) & 0x0f0f0f0fu) | (((W1 >> 6) & 0x03030303u) << 4)) : (W1 & 0x3f3f3f3fu);
            const int sh = 16 * (c & 1);
            const int sc0 = (int)((scw >> sh) & 0xffu), sc1 = (int)((scw >> (sh + 8)) & 0xffu);
            const int m0 = (int)((mnw >> sh) & 0xffu), m1 = (int)((mnw >> (sh + 8)) & 0xffu);
            const uint32_t q[8] = {(uint32_t)qa[r].x, (uint32_t)qa[r].y, (uint32_t)qa[r].z, (uint32_t)qa[r].w,
                                   (uint32_t)qb[r].x, (uint32_t)qb[r].y, (uint32_t)qb[r].z, (uint32_t)qb[r].w};
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                if (m < p.M) {
                    const uint32_t xb = s.xs + m * xrow;
                    const int4 x0 = lds128(xb + c0), x1 = lds128(xb + c1), x2 = lds128(xb + c2), x3 = lds128(xb + c3);
                    const uint32_t xl[8] = {(uint32_t)x0.x, (uint32_t)x0.y, (uint32_t)x0.z, (uint32_t)x0.w,
                                            (uint32_t)x1.x, (uint32_t)x1.y, (uint32_t)x1.z, (uint32_t)x1.w};
                    const uint32_t xh[8] = {(uint32_t)x2.x, (uint32_t)x2.y, (uint32_t)x2.z, (uint32_t)x2.w,
                                            (uint32_t)x3.x, (uint32_t)x3.y, (uint32_t)x3.z, (uint32_t)x3.w};
                    int i0 = 0, i1 = 0;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        i0 = __dp4a((int)(q[i] & 0x0F0F0F0Fu), (int)xl[i], i0);
                        i1 = __dp4a((int)((q[i] >> 4) & 0x0F0F0F0Fu), (int)xh[i], i1);
                    }
                    const uint32_t so = (uint32_t)(m * p.nbp + 2 * sp) * 4;
                    const float2 xd = lds64f(s.xds + so), xs2 = lds64f(s.xcs + so);
                    const float S = (float)(sc0 * i0 + sc1 * i1);
                    const float Mv = fmaf((float)m1, xs2.y, (float)m0 * xs2.x);
                    acc[r][m] = fmaf(dw * xd.x, S, acc[r][m]);
                    acc[r][m] = fmaf(-(dmw * xd.x), Mv, acc[r][m]);
                }
            }
        }
    }
}

template <int MT, bool TWO>
__device__ __forceinline__ void staged_rows(const Smem &s, const GemvParams &p, uint32_t rowA, uint32_t rowB,
                                            int lane, float (&acc)[2][MT]) {
    const int npairs = p.nb >> 1;
    for (int pp = lane; pp < npairs; pp += 32) {
        const uint32_t a = rowA + pp * 36, b = rowB + pp * 36;
        uint32_t wa[9], wb[9];
#pragma unroll
        for (int i = 0; i < 9; ++i) wa[i] = lds32(a + 4 * i);
        if (TWO) {
#pragma unroll
            for (int i = 0; i < 9; ++i) wb[i] = lds32(b + 4 * i);
        }
        const Blk a0 = unpack(__funnelshift_r(wa[0], wa[1], 16), __funnelshift_r(wa[1], wa[2], 16),
                              __funnelshift_r(wa[2], wa[3], 16), __funnelshift_r(wa[3], wa[4], 16), wa[0] & 0xffffu);
        const Blk a1 = unpack(wa[5], wa[6], wa[7], wa[8], wa[4] >> 16);
        Blk b0 = a0, b1 = a1;
        if (TWO) {
            b0 = unpack(__funnelshift_r(wb[0], wb[1], 16), __funnelshift_r(wb[1], wb[2], 16),
                        __funnelshift_r(wb[2], wb[3], 16), __funnelshift_r(wb[3], wb[4], 16), wb[0] & 0xffffu);
            b1 = unpack(wb[5], wb[6], wb[7], wb[8], wb[4] >> 16);
        }
        pair_dot<MT, TWO>(a0, a1, b0, b1, pp, s, p, acc);
    }
}

template <int MT, bool TWO>
__device__ __forceinline__ void global_rows(const Smem &s, const GemvParams &p, const uint8_t *rowA,
                                            const uint8_t *rowB, int lane, float (&acc)[2][MT]) {
    for (int b = lane; b < p.nb; b += 32) {
        const Blk a = load_block_global(rowA + b * 18);
        const Blk bb = TWO ? load_block_global(rowB + b * 18) : a;
        single_dot<MT, TWO>(a, bb, b, s, p, acc);
    }
}

// WF: weight format, 0 = Q4_0, 1 = Q8_0, 2 = Q4_K.
template <int MT, bool STAGED, int XM, int WF>
__global__ void __launch_bounds__(kThreads, (MT <= 8) ? 2 : 1) q4_gemv_q8_kernel(const GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const Smem s = carve(smem_raw, p);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t G = gridDim.x, c = blockIdx.x;
    // (gate, up) row pairs never straddle two CTAs: partition in pairs then;
    // with the planar Q8_0 epilogue, in whole 32-column blocks of y
    const bool pairs = (p.flags & TN_EPILOGUE_SILU_MUL_PAIRS) != 0;
    const int64_t gran = (pairs ? 2 : 1) * (p.oq ? 32 : 1);
    const int64_t r0 = c * (p.N / gran) / G * gran, r1 = (c + 1) * (p.N / gran) / G * gran;
    const int nrows = (int)(r1 - r0);
    const int64_t ycol0 = pairs ? r0 >> 1 : r0;
    // Chunks of R = rpw * wpc consecutive rows; chunk j lives in slot j % nslots
    // and is consumed by warp group j % groups (wpc warps, two rows each).
    const int wpc = p.wpc, R = p.rpw * p.wpc, groups = kConsumerWarps / p.wpc;
    const int nchunks = (nrows + R - 1) / R;

    if (STAGED && threadIdx.x == 0) {
        for (int i = 0; i < p.nslots; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], (uint32_t)wpc);
        }
        fence_mbar_init();
    }
    __syncthreads();
    // Let the next kernel in the stream be scheduled now: it waits for this
    // grid's completion (griddepcontrol.wait) before it reads anything this
    // grid writes, and until then only prefetches its own static weights.
    if (threadIdx.x == 0) pdl_launch_dependents();

    if (warp == kConsumerWarps) {
        // ---------------- producer: one lane streams this CTA's weight rows,
        // one bulk copy per chunk (the CTA's rows are contiguous in the blob).
        if (STAGED && lane == 0) {
            // Unless the caller vouches that nothing queued before this call
            // writes the weights (TN_WEIGHTS_STATIC), wait for the previous
            // kernel like the consumers do; otherwise start streaming weights
            // while it finishes.
            if (!(p.flags & TN_WEIGHTS_STATIC)) pdl_wait();
            const uint64_t pol = policy_evict_first();
            int issued = 0;
            for (int j = 0; j < nchunks; ++j) {
                const int slot = j % p.nslots, use = j / p.nslots;
                if (use > 0 && !mbar_wait(&s.empty[slot], (use - 1) & 1)) {
                    record_device_error(p.err, DEV_ERR_WAIT_EMPTY);
                    break;
                }
                const int rows = min(R, nrows - j * R);
                const uint32_t bytes = (uint32_t)rows * (uint32_t)p.rowbytes;
                mbar_arrive_expect_tx(&s.full[slot], bytes);
                bulk_g2s_hint_u32(s.slots + (uint32_t)slot * p.slot_bytes, p.w + (r0 + (int64_t)j * R) * p.rowbytes,
                                  bytes, &s.full[slot], pol);
                issued = j + 1;
            }
            // Drain: every copy issued must have landed before the CTA exits.
            // (On the normal path the consumers already waited for all of them.)
            for (int j = issued > p.nslots ? issued - p.nslots : 0; j < issued; ++j) {
                if (!mbar_wait(&s.full[j % p.nslots], (j / p.nslots) & 1)) {
                    record_device_error(p.err, DEV_ERR_DRAIN);
                    break;
                }
            }
        }
        return;
    }

    // ---------------- consumers
    pdl_wait();  // the activations may come from the previous kernel in the stream
    if (p.tp_reduce && threadIdx.x == 0)  // (visible to the other consumers after the staging barrier)
        g_red_tag = (uint32_t)ld_acquire_sys(reinterpret_cast<const int *>(p.tp_bases[p.tp_rank] + kTpEpochOff)) *
                        (uint32_t)kTpRedSlots + (uint32_t)p.tp_slot + 1u;
    if (p.tp_wait >= 0) {  // gathered activations: every rank's producer has signalled this step
        if (threadIdx.x == 0) {
            const uint8_t *lb = p.tp_bases[p.tp_rank];
            const int epoch = ld_acquire_sys(reinterpret_cast<const int *>(lb + kTpEpochOff));
            tp_wait_counts(lb, p.tp_wait, p.tp_world, epoch + 1, p.err);
        }
        asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
    }
    if constexpr (XM == X_PLANAR) {
        stage_x(s, p, threadIdx.x, kConsumerWarps * 32);
    } else {
        __shared__ float red[kMaxFusedRows * kConsumerWarps];
        stage_x_fused<MT, XM>(s, p, threadIdx.x, warp, lane, red);
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");

    const int group = warp / wpc, gw = warp % wpc;
    bool failed = false;
    for (int j = group; j < nchunks && !failed; j += groups) {
        const int i = j * R + p.rpw * gw;  // my first row within the CTA's range
        const bool has_a = i < nrows, has_b = p.rpw == 2 && i + 1 < nrows;
        float acc[2][MT];
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int m = 0; m < MT; ++m) acc[r][m] = 0.0f;
        if (STAGED) {
            const int slot = j % p.nslots;
            if (!mbar_wait(&s.full[slot], (j / p.nslots) & 1)) {
                record_device_error(p.err, DEV_ERR_WAIT_FULL);
                failed = true;
                break;
            }
            const uint32_t ra = s.slots + (uint32_t)slot * p.slot_bytes + (uint32_t)(p.rpw * gw) * p.rowbytes;
            if constexpr (WF == 1) {
                if (has_b)
                    staged_rows8<MT, true>(s, p, ra, ra + p.rowbytes, lane, acc);
                else if (has_a)
                    staged_rows8<MT, false>(s, p, ra, ra, lane, acc);
            } else if constexpr (WF == 2) {
                if (has_b)
                    staged_rows_k<MT, true>(s, p, ra, ra + p.rowbytes, lane, acc);
                else if (has_a)
                    staged_rows_k<MT, false>(s, p, ra, ra, lane, acc);
            } else {
                if (has_b)
                    staged_rows<MT, true>(s, p, ra, ra + p.rowbytes, lane, acc);
                else if (has_a)
                    staged_rows<MT, false>(s, p, ra, ra, lane, acc);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.empty[slot]);
        } else if (has_a) {
            const uint8_t *ra = p.w + (r0 + i) * (int64_t)p.rowbytes;
            if constexpr (WF == 1) {
                if (has_b)
                    global_rows8<MT, true>(s, p, ra, ra + p.rowbytes, lane, acc);
                else
                    global_rows8<MT, false>(s, p, ra, ra, lane, acc);
            } else if constexpr (WF == 2) {
                // Q4_K launches are always staged (16-byte aligned rows of 144-byte super-blocks)
            } else {
                if (has_b)
                    global_rows<MT, true>(s, p, ra, ra + p.rowbytes, lane, acc);
                else
                    global_rows<MT, false>(s, p, ra, ra, lane, acc);
            }
        }
        if (has_a) finish_rows<MT>(acc, p, r0 + i, has_b, lane, s, ycol0);
    }
    if (p.oq) {
        // Planar Q8_0 of this CTA's blocks of y, from the bf16 values it
        // stored (q8_0_quantize_planar's arithmetic: k_quants.rs:676-706), one
        // warp per (row, block), one element per lane.
        asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
        const int nblk = (pairs ? nrows >> 1 : nrows) / 32;
        const int64_t nbo = (pairs ? p.N >> 1 : p.N) / 32, blk0 = ycol0 / 32;
        for (int t = warp; t < p.M * nblk; t += kConsumerWarps) {
            const int m = t / nblk, bl = t % nblk;
            float v;
            asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(s.ys + (uint32_t)(m * kYCap + bl * 32 + lane) * 4));
            // the largest |v| (NaN counts as 0, as fmaxf skips it): non-negative
            // floats order like their bit patterns
            const float av = fabsf(v);
            const float amax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(av == av ? av : 0.0f)));
            const float d = __fdiv_rn(amax, 127.0f);
            const float id = (d != 0.0f) ? __fdiv_rn(1.0f, d) : 0.0f;
            const int q = sat_i8r(roundf(__fmul_rn(v, id)));
            const int sum = __reduce_add_sync(0xffffffffu, q);
            p.oq[m * p.oq_row_stride + (blk0 + bl) * 32 + lane] = (int8_t)q;
            if (lane == 0) {
                p.od[m * nbo + blk0 + bl] = __half2float(__float2half_rn(d));
                p.oc[m * nbo + blk0 + bl] = 12582912.0f + 8.0f * (float)sum;
            }
        }
    }
    if (p.tp_slot >= 0 && p.tp_reduce) {
        // Row-parallel all-reduce of this CTA's columns: poll every rank's
        // tagged partial word of each (row, column) until it carries this
        // launch's tag (bounded), and sum rank 0's + rank 1's + ... in that
        // order -- the same bits on every rank. A wait that gives up records
        // the error; the others then stop at once and y is left unwritten.
        const int nthr = kConsumerWarps * 32;
        const uint32_t tag = g_red_tag;
        const uint8_t *part = p.tp_bases[p.tp_rank] + kTpDataOff + p.tp_dst_off;
        const long long budget = wait_budget(p.err);
        bool ok = true;
        for (int t = threadIdx.x; t < p.M * nrows && ok; t += nthr) {
            const int m = t / nrows;
            const int64_t n = r0 + t % nrows;
            float acc = 0.0f;
            for (int g = 0; g < p.tp_world; ++g) {
                const uint8_t *w = part + (m * p.tp_dst_row + (int64_t)g * p.tp_cols + n) * 8;
                uint64_t x = ld_relaxed_sys_u64(w);
                if ((uint32_t)(x >> 32) != tag) {
                    const long long start = clock64();
                    while ((uint32_t)(x >> 32) != tag) {
                        if ((p.err && *reinterpret_cast<volatile int *>(p.err) != 0) || clock64() - start > budget) {
                            record_device_error(p.err, DEV_ERR_WAIT_FULL);
                            ok = false;
                            break;
                        }
                        x = ld_relaxed_sys_u64(w);
                    }
                    if (!ok) break;
                }
                acc += __uint_as_float((uint32_t)x);
            }
            if (ok) store_out(p.y, p.y_dtype, m * p.y_row_stride + n, acc);
        }
    } else if (p.tp_slot >= 0) {
        // Every consumer's rows are stored in this rank's region. The launch's
        // last CTA (ticket) copies the whole slice to every other rank, fences
        // system-wide and signals every rank -- also after a failed wait, so
        // that peers do not stall.
        __shared__ int tp_last;
        asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
        if (threadIdx.x == 0) {
            __threadfence();
            int *ticket = reinterpret_cast<int *>(p.tp_bases[p.tp_rank] + kTpTicketOff) + p.tp_slot;
            tp_last = atomicAdd(ticket, 1) == (int)gridDim.x - 1;
            if (tp_last) {
                *ticket = 0;
                __threadfence();
            }
        }
        asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
        if (tp_last) {
            const int nthr = kConsumerWarps * 32;
            const int64_t es = p.y_dtype == TN_F32 ? 4 : 2;
            const int64_t row_b = p.tp_cols * es, col0 = (int64_t)p.tp_rank * row_b, stride_b = p.tp_dst_row * es;
            const uint8_t *src = p.tp_bases[p.tp_rank] + kTpDataOff + p.tp_dst_off;
            if (((row_b | col0 | stride_b | p.tp_dst_off) & 15) == 0) {
                const int64_t per = row_b / 16, n = (int64_t)p.M * per;
                for (int64_t i = threadIdx.x; i < n; i += nthr) {
                    const int64_t off = (i / per) * stride_b + col0 + (i % per) * 16;
                    const uint4 v = __ldcg(reinterpret_cast<const uint4 *>(src + off));
                    for (int g = 0; g < p.tp_world; ++g)
                        if (g != p.tp_rank)
                            *reinterpret_cast<uint4 *>(p.tp_bases[g] + kTpDataOff + p.tp_dst_off + off) = v;
                }
            } else {
                const int64_t per = row_b / 2, n = (int64_t)p.M * per;
                for (int64_t i = threadIdx.x; i < n; i += nthr) {
                    const int64_t off = (i / per) * stride_b + col0 + (i % per) * 2;
                    const unsigned short v = __ldcg(reinterpret_cast<const unsigned short *>(src + off));
                    for (int g = 0; g < p.tp_world; ++g)
                        if (g != p.tp_rank)
                            *reinterpret_cast<unsigned short *>(p.tp_bases[g] + kTpDataOff + p.tp_dst_off + off) = v;
                }
            }
            asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
            if (threadIdx.x == 0) {
                __threadfence_system();
                for (int g = 0; g < p.tp_world; ++g)
                    atomicAdd_system(reinterpret_cast<int *>(p.tp_bases[g] + kTpCountOff) +
                                         p.tp_slot * p.tp_world + p.tp_rank,
                                     1);
            }
        }
    }
}

template <int MT, bool STAGED, int XM, int WF = 0>
int launch_variant(const GemvParams &p, int grid, size_t smem, cudaStream_t stream) {
    static int configured_for[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && configured_for[dev] < (int)smem) {
        int st = check_cuda(cudaFuncSetAttribute(q4_gemv_q8_kernel<MT, STAGED, XM, WF>,
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
    int st = check_cuda(cudaLaunchKernelEx(&cfg, q4_gemv_q8_kernel<MT, STAGED, XM, WF>, p), "torch._C._quantized_linear",
                        "cudaLaunchKernelEx");
    if (st) return st;
    __atomic_fetch_add(STAGED ? &counters().q4_gemv_launches : &counters().q4_gemv_generic, 1ull, __ATOMIC_RELAXED);
    return TN_OK;
}

size_t smem_bytes(int M, int nbp, int nslots, int slot_bytes, int ycols) {
    size_t off = 16 * kMaxSlots + (size_t)M * nbp * 40 + (size_t)M * ycols * 4;
    off = (off + 127) & ~size_t(127);
    return off + (size_t)nslots * slot_bytes;
}

struct Plan {
    bool ok;
    int wpc, slot_bytes, nslots, rpw;
};

// Chunk size and ring depth. A chunk is rpw * wpc rows copied by one bulk copy:
// the largest wpc whose chunk stays within ~24 KB (many small copies in flight
// were measured to cap the fetch rate), and enough slots for ~128 KB in flight
// per SM. nslots is a multiple of the number of warp groups, so chunk j and
// chunk j - nslots belong to the same group and no warp ever waits on a slot's
// barrier more than one phase ahead (parity waits cannot tell phases two apart).
Plan plan_slots(int M, int nbp, int rowbytes, bool staged, size_t budget, size_t in_flight, int ycols = 0,
                int rpw = 2) {
    Plan pl{false, 1, 0, 0, 2};
    const size_t base = smem_bytes(M, nbp, 0, 0, ycols);
    if (!staged) {
        pl.ok = base <= budget;
        pl.wpc = kConsumerWarps / 2;
        return pl;
    }
    int wpc = kConsumerWarps;
    while (wpc > 1 && rpw * wpc * rowbytes > 24 * 1024) wpc >>= 1;
    const int groups = kConsumerWarps / wpc;
    const int slot_bytes = rpw * wpc * rowbytes;
    if (slot_bytes <= 0) return pl;  // no weight bytes to stage (K == 0): no plan
    if (base + (size_t)groups * slot_bytes > budget) return pl;
    int nslots = (int)((budget - base) / slot_bytes);
    const int want = (int)((in_flight + slot_bytes - 1) / slot_bytes);
    nslots = nslots < want ? nslots : want;
    nslots = nslots < kMaxSlots ? nslots : kMaxSlots;
    nslots = (nslots / groups) * groups;
    if (nslots < groups) return pl;
    pl = Plan{true, wpc, slot_bytes, nslots, rpw};
    return pl;
}

}  // namespace

int q4_gemv_max_rows(int64_t K, int wfmt) {
    DeviceFacts f{};
    if (device_facts(&f)) return 0;
    const int nb = (int)(K / 32), nbp = (nb + 1) & ~1;
    const int rowbytes = wfmt == 2 ? (int)(K / 256) * 144 : (wfmt ? 34 : 18) * nb;
    const bool staged = (K % 256 == 0);
    for (int mt = 16; mt >= 1; mt >>= 1) {
        if (staged && plan_slots(mt, nbp, rowbytes, true, (size_t)f.smem_optin - 1024, 128 * 1024).ok) return mt;
        if (staged && plan_slots(mt, nbp, rowbytes, true, (size_t)f.smem_optin - 1024, 128 * 1024, 0, 1).ok)
            return mt;
        // rows too long for the staged ring: the unstaged path
        if (plan_slots(mt, nbp, rowbytes, false, (size_t)f.smem_optin - 1024, 128 * 1024).ok) return mt;
    }
    return 0;
}

namespace {

int launch_gemv(GemvParams p, int M, int64_t N, int64_t K, int flags, cudaStream_t stream) {
    const char *op = "torch._C._quantized_linear";
    DeviceFacts f{};
    int st = device_facts(&f);
    if (st) return st;
    p.N = N;
    p.M = M;
    p.nb = (int)(K / 32);
    p.nbp = (p.nb + 1) & ~1;
    p.rowbytes = p.wfmt == 2 ? (int)(K / 256) * 144 : (p.wfmt ? 34 : 18) * p.nb;
    p.err = device_error_word();
    bool staged = (K % 256 == 0) && ((reinterpret_cast<uintptr_t>(p.w) & 15) == 0);
    const int ycols = p.oq ? kYCap : 0;
    // Two CTAs per SM for M <= 8 when both fit (each with ~64 KB in flight):
    // the next kernel's CTAs can then start streaming while this one's last
    // CTAs drain, and from 3 rows on the dot products, not HBM, bound one
    // CTA's 8 consumer warps -- a second CTA doubles the warps that hide
    // their latency.
    Plan plan{false, 1, 0, 0, 2};
    int ctas_per_sm = 1;
    if (M <= 8) {
        plan = plan_slots(M, p.nbp, p.rowbytes, staged, kTwoCtaBudget, 64 * 1024, ycols);
        if (plan.ok) ctas_per_sm = 2;
    }
    if (!plan.ok) plan = plan_slots(M, p.nbp, p.rowbytes, staged, (size_t)f.smem_optin - 1024, 128 * 1024, ycols);
    if (!plan.ok && staged && !(flags & TN_EPILOGUE_SILU_MUL_PAIRS))
        // Rows too long for a ring of 2 rows per consumer warp (Q8_0 weights at
        // K = 14336: 16 rows of 15 KB): one row per warp (8 rows in the ring).
        plan = plan_slots(M, p.nbp, p.rowbytes, true, (size_t)f.smem_optin - 1024, 128 * 1024, ycols, 1);
    if (!plan.ok && staged) {
        // Still too long: stream them from global memory instead.
        staged = false;
        plan = plan_slots(M, p.nbp, p.rowbytes, false, (size_t)f.smem_optin - 1024, 128 * 1024, ycols);
    }
    if (!plan.ok)
        return set_error(TN_ERR_NOT_IMPLEMENTED, std::string(op) + ": internal: activation tile too large for "
                                                                   "shared memory");
    p.wpc = plan.wpc;
    p.rpw = plan.rpw;
    p.slot_bytes = plan.slot_bytes;
    p.nslots = plan.nslots;
    p.flags = flags;
    const size_t smem = smem_bytes(M, p.nbp, plan.nslots, plan.slot_bytes, ycols);
    int64_t grid = (int64_t)f.sm_count * ctas_per_sm;
    const int64_t by_rows = (N + plan.rpw * plan.wpc - 1) / (plan.rpw * plan.wpc);
    if (by_rows < grid) grid = by_rows > 0 ? by_rows : 1;
    if (p.oq) {
        // whole blocks per CTA, at most kYCap columns of them
        const int64_t blocks = ((flags & TN_EPILOGUE_SILU_MUL_PAIRS) ? N / 2 : N) / 32;
        if (blocks < grid) grid = blocks;
        if ((blocks + grid - 1) / grid * 32 > kYCap)
            return set_error(TN_ERR_NOT_IMPLEMENTED, std::string(op) + ": too many output blocks per CTA for the "
                                                                       "planar Q8_0 epilogue");
    }
    // One kernel per (rows, staging, activation source): each holds only the
    // prologue it runs (the prologue executes once per CTA, from a cold
    // instruction cache, so its code size is latency).
#define TN_GEMV_LAUNCH(MT, XM)                                                             \
    return staged ? launch_variant<MT, true, XM>(p, (int)grid, smem, stream)               \
                  : launch_variant<MT, false, XM>(p, (int)grid, smem, stream);
#define TN_GEMV_CASE_FUSED(MT)                                                             \
    if (M <= MT) {                                                                         \
        switch (p.x_mode) {                                                                \
        case X_BF16: TN_GEMV_LAUNCH(MT, X_BF16)                                            \
        case X_NORM: TN_GEMV_LAUNCH(MT, X_NORM)                                            \
        case X_SILU: TN_GEMV_LAUNCH(MT, X_SILU)                                            \
        default: TN_GEMV_LAUNCH(MT, X_PLANAR)                                              \
        }                                                                                  \
    }
    if (p.wfmt == 2) {  // Q4_K weights: planar Q8_K activations, staged rows only
        if (p.x_mode != X_PLANAR || p.oq || !staged)
            return set_error(TN_ERR_NOT_IMPLEMENTED, std::string(op) + ": internal: Q4_K weights take planar "
                                                                       "activations and 16-byte aligned staged rows");
#define TN_GEMV_LAUNCHK(MT) return launch_variant<MT, true, X_PLANAR, 2>(p, (int)grid, smem, stream);
        if (M <= 1) TN_GEMV_LAUNCHK(1)
        if (M <= 2) TN_GEMV_LAUNCHK(2)
        if (M <= 4) TN_GEMV_LAUNCHK(4)
        if (M <= 8) TN_GEMV_LAUNCHK(8)
        if (M <= 16) TN_GEMV_LAUNCHK(16)
#undef TN_GEMV_LAUNCHK
        return set_error(TN_ERR_NOT_IMPLEMENTED, std::string(op) + ": internal: GEMV called with M > 16");
    }
    if (p.wfmt == 1) {  // Q8_0 weights: planar activations only
        if (p.x_mode != X_PLANAR || p.oq)
            return set_error(TN_ERR_NOT_IMPLEMENTED, std::string(op) + ": internal: Q8_0 weights take planar "
                                                                       "activations");
#define TN_GEMV_LAUNCH8(MT)                                                                \
    return staged ? launch_variant<MT, true, X_PLANAR, 1>(p, (int)grid, smem, stream)      \
                  : launch_variant<MT, false, X_PLANAR, 1>(p, (int)grid, smem, stream);
        if (M <= 1) TN_GEMV_LAUNCH8(1)
        if (M <= 2) TN_GEMV_LAUNCH8(2)
        if (M <= 4) TN_GEMV_LAUNCH8(4)
        if (M <= 8) TN_GEMV_LAUNCH8(8)
        if (M <= 16) TN_GEMV_LAUNCH8(16)
#undef TN_GEMV_LAUNCH8
        return set_error(TN_ERR_NOT_IMPLEMENTED, std::string(op) + ": internal: GEMV called with M > 16");
    }
    TN_GEMV_CASE_FUSED(1)
    TN_GEMV_CASE_FUSED(2)
    TN_GEMV_CASE_FUSED(4)
    if (p.x_mode != X_PLANAR)
        return set_error(TN_ERR_NOT_IMPLEMENTED, std::string(op) + ": internal: fused prologue with M > 4");
    if (M <= 8) TN_GEMV_LAUNCH(8, X_PLANAR)
    if (M <= 16) TN_GEMV_LAUNCH(16, X_PLANAR)
#undef TN_GEMV_CASE_FUSED
#undef TN_GEMV_LAUNCH
    return set_error(TN_ERR_NOT_IMPLEMENTED, std::string(op) + ": internal: GEMV called with M > 16");
}

}  // namespace

namespace {

void set_link(GemvParams &p, const tn_tp_link *link, int64_t out_cols) {
    p.tp_slot = p.tp_wait = -1;
    p.tp_world = 1;
    p.tp_reduce = 0;
    if (!link) return;
    p.tp_reduce = link->reduce;
    p.tp_world = link->world;
    p.tp_rank = link->rank;
    p.tp_slot = link->slot;
    p.tp_wait = link->wait_slot;
    p.tp_dst_off = link->dst_offset;
    p.tp_dst_row = link->dst_row_stride;
    p.tp_cols = out_cols;
    for (int g = 0; g < kTpMaxRanks; ++g) p.tp_bases[g] = g < link->world ? static_cast<uint8_t *>(link->bases[g]) : nullptr;
}

}  // namespace

int launch_q4_gemv_q8(const uint8_t *w, const int8_t *xq, const float *xd, const float *xc, int64_t xq_row_stride,
                      const float *bias, void *y, int y_dtype, int64_t y_row_stride, int M, int64_t N, int64_t K,
                      int flags, cudaStream_t stream, const tn_tp_link *link) {
    GemvParams p{};
    set_link(p, link, (flags & TN_EPILOGUE_SILU_MUL_PAIRS) ? N / 2 : N);
    p.w = w;
    p.xq = xq;
    p.xd = xd;
    p.xc = xc;
    p.bias = bias;
    p.y = y;
    p.xq_row_stride = xq_row_stride;
    p.y_row_stride = y_row_stride;
    p.y_dtype = y_dtype;
    p.x_mode = X_PLANAR;
    return launch_gemv(p, M, N, K, flags, stream);
}

int launch_q8w_gemv(const uint8_t *w, const int8_t *xq, const float *xd, const float *xc, int64_t xq_row_stride,
                    const float *bias, void *y, int y_dtype, int64_t y_row_stride, int M, int64_t N, int64_t K,
                    int flags, cudaStream_t stream) {
    GemvParams p{};
    set_link(p, nullptr, N);
    p.w = w;
    p.xq = xq;
    p.xd = xd;
    p.xc = xc;
    p.bias = bias;
    p.y = y;
    p.xq_row_stride = xq_row_stride;
    p.y_row_stride = y_row_stride;
    p.y_dtype = y_dtype;
    p.x_mode = X_PLANAR;
    p.wfmt = 1;
    return launch_gemv(p, M, N, K, flags & ~TN_EPILOGUE_SILU_MUL_PAIRS, stream);
}

int launch_q4k_gemv(const uint8_t *w, const int8_t *xq, const float *xd, const float *xc, int64_t xq_row_stride,
                    const float *bias, void *y, int y_dtype, int64_t y_row_stride, int M, int64_t N, int64_t K,
                    cudaStream_t stream) {
    GemvParams p{};
    set_link(p, nullptr, N);
    p.w = w;
    p.xq = xq;
    p.xd = xd;
    p.xc = xc;
    p.bias = bias;
    p.y = y;
    p.xq_row_stride = xq_row_stride;
    p.y_row_stride = y_row_stride;
    p.y_dtype = y_dtype;
    p.x_mode = X_PLANAR;
    p.wfmt = 2;
    return launch_gemv(p, M, N, K, TN_WEIGHTS_STATIC, stream);
}

int launch_q4_gemv_fused(int x_mode, const void *xb, int64_t xb_row_stride, const void *xdelta, void *xh_out,
                         const void *norm_w, float eps, const uint8_t *w, const float *bias, void *y, int y_dtype,
                         int64_t y_row_stride, int M, int64_t N, int64_t K, int flags, cudaStream_t stream,
                         const tn_tp_link *link, const Q8Out *q8) {
    GemvParams p{};
    set_link(p, link, (flags & TN_EPILOGUE_SILU_MUL_PAIRS) ? N / 2 : N);
    if (q8) {
        p.oq = q8->codes;
        p.od = q8->scales;
        p.oc = q8->offsets;
        p.oq_row_stride = q8->codes_row_stride;
    }
    p.w = w;
    p.bias = bias;
    p.y = y;
    p.y_row_stride = y_row_stride;
    p.y_dtype = y_dtype;
    p.x_mode = x_mode;
    p.xb = static_cast<const __nv_bfloat16 *>(xb);
    p.xdelta = static_cast<const __nv_bfloat16 *>(xdelta);
    p.xh_out = static_cast<__nv_bfloat16 *>(xh_out);
    p.xw = static_cast<const __nv_bfloat16 *>(norm_w);
    p.eps = eps;
    p.xb_row_stride = xb_row_stride;
    return launch_gemv(p, M, N, K, flags, stream);
}

}  // namespace tn
