// decode_mega.cu -- one greedy decode token of a Llama-shaped Q4_0 model at
// batch 1 as ONE persistent kernel (tn_llama_decode_*).
//
// Why one kernel. A token is 32 layers x {RMSNorm + q/k/v, RoPE + KV append +
// attention, o_proj + residual, RMSNorm + gate/up + SiLU*up, down_proj +
// residual}, then the final norm, lm_head and argmax. As separate launches
// every boundary costs the grid drain and refill (1.3-2 us each, 160 a token),
// and each launch re-reads its activations and restarts its weight stream. Here
// one CTA per SM lives for the whole token, and its weight stream never stops:
//
//   * one producer lane per CTA walks the token's whole schedule of static
//     bytes -- this CTA's rows of every weight matrix in order, and its split of
//     every layer's past K/V -- issuing cp.async.bulk copies into a ring of
//     fixed 9 KB slots (mbarrier full/empty pairs), two per consumer warp so
//     that a warp's next item streams in while it computes the current one. Those bytes never
//     depend on activations, so the producer runs ahead of the math by as much
//     as the ring holds (~200 KB per SM, ~4 us of HBM time across the GPU);
//   * 11 consumer warps wait on grid-wide phase barriers (a monotonically
//     increasing arrival counter in global memory; bounded spins) only for the
//     activations, build the phase's Q8_0 activation tile in shared memory and
//     take the dot products from the ring slots as they land.
//
// Phases per layer (B_x = grid barrier after phase x):
//   Q  RMSNorm(h) -> Q8_0 in every CTA (the whole vector: the norm's sum is
//      taken in each CTA, so no partial sums cross CTAs), q/k/v rows -> qkv_out
//   A  per (KV head, key split): q (and, in the last split, the new k) rotated,
//      new k/v appended at slot pos, online softmax over the split's K/V tiles
//      from the ring; the split's partial (m, l, o) to global memory; the last
//      split of a head to arrive (ticket) merges the head's query rows and
//      writes their bf16 output and planar Q8_0
//   O  o_proj rows over the staged codes; h[row] = bf16(h[row] + bf16(y))
//   G  RMSNorm(h) -> Q8_0; gate/up row pairs -> bf16(bf16(silu(g)) * u); each
//      CTA owns whole 32-column blocks of act and quantises them to planar Q8_0
//   D  down_proj rows; h[row] += y as in O
// then F: final RMSNorm, lm_head rows -> bf16 logits, per-CTA argmax (first
// index of the maximum), and CTA 0 reduces the partials into the next token
// and advances the position.
//
// Arithmetic is the decode GEMV's (q4_gemv.cu): exact dp4a block dots through
// the 0x4B400000 magic float, one fmaf per block with d_w * d_x, a per-lane
// chain of at most 16 blocks then a 5-level shuffle tree -- inside the
// reference's counted bound (K/32 + 3 accumulations, q4_gguf_ref.py:398-465).
// The RMSNorm prologue is the fused GEMV's packed-bf16 one, thread for thread
// (so its mean of squares is summed in the same order). Attention follows
// sdpa_flash_cpu's default arithmetic (aten.rs:10327-10420) up to the order of
// its sums: f32 scores, softmax with the row maximum, f32 accumulation.
//
// Every wait is bounded; a wait that gives up records the device error word,
// raises this launch's abort flag (seen by the other CTAs' waits) and the CTA
// drains its own copies before returning.
#include <cmath>
#include <vector>

#include "tn_common.cuh"

namespace tn {
namespace {

constexpr int kCW = 11;                   // consumer warps: one per ring slot (see consume_linear)
constexpr int kCT = kCW * 32;             // consumer threads
constexpr int kThreads = kCT + 32;        // + the producer warp
constexpr int kSlot = 9216;               // ring slot bytes (four rows of K = 4096; one bulk copy each)
constexpr int kMaxSlots = 32;
constexpr int kMaxRows = 8;               // rows per ring item (per-lane accumulators)
constexpr int kD = 128;                   // head dimension
constexpr int kRep = 4;                   // query heads per KV head
constexpr int kTile = 32;                 // keys per K or V ring item (32 x 256 B): 4 per attention warp
constexpr int kChunk = 4;                 // key tiles per online-softmax update
constexpr int kAttnWarps = 8;             // warps that take K/V tiles
constexpr int kMaxSplits = 64;            // key splits per KV head
constexpr uint32_t kMagic = 0x4B400000u;  // 12582912.0f
constexpr int kMaxK = 16384;              // in_features the activation tile holds
constexpr int kMaxUnitsG = 8;             // gate/up 64-row units per CTA

struct MegaLayer {
    const uint8_t *qkv, *o, *gate_up, *down;
    const __nv_bfloat16 *attn_norm, *mlp_norm;
    __nv_bfloat16 *kc, *vc;  // [Hkv][cap][D] (batch 1)
};

struct MegaParams {
    const MegaLayer *layers;
    int n_layers;
    const __nv_bfloat16 *embed, *final_norm;
    const uint8_t *lm_head;
    const float *inv_freq;
    int H, I, Hq, Hkv, V;
    float eps;
    float scale_log2;  // softmax scale * log2(e)
    int64_t cap, kv_hstride;
    int *tokens, *pos;
    __nv_bfloat16 *logits;
    // scratch (one plan's device block)
    __nv_bfloat16 *h, *qkv_out, *attn_out, *act_out, *o_out, *down_out;
    int8_t *aq;
    float *ad, *ac;
    int8_t *gq;
    float *gd, *gc;
    float *part_o, *part_ml;
    int *tickets;
    unsigned long long *bar;
    unsigned int *epoch;
    float2 *amax_part;
    int *err;
    int *diag;    // [4]: where the first wait that gave up was (CTA + 1, kind, index, parity)
    int splits;   // key splits per KV head
    int nslots;
    int trace_layer;  // layer whose activations are copied to `trace` (-1: none)
    uint8_t *trace;
    unsigned long long *stamps;  // [G][kStamps] %globaltimer phase timeline of layer 1 (or null)
};

// Timeline events (per CTA, layer 1): consumer thread 0 after each phase's
// grid wait and after its work; the producer lane when it issues the first
// item of each phase and when it has issued the layer's last item.
enum : int {
    kStStart = 0, kStQWait, kStQDone, kStAWait, kStADone, kStOWait, kStODone, kStGWait, kStGDone, kStDWait,
    kStDDone, kStPQ, kStPA, kStPO, kStPG, kStPD, kStPEnd, kStEnd, kStQStaged, kStAStaged, kStAMerged,
    kStATicket,
    kStQWarp0,  // [kStQWarp0, + kCW): when each consumer warp finished its last q/k/v item
    kStAWarp0 = kStQWarp0 + 16,  // [kStAWarp0, + kAttnWarps): when each attention warp finished its keys
    kStAHeadWait = kStAWarp0 + 8,  // when this split saw every split of its head posted
    kStAW0Waited, kStAW0Scored, kStAW0Done,  // attention warp 0, first chunk: ring waits, scores, values
    kStAW0Item0,  // [+8): attention warp 0, first chunk: when each K/V ring wait returned
    kStQW0Item = kStAW0Item0 + 8,  // consumer warp 0's first q/k/v item: ring wait returned
    kStQW0Dot,    // its dot products done
    kStAItemIdx,  // the ring index of warp 0's first K item (to compare with the producer's count)
    kStPKV0,      // producer: when it started issuing this layer's K/V items
    kStamps = 64  // slots per CTA (tn_llama_decode_token_timeline)
};
static_assert(kStPKV0 < kStamps, "timeline slots");
enum : int {
    kStUnused = kStamps
};

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// ---- shared-memory layout --------------------------------------------------
// [0, 16*kMaxSlots)         full[], empty[] mbarriers
// xs   kMaxK bytes          activation codes, pair-swizzled
// xds  kMaxK/32 floats      widened scales
// xcs  kMaxK/32 floats      offset constants (12582912 + 8 * sum of codes)
// misc 4 KB                 reductions, broadcast words, attention q, act values
// ring nslots * kSlot       (attention reuses xs.. for its per-warp partials)
constexpr int kMiscBytes = 8192;
constexpr size_t kXsOff = 16 * kMaxSlots;
constexpr size_t kXdsOff = kXsOff + kMaxK;
constexpr size_t kXcsOff = kXdsOff + (kMaxK / 32) * 4;
constexpr size_t kMiscOff = kXcsOff + (kMaxK / 32) * 4;
constexpr size_t kRingOff = (kMiscOff + kMiscBytes + 127) & ~size_t(127);

// misc area (floats unless noted)
constexpr int kRedOff = 0;          // [kCW] block-reduction partials
constexpr int kBcastOff = 64;       // ints: abort flag, ticket result, token
constexpr int kQOff = 128;          // [kRep][kD] rotated query (f32)
constexpr int kKNewOff = 128 + kRep * kD;      // [kD] rotated new key (f32)
constexpr int kVNewOff = kKNewOff + kD;        // [kD] new value (f32)
constexpr int kActOff = kVNewOff + kD;         // [kMaxUnitsG * 32] act values (f32)
constexpr int kArgOff = kActOff + kMaxUnitsG * 32;  // [kCW] (value, index) pairs
static_assert((kArgOff + 2 * kCW) * 4 <= kMiscBytes, "misc area");

struct Ctx {
    uint8_t *base;
    uint64_t *full, *empty;
    uint32_t xs, xds, xcs, ring;
    float *misc;
    volatile int *abort;
    int G, c;
    unsigned long long bar_base;  // arrivals before this launch's first barrier
    unsigned int epoch;           // tokens this plan has completed before this launch
};

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
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ float2 lds64f(uint32_t a) {
    float2 v;
    asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ void sts128(uint32_t a, int4 v) {
    asm volatile("st.shared.v4.s32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}
__device__ __forceinline__ void stsf(uint32_t a, float v) {
    asm volatile("st.shared.f32 [%0], %1;" ::"r"(a), "f"(v) : "memory");
}
__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"r"(kCT) : "memory"); }

// Release a ring slot: its empty barrier completes a phase after kAttnWarps
// arrivals -- all of them from the one warp that consumed a weight item, one
// from each attention warp for a K/V item (every attention warp reads its
// eighth of each key tile).
__device__ __forceinline__ void slot_release(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Byte offset of 16-byte chunk c (0..3) of block pair `pair` in the staged
// codes (chunks 0/1: low/high 16 codes of block 2*pair, 2/3: of 2*pair+1),
// XOR-swizzled so the 8 lanes of a quarter-warp hit 8 different bank groups.
__device__ __forceinline__ uint32_t xchunk(int pair, int c) {
    return (uint32_t)(pair * 64 + 16 * (c ^ ((pair >> 1) & 3)));
}

__device__ __forceinline__ float bfr(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
__device__ __forceinline__ uint32_t bf2_bits(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t *>(&v); }
__device__ __forceinline__ __nv_bfloat162 bf2_of(uint32_t u) { return *reinterpret_cast<__nv_bfloat162 *>(&u); }

__device__ __forceinline__ int sat_i8r(float v) {
    if (!(v == v)) return 0;
    if (v <= -128.0f) return -128;
    if (v >= 127.0f) return 127;
    return __float2int_rz(v);
}

// ---- bounded waits -----------------------------------------------------------

__device__ __forceinline__ void raise_abort(const Ctx &x, const MegaParams &p, int code) {
    *x.abort = 1;
    record_device_error(p.err, code);
}

// Record where a wait gave up (kind 1: a consumer's full wait, 2: the
// producer's empty wait, 3: a grid barrier), first one only.
__device__ __forceinline__ void note_wait(const Ctx &x, const MegaParams &p, int kind, int index, int parity) {
    if (atomicCAS(p.diag, 0, x.c + 1) == 0) {
        p.diag[1] = kind;
        p.diag[2] = index;
        p.diag[3] = parity;
    }
}

// mbarrier phase wait; false on timeout or when this launch already aborted
// (this CTA's flag, or the device error word another CTA set). A false return
// never changes a warp's barrier sequence: callers skip work, not barriers.
__device__ __forceinline__ bool ring_wait(const Ctx &x, const MegaParams &p, uint64_t *bar, uint32_t parity,
                                          int kind = 1, int index = -1) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long start = clock64(), budget = wait_budget(p.err);
    int spins = 0;
    while (!mbar_try_wait(bar, parity)) {
        if ((++spins & 255) == 0) {
            if (*x.abort || *reinterpret_cast<volatile int *>(p.err) != 0) {
                *x.abort = 1;
                return false;
            }
            if (clock64() - start > budget) {
                note_wait(x, p, kind, index, (int)parity);
                raise_abort(x, p, DEV_ERR_WAIT_FULL);
                return false;
            }
        }
    }
    return true;
}

// Grid barrier b of this launch: every CTA arrives once (after the consumer
// threads' stores, one thread, release); the wait spins (acquire) until all G
// CTAs of barrier b have arrived. Consumer threads only.
__device__ __forceinline__ void grid_arrive(const Ctx &x, const MegaParams &p) {
    consumers_sync();
    if (threadIdx.x == 0) {
        // release at gpu scope: cumulative over the consumer threads' stores,
        // which the CTA barrier above ordered before this thread's arrival
        asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(p.bar) : "memory");
    }
}


// The return value is the same in every consumer thread: thread 0 takes the
// decision and publishes it in a word nothing else writes (the producer may
// raise the abort flag at any moment, so the flag itself is not read twice).
__device__ __forceinline__ bool grid_wait(const Ctx &x, const MegaParams &p, int b) {
    volatile int *decision = reinterpret_cast<volatile int *>(x.misc + kBcastOff) + 2;
    if (threadIdx.x == 0) {
        const unsigned long long target = x.bar_base + (unsigned long long)(b + 1) * (unsigned long long)x.G;
        if (ld_acquire_u64(p.bar) < target) {
            const long long start = clock64(), budget = wait_budget(p.err);
            int spins = 0;
            while (ld_acquire_u64(p.bar) < target) {
                if ((++spins & 63) == 0) {
                    if (*x.abort || *reinterpret_cast<volatile int *>(p.err) != 0) {
                        *x.abort = 1;
                        break;
                    }
                    if (clock64() - start > budget) {
                        note_wait(x, p, 3, b, (int)(ld_acquire_u64(p.bar) - x.bar_base));
                        raise_abort(x, p, DEV_ERR_WAIT_FULL);
                        break;
                    }
                }
            }
        }
        *decision = (*x.abort == 0 && *reinterpret_cast<volatile int *>(p.err) == 0) ? 1 : 0;
    }
    consumers_sync();
    return *decision != 0;
}

// ---- schedule (computed identically by the producer and the consumers) -----

// A linear's share for CTA c: output rows [r0, r1) in ring items of R rows
// (R = the rows of K/32 blocks of 18 bytes that fill a slot, at most
// kMaxRows); unit = item, one consumer warp each.
struct Lin {
    int r0, r1, R, nb, rowbytes, units, items;
};

__device__ __forceinline__ Lin lin_share(int N, int K, int c, int G, int rmax = kMaxRows) {
    Lin s;
    s.nb = K / 32;
    s.rowbytes = 18 * s.nb;
    s.r0 = (int)((int64_t)c * N / G);
    s.r1 = (int)((int64_t)(c + 1) * N / G);
    s.R = kSlot / s.rowbytes;
    if (s.R > rmax) s.R = rmax;
    while (s.R & (s.R - 1)) s.R &= s.R - 1;  // a power of two: dot_item's row counts
    s.units = (s.r1 - s.r0 + s.R - 1) / s.R;
    s.items = s.units;
    return s;
}

// gate/up: whole 64-row units (32 act columns = one Q8_0 block of act).
__device__ __forceinline__ Lin gu_share(int I, int K, int c, int G) {
    const int U = 2 * I / 64;
    const int u0 = (int)((int64_t)c * U / G), u1 = (int)((int64_t)(c + 1) * U / G);
    Lin s = lin_share(2 * I, K, 0, 1);
    s.r0 = 64 * u0;
    s.r1 = 64 * u1;
    s.units = (s.r1 - s.r0 + s.R - 1) / s.R;  // R even: whole (gate, up) pairs per item
    s.items = s.units;
    return s;
}

// Attention share: KV head g, split s of the past keys [0, pos); the last
// split of each head also takes the new key (index pos).
struct Att {
    bool active;
    int g, s, k0, k1, tiles;
};

__device__ __forceinline__ Att att_share(const MegaParams &p, int c, int pos) {
    Att a;
    a.active = c < p.Hkv * p.splits;
    a.g = c / p.splits;
    a.s = c % p.splits;
    a.k0 = (int)((int64_t)a.s * pos / p.splits);
    a.k1 = (int)((int64_t)(a.s + 1) * pos / p.splits);
    a.tiles = a.active ? (a.k1 - a.k0 + kTile - 1) / kTile : 0;
    if (!a.active) a.k0 = a.k1 = 0;
    return a;
}

// K/V tiles of a layer issued ahead of its q/k/v weights: as many as the ring
// holds beside the q/k/v items. They are consumed after those items, so no
// q/k/v item may need a slot an early K/V item still holds (deadlock), nor
// wait on a slot two fills ahead: 2 * early + q/k/v items <= nslots.
__device__ __forceinline__ int kv_early(const MegaParams &p, const Att &a, int nq) {
    int e = (p.nslots - nq) / 2;
    if (e < 0) e = 0;
    return a.tiles < e ? a.tiles : e;
}

// ---- producer ----------------------------------------------------------------

struct Prod {
    uint32_t item;
    uint64_t policy;
};

__device__ __forceinline__ bool issue(const Ctx &x, const MegaParams &p, Prod &pr, const void *src, uint32_t bytes) {
    const uint32_t slot = pr.item % (uint32_t)p.nslots, fill = pr.item / (uint32_t)p.nslots;
    if (fill > 0 && !ring_wait(x, p, &x.empty[slot], (fill - 1) & 1, 2, (int)pr.item)) return false;
    mbar_arrive_expect_tx(&x.full[slot], bytes);
    bulk_g2s_hint_u32(x.ring + slot * kSlot, src, bytes, &x.full[slot], pr.policy);
    ++pr.item;
    return true;
}

__device__ __forceinline__ bool issue_linear(const Ctx &x, const MegaParams &p, Prod &pr, const uint8_t *w,
                                             const Lin &s) {
    for (int u = 0; u < s.units; ++u) {
        const int r = s.r0 + u * s.R;
        const int nr = (s.r1 - r) < s.R ? (s.r1 - r) : s.R;
        if (!issue(x, p, pr, w + (int64_t)r * s.rowbytes, (uint32_t)(nr * s.rowbytes))) return false;
    }
    return true;
}

__device__ void producer(const Ctx &x, const MegaParams &p, int pos) {
    Prod pr{0u, policy_evict_first()};
    const int G = x.G, c = x.c;
    const int QKV = (p.Hq + 2 * p.Hkv) * kD;
    const Att at = att_share(p, c, pos);
    bool ok = true;
    unsigned long long *st = (p.stamps && p.n_layers > 1) ? p.stamps + (size_t)c * kStamps : nullptr;
    for (int l = 0; l < p.n_layers && ok; ++l) {
        const MegaLayer &L = p.layers[l];
        const bool tl = st && l == 1;
        // the layer's past K/V first: those bytes are ready long before the
        // q/k/v weights are needed, and behind the weights they would land
        // only as the attention phase starts
        const Lin sq = lin_share(QKV, p.H, c, G, 4);
        const int early = kv_early(p, at, sq.items);
        auto issue_tile = [&](int t) {
            const int k = at.k0 + t * kTile;
            const int n = (at.k1 - k) < kTile ? (at.k1 - k) : kTile;
            const int64_t off = (int64_t)at.g * p.kv_hstride + (int64_t)k * kD;
            return issue(x, p, pr, L.kc + off, (uint32_t)(n * kD * 2)) &&
                   issue(x, p, pr, L.vc + off, (uint32_t)(n * kD * 2));
        };
        if (tl) st[kStPA] = globaltimer();
        for (int t = 0; ok && t < early; ++t) ok = issue_tile(t);
        if (tl) st[kStPQ] = globaltimer();
        ok = ok && issue_linear(x, p, pr, L.qkv, sq);
        for (int t = early; ok && t < at.tiles; ++t) ok = issue_tile(t);
        if (tl) st[kStPO] = globaltimer();
        ok = ok && issue_linear(x, p, pr, L.o, lin_share(p.H, p.Hq * kD, c, G, 4));
        if (tl) st[kStPG] = globaltimer();
        ok = ok && issue_linear(x, p, pr, L.gate_up, gu_share(p.I, p.H, c, G));
        if (tl) st[kStPD] = globaltimer();
        ok = ok && issue_linear(x, p, pr, L.down, lin_share(p.H, p.I, c, G));
        if (tl) st[kStPEnd] = globaltimer();
    }
    if (ok) ok = issue_linear(x, p, pr, p.lm_head, lin_share(p.V, p.H, c, G));
    // Drain: every slot's most recent copy lands before the CTA may exit.
    for (uint32_t s = 0; s < (uint32_t)p.nslots && s < pr.item; ++s) {
        const uint32_t last = pr.item - 1 - ((pr.item - 1 - s) % (uint32_t)p.nslots);
        const uint32_t fill = last / (uint32_t)p.nslots;
        if (!mbar_wait(&x.full[s], fill & 1)) {
            record_device_error(p.err, DEV_ERR_DRAIN);
            break;
        }
    }
}

// ---- consumers: activation staging ---------------------------------------

// One Q8_0 block (k_quants.rs:676-706) from 16 bf16 values per lane of a lane
// pair (the fused GEMV's packed arithmetic): codes into the swizzled tile,
// widened scale and offset constant into xds / xcs.
__device__ __forceinline__ void q8_half_block(const uint32_t (&v)[8], int b, int half, const Ctx &x, int lane) {
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
        w[k] = __byte_perm(__byte_perm((uint32_t)q0, (uint32_t)q1, 0x0040),
                           __byte_perm((uint32_t)q2, (uint32_t)q3, 0x0040), 0x5410);
        sum = __dp4a((int)w[k], 0x01010101, sum);
    }
    sum += __shfl_xor_sync(pm, sum, 1);
    sts128(x.xs + xchunk(b >> 1, (b & 1) * 2 + half), make_int4((int)w[0], (int)w[1], (int)w[2], (int)w[3]));
    if (half == 0) {
        stsf(x.xds + b * 4, __half2float(__float2half_rn(d)));
        stsf(x.xcs + b * 4, 12582912.0f + 8.0f * (float)sum);
    }
}

// RMSNorm (transformers' LlamaRMSNorm: w * bf16(h * rsqrt(mean(h^2) + eps)))
// of the bf16 vector `src` (K elements; read from L2, it was written by other
// CTAs) to the Q8_0 tile; thread t takes half-block t. If h_rows is set, the
// thread also writes the rows of src in [h_r0, h_r1) to h_rows (the layer-0
// embedding becoming the residual stream). Returns false on abort.
__device__ __forceinline__ void stage_rmsnorm(const Ctx &x, const MegaParams &p, const __nv_bfloat16 *src,
                                              const __nv_bfloat16 *w, int K, __nv_bfloat16 *h_rows, int h_r0,
                                              int h_r1) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nb = K / 32;
    float *red = x.misc + kRedOff;
    uint32_t hb[8], wp[8];
    float ss = 0.0f;
    const bool act = tid < 2 * nb;
    const int b = tid >> 1, hf = tid & 1, e0 = b * 32 + 16 * hf;
    if (act) {
        int4 xr[2], wr[2];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            xr[c] = __ldcg(reinterpret_cast<const int4 *>(src + e0) + c);
            wr[c] = __ldg(reinterpret_cast<const int4 *>(w + e0) + c);
        }
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            hb[4 * c] = (uint32_t)xr[c].x, hb[4 * c + 1] = (uint32_t)xr[c].y;
            hb[4 * c + 2] = (uint32_t)xr[c].z, hb[4 * c + 3] = (uint32_t)xr[c].w;
            wp[4 * c] = (uint32_t)wr[c].x, wp[4 * c + 1] = (uint32_t)wr[c].y;
            wp[4 * c + 2] = (uint32_t)wr[c].z, wp[4 * c + 3] = (uint32_t)wr[c].w;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float lo = bf_lo(hb[i]), hi = bf_hi(hb[i]);
            ss = fmaf(lo, lo, ss);
            ss = fmaf(hi, hi, ss);
        }
        if (h_rows && e0 + 16 > h_r0 && e0 < h_r1) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int e = e0 + 2 * i;
                if (e >= h_r0 && e < h_r1) h_rows[e] = __ushort_as_bfloat16((unsigned short)(hb[i] & 0xffff));
                if (e + 1 >= h_r0 && e + 1 < h_r1) h_rows[e + 1] = __ushort_as_bfloat16((unsigned short)(hb[i] >> 16));
            }
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (lane == 0) red[warp] = ss;
    consumers_sync();
    float t = 0.0f;
#pragma unroll
    for (int i = 0; i < kCW; ++i) t += red[i];
    const float r = rsqrtf(t / (float)K + p.eps);
    if (act) {
        uint32_t v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const __nv_bfloat162 hr = __floats2bfloat162_rn(bf_lo(hb[i]) * r, bf_hi(hb[i]) * r);
            v[i] = bf2_bits(__hmul2(bf2_of(wp[i]), hr));
        }
        q8_half_block(v, b, hf, x, lane);
    }
    consumers_sync();
}

// Planar Q8_0 written by other CTAs (codes [K], scales/offsets [K/32]) into
// the tile.
__device__ __forceinline__ void stage_planar(const Ctx &x, const int8_t *q, const float *d, const float *c, int K) {
    const int tid = threadIdx.x;
    for (int ci = tid; ci < K / 16; ci += kCT) {
        const int4 v = __ldcg(reinterpret_cast<const int4 *>(q) + ci);
        const int b = ci >> 1, half = ci & 1;
        sts128(x.xs + xchunk(b >> 1, (b & 1) * 2 + half), v);
    }
    for (int b = tid; b < K / 32; b += kCT) {
        stsf(x.xds + b * 4, __ldcg(d + b));
        stsf(x.xcs + b * 4, __ldcg(c + b));
    }
    consumers_sync();
}

// ---- consumers: dot products ------------------------------------------------

// Add the blocks of one ring item (R rows of nb blocks, rows rowstride bytes
// apart) into acc[0..R-1]: lanes over block pairs, 9 words per pair
// (conflict-free: 9 is odd), each activation load serving every row, exact
// integer dots, one fmaf per block. R is a compile-time row count: an item
// with fewer rows computes garbage for the missing ones (stale bytes of its
// own slot) and the epilogue drops them, so the loop body has no branch and
// every row's loads can be issued together. Each block's 32-term dot is two
// independent dp4a chains of four (low and high nibbles) joined by one
// integer add, the magic constant riding on the first.
template <int R>
__device__ __forceinline__ void dot_item(const Ctx &x, uint32_t ws, int rowstride, int nb, float (&acc)[kMaxRows],
                                         int lane) {
    const int npairs = nb >> 1;
#pragma unroll 2
    for (int pair = lane; pair < npairs; pair += 32) {
        const uint32_t xb = x.xs;
        const int4 x0 = lds128(xb + xchunk(pair, 0)), x1 = lds128(xb + xchunk(pair, 1));
        const int4 x2 = lds128(xb + xchunk(pair, 2)), x3 = lds128(xb + xchunk(pair, 3));
        const float2 xd = lds64f(x.xds + pair * 8), xc = lds64f(x.xcs + pair * 8);
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const uint32_t a = ws + r * rowstride + pair * 36;
            uint32_t wv[9];
#pragma unroll
            for (int i = 0; i < 9; ++i) wv[i] = lds32(a + 4 * i);
            // block A: d = low half of word 0, codes = bytes 2..17; block B: d =
            // high half of word 4, codes = words 5..8
            const uint32_t qa[4] = {__funnelshift_r(wv[0], wv[1], 16), __funnelshift_r(wv[1], wv[2], 16),
                                    __funnelshift_r(wv[2], wv[3], 16), __funnelshift_r(wv[3], wv[4], 16)};
            const float da = half_bits_to_f32(wv[0]), db = half_bits_to_f32(wv[4] >> 16);
            int Ia = (int)kMagic, Ja = 0, Ib = (int)kMagic, Jb = 0;
            Ia = __dp4a((int)(qa[0] & 0x0F0F0F0Fu), x0.x, Ia);
            Ja = __dp4a((int)((qa[0] >> 4) & 0x0F0F0F0Fu), x1.x, Ja);
            Ib = __dp4a((int)(wv[5] & 0x0F0F0F0Fu), x2.x, Ib);
            Jb = __dp4a((int)((wv[5] >> 4) & 0x0F0F0F0Fu), x3.x, Jb);
            Ia = __dp4a((int)(qa[1] & 0x0F0F0F0Fu), x0.y, Ia);
            Ja = __dp4a((int)((qa[1] >> 4) & 0x0F0F0F0Fu), x1.y, Ja);
            Ib = __dp4a((int)(wv[6] & 0x0F0F0F0Fu), x2.y, Ib);
            Jb = __dp4a((int)((wv[6] >> 4) & 0x0F0F0F0Fu), x3.y, Jb);
            Ia = __dp4a((int)(qa[2] & 0x0F0F0F0Fu), x0.z, Ia);
            Ja = __dp4a((int)((qa[2] >> 4) & 0x0F0F0F0Fu), x1.z, Ja);
            Ib = __dp4a((int)(wv[7] & 0x0F0F0F0Fu), x2.z, Ib);
            Jb = __dp4a((int)((wv[7] >> 4) & 0x0F0F0F0Fu), x3.z, Jb);
            Ia = __dp4a((int)(qa[3] & 0x0F0F0F0Fu), x0.w, Ia);
            Ja = __dp4a((int)((qa[3] >> 4) & 0x0F0F0F0Fu), x1.w, Ja);
            Ib = __dp4a((int)(wv[8] & 0x0F0F0F0Fu), x2.w, Ib);
            Jb = __dp4a((int)((wv[8] >> 4) & 0x0F0F0F0Fu), x3.w, Jb);
            acc[r] = fmaf(__int_as_float(Ia + Ja) - xc.x, da * xd.x, acc[r]);
            acc[r] = fmaf(__int_as_float(Ib + Jb) - xc.y, db * xd.y, acc[r]);
        }
    }
}

// Reduce-scatter of the 8 per-lane row sums: afterwards lane L holds the
// warp-wide sum of row (L >> 2) & 7 (a 5-level tree, like warp_sum).
__device__ __forceinline__ float reduce_rows8(float (&v)[kMaxRows], int lane) {
#pragma unroll
    for (int lev = 0; lev < 3; ++lev) {
        const int off = 16 >> lev, n = 4 >> lev;
        const bool up = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if (i < n) {
                const float send = up ? v[i] : v[i + n];
                const float keep = up ? v[i + n] : v[i];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
            }
        }
    }
    float t = v[0];
    t += __shfl_xor_sync(0xffffffffu, t, 2);
    t += __shfl_xor_sync(0xffffffffu, t, 1);
    return t;
}


// Consume a linear phase's items. Ring item j (counted over the whole
// launch) goes to consumer warp j % kCW, and nslots is a multiple of kCW, so
// the item that held the same slot before it, j - nslots, was this warp's own: when a warp waits on a
// slot's full barrier the slot is exactly one phase behind -- a parity wait
// cannot tell a phase from the one two ahead, and a warp that could run two
// fills ahead of its slot would take stale bytes. (K/V items, which every
// attention warp reads, keep the property too: each attention warp reads
// every one of them in order, and items of earlier phases are all released
// before a grid barrier lets the next phase start.) Per finished item the row
// sums are spread over the warp (lane 4k holds row k, k < nr) and
// `ep(lane, row0, v, nr)` runs on every lane (the epilogue picks its lanes).
// `item` is this CTA's ring position at the phase start and is advanced past
// the phase's items.
template <typename Ep>
__device__ __forceinline__ void consume_linear(const Ctx &x, const MegaParams &p, const Lin &s, uint32_t &item,
                                               Ep ep, unsigned long long *w0 = nullptr) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int W = kCW;  // nslots is a multiple of kCW: items j and j + nslots share a warp
    const int u0 = (int)((uint32_t)(warp + W) - item % (uint32_t)W) % W;
    for (int u = u0; u < s.units; u += W) {
        float acc[kMaxRows];
#pragma unroll
        for (int r = 0; r < kMaxRows; ++r) acc[r] = 0.0f;
        const uint32_t it = item + (uint32_t)u;
        const uint32_t slot = it % (uint32_t)p.nslots;
        const int r0 = s.r0 + u * s.R;
        const int nr = (s.r1 - r0) < s.R ? (s.r1 - r0) : s.R;
        if (!ring_wait(x, p, &x.full[slot], (it / (uint32_t)p.nslots) & 1, 1, (int)it)) break;
        if (w0 && u == u0) w0[kStQW0Item] = globaltimer();
        const uint32_t ws = x.ring + slot * kSlot;
        if (s.R == 8)
            dot_item<8>(x, ws, s.rowbytes, s.nb, acc, lane);
        else if (s.R == 4)
            dot_item<4>(x, ws, s.rowbytes, s.nb, acc, lane);
        else if (s.R == 2)
            dot_item<2>(x, ws, s.rowbytes, s.nb, acc, lane);
        else
            dot_item<1>(x, ws, s.rowbytes, s.nb, acc, lane);
        __syncwarp();
        if (w0 && u == u0) w0[kStQW0Dot] = globaltimer();
        if (lane == 0) slot_release(&x.empty[slot], kAttnWarps);
        const float v = reduce_rows8(acc, lane);
        ep(lane, r0, v, nr);
    }
    item += (uint32_t)s.items;
}

// ---- consumers: attention --------------------------------------------------

// RoPE (transformers' rotate_half with cos/sin rounded to bf16; the same
// arithmetic as tn_llama_rope_append) of head `src` (bf16, D elements) at
// position pos: element i of the result for i < D/2 pairs (i, i + D/2).
__device__ __forceinline__ void rope_pair(const __nv_bfloat16 *src, const float *inv_freq, int pos, int i, float &y1,
                                          float &y2) {
    const float f = inv_freq[i] * (float)pos;
    const float c = bfr(cosf(f)), s = bfr(sinf(f));
    const float x1 = __bfloat162float(__ldcg(src + i)), x2 = __bfloat162float(__ldcg(src + i + kD / 2));
    y1 = bfr(bfr(x1 * c) + bfr(-x2 * s));
    y2 = bfr(bfr(x2 * c) + bfr(x1 * s));
}

// Reduce-scatter of 16 per-lane partial values over the warp: afterwards
// lanes L and L ^ 1 both hold the warp-wide sum of value (L >> 1) & 15.
__device__ __forceinline__ float reduce_scatter16(float (&v)[16], int lane) {
#pragma unroll
    for (int lev = 0; lev < 4; ++lev) {
        const int off = 16 >> lev, n = 8 >> lev;
        const bool up = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (i < n) {
                const float send = up ? v[i] : v[i + n];
                const float keep = up ? v[i + n] : v[i];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
            }
        }
    }
    return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
}

// One warp's running softmax state for the kRep (= 4) query heads of its KV
// head: lane L scores key (L >> 3) & 3 of a 4-key step for head (L >> 1) & 3
// (lanes L and L ^ 1 hold the same value) and keeps that head's running
// maximum m (log2 units) and sum l; o[h][e] is this lane's output dims
// 4 * lane + e of head h.
struct AttnState {
    float m, l;
    float o[kRep][4];
};

__device__ __forceinline__ void bf4(uint2 raw, float (&f)[4]) {
    f[0] = bf_lo(raw.x), f[1] = bf_hi(raw.x), f[2] = bf_lo(raw.y), f[3] = bf_hi(raw.y);
}

// Online softmax over kChunk 4-key steps for the 4 heads: nn[c] (<= 4) keys
// of step c at kb[c] / vb[c] (shared addresses of this lane's 8 bytes of key /
// value row 0; rows kD * 2 bytes apart; rows >= nn[c] are read as row 0 and
// masked). q: the rotated queries [kRep][kD] f32 in shared memory. The steps'
// score reductions are independent, so they overlap; the running maximum
// moves once per chunk.
__device__ __forceinline__ void attend_chunk(AttnState &st, const float *q, const uint32_t (&kb)[kChunk],
                                             const uint32_t (&vb)[kChunk], const int (&nn)[kChunk], float scale2,
                                             int lane, unsigned long long *w0 = nullptr) {
    const int kj = (lane >> 3) & 3;
    float qv[kRep][4];
#pragma unroll
    for (int h = 0; h < kRep; ++h) {
        const float4 qh = *reinterpret_cast<const float4 *>(q + h * kD + 4 * lane);
        qv[h][0] = qh.x, qv[h][1] = qh.y, qv[h][2] = qh.z, qv[h][3] = qh.w;
    }
    float s2[kChunk];
#pragma unroll
    for (int c = 0; c < kChunk; ++c) {
        float part[16];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float k[4];
            bf4(lds64(kb[c] + (j < nn[c] ? j : 0) * kD * 2), k);
#pragma unroll
            for (int h = 0; h < kRep; ++h)
                part[4 * j + h] = fmaf(qv[h][3], k[3], fmaf(qv[h][2], k[2], fmaf(qv[h][1], k[1], qv[h][0] * k[0])));
        }
        const float tot = reduce_scatter16(part, lane);
        s2[c] = (kj < nn[c]) ? tot * scale2 : -INFINITY;
    }
    float mx = s2[0];
#pragma unroll
    for (int c = 1; c < kChunk; ++c) mx = fmaxf(mx, s2[c]);
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
    const float m_new = fmaxf(st.m, mx);
    if (w0) w0[kStAW0Scored] = globaltimer();
    if (m_new == -INFINITY) return;  // no live key in the chunk (uniform over the warp per head)
    const float alpha = (st.m == -INFINITY) ? 0.0f : exp2f(st.m - m_new);
    float pj[kChunk], ps = 0.0f;
#pragma unroll
    for (int c = 0; c < kChunk; ++c) {
        pj[c] = (s2[c] == -INFINITY) ? 0.0f : exp2f(s2[c] - m_new);
        ps += pj[c];
    }
    ps += __shfl_xor_sync(0xffffffffu, ps, 8);
    ps += __shfl_xor_sync(0xffffffffu, ps, 16);
    st.l = st.l * alpha + ps;
    st.m = m_new;
#pragma unroll
    for (int h = 0; h < kRep; ++h) {
        const float ah = __shfl_sync(0xffffffffu, alpha, 2 * h);  // head h's alpha sits in lane 2h
#pragma unroll
        for (int e = 0; e < 4; ++e) st.o[h][e] *= ah;
    }
#pragma unroll
    for (int c = 0; c < kChunk; ++c) {
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            if (jj >= nn[c]) break;
            float v[4];
            bf4(lds64(vb[c] + jj * kD * 2), v);
#pragma unroll
            for (int h = 0; h < kRep; ++h) {
                const float pw = __shfl_sync(0xffffffffu, pj[c], 8 * jj + 2 * h);  // p of (key jj, head h)
#pragma unroll
                for (int e = 0; e < 4; ++e) st.o[h][e] = fmaf(pw, v[e], st.o[h][e]);
            }
        }
    }
}

// The attention phase of one layer for this CTA (consumer threads).
__device__ void attention_phase(const Ctx &x, const MegaParams &p, const MegaLayer &L, int layer, int pos,
                                uint32_t kv0, uint32_t kv1, int early, unsigned long long *sl) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const Att a = att_share(p, x.c, pos);
    const bool last_split = a.active && a.s == p.splits - 1;
    float *qs = x.misc + kQOff, *kn = x.misc + kKNewOff, *vn = x.misc + kVNewOff;
    if (a.active) {
        // rotated queries of the group (and the new key / value in the last split)
        for (int t = tid; t < kRep * (kD / 2); t += kCT) {
            const int h = t / (kD / 2), i = t % (kD / 2);
            float y1, y2;
            rope_pair(p.qkv_out + (a.g * kRep + h) * kD, p.inv_freq, pos, i, y1, y2);
            qs[h * kD + i] = y1;
            qs[h * kD + i + kD / 2] = y2;
        }
        if (last_split) {
            for (int i = tid; i < kD / 2; i += kCT) {
                float y1, y2;
                rope_pair(p.qkv_out + (p.Hq + a.g) * kD, p.inv_freq, pos, i, y1, y2);
                __nv_bfloat16 *kr = reinterpret_cast<__nv_bfloat16 *>(kn);
                kr[i] = __float2bfloat16_rn(y1);
                kr[i + kD / 2] = __float2bfloat16_rn(y2);
                __nv_bfloat16 *kc = L.kc + (int64_t)a.g * p.kv_hstride + (int64_t)pos * kD;
                kc[i] = __float2bfloat16_rn(y1);
                kc[i + kD / 2] = __float2bfloat16_rn(y2);
            }
            for (int i = tid; i < kD; i += kCT) {
                const __nv_bfloat16 v = __ldcg(p.qkv_out + (p.Hq + p.Hkv + a.g) * kD + i);
                reinterpret_cast<__nv_bfloat16 *>(vn)[i] = v;
                (L.vc + (int64_t)a.g * p.kv_hstride + (int64_t)pos * kD)[i] = v;
            }
        }
    }
    consumers_sync();
    if (sl) sl[kStAStaged] = globaltimer();
    // per-warp online softmax over the warp's keys: every attention warp takes
    // keys [4 warp, 4 warp + 4) of each tile, tiles in chunks of kChunk whose
    // score reductions run side by side, one softmax update per chunk
    float *wpart = reinterpret_cast<float *>(x.base + kXsOff);  // [kAttnWarps][kRep][kD + 2]
    constexpr int WP = kRep * (kD + 2);
    if (a.active && warp < kAttnWarps) {
        AttnState st;
#pragma unroll
        for (int h = 0; h < kRep; ++h)
#pragma unroll
            for (int e = 0; e < 4; ++e) st.o[h][e] = 0.0f;
        st.m = -INFINITY;
        st.l = 0.0f;
        bool ok = true;
        const uint32_t off = (uint32_t)(4 * warp * kD * 2) + lane * 8;
        for (int t0 = 0; t0 < a.tiles && ok; t0 += kChunk) {
            const int nt = (a.tiles - t0) < kChunk ? (a.tiles - t0) : kChunk;
            uint32_t kb[kChunk], vb[kChunk];
            int nn[kChunk];
#pragma unroll
            for (int c = 0; c < kChunk; ++c) {
                nn[c] = 0;
                kb[c] = vb[c] = 0;
                if (c < nt) {
                    const int t = t0 + c;
                    const uint32_t ik = (t < early ? kv0 + 2 * t : kv1 + 2 * (t - early)), iv = ik + 1;
                    const uint32_t sk = ik % (uint32_t)p.nslots, sv = iv % (uint32_t)p.nslots;
                    if (!ring_wait(x, p, &x.full[sk], (ik / (uint32_t)p.nslots) & 1, 4, (int)ik) ||
                        !ring_wait(x, p, &x.full[sv], (iv / (uint32_t)p.nslots) & 1, 4, (int)iv))
                        ok = false;
                    if (sl && warp == 0 && lane == 0 && t0 == 0) {
                        sl[kStAW0Item0 + c] = globaltimer();
                        if (c == 0) sl[kStAItemIdx] = ik;
                    }
                    const int kbase = a.k0 + (t0 + c) * kTile + 4 * warp;
                    const int k_left = a.k1 - kbase;
                    nn[c] = ok ? (k_left < 0 ? 0 : (k_left < 4 ? k_left : 4)) : 0;
                    kb[c] = x.ring + sk * kSlot + off;
                    vb[c] = x.ring + sv * kSlot + off;
                }
            }
            unsigned long long *w0 = (sl && warp == 0 && lane == 0 && t0 == 0) ? sl : nullptr;
            if (w0) w0[kStAW0Waited] = globaltimer();
            attend_chunk(st, qs, kb, vb, nn, p.scale_log2, lane, w0);
            if (w0) w0[kStAW0Done] = globaltimer();
            __syncwarp();
            if (lane == 0)
                for (int c = 0; c < nt; ++c) {
                    const int t = t0 + c;
                    const uint32_t ik = (t < early ? kv0 + 2 * t : kv1 + 2 * (t - early));
                    slot_release(&x.empty[ik % (uint32_t)p.nslots], 1);
                    slot_release(&x.empty[(ik + 1) % (uint32_t)p.nslots], 1);
                }
        }
        if (last_split && warp == 0) {
            // the new key (index pos): its bf16 row and the value's, staged in
            // the misc area as packed bf16 (one 256-byte row each)
            uint32_t kb[kChunk] = {}, vb[kChunk] = {};
            int nn[kChunk] = {};
            kb[0] = smem_u32(kn) + lane * 8;
            vb[0] = smem_u32(vn) + lane * 8;
            nn[0] = 1;
            attend_chunk(st, qs, kb, vb, nn, p.scale_log2, lane);
        }
        if (sl && lane == 0) sl[kStAWarp0 + warp] = globaltimer();
        // this warp's partial: m, l per head (lane 2h holds head h), o
        float *wp = wpart + warp * WP;
#pragma unroll
        for (int h = 0; h < kRep; ++h)
#pragma unroll
            for (int e = 0; e < 4; ++e) wp[h * (kD + 2) + 4 * lane + e] = st.o[h][e];
        if (lane < 2 * kRep && (lane & 1) == 0) {
            wp[(lane >> 1) * (kD + 2) + kD] = st.m;
            wp[(lane >> 1) * (kD + 2) + kD + 1] = st.l;
        }
    }
    // (a warp whose ring wait failed carries on with what it has: the barrier
    // sequence stays the same in every warp, and the launch's next grid wait
    // reports the abort)
    consumers_sync();
    if (a.active) {
        // combine the warps into this split's partial (unnormalised o, m, l)
        for (int t = tid; t < kRep * kD; t += kCT) {
            const int h = t / kD, d = t % kD;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, wpart[w * WP + h * (kD + 2) + kD]);
            float o = 0.0f, l = 0.0f;
            for (int w = 0; w < kAttnWarps; ++w) {
                const float mw = wpart[w * WP + h * (kD + 2) + kD];
                if (mw == -INFINITY) continue;
                const float e = exp2f(mw - M);
                o = fmaf(e, wpart[w * WP + h * (kD + 2) + d], o);
                l = fmaf(e, wpart[w * WP + h * (kD + 2) + kD + 1], l);
            }
            const int row = a.g * kRep + h;
            p.part_o[((int64_t)row * p.splits + a.s) * kD + d] = o;
            if (d == 0) {
                p.part_ml[((int64_t)row * p.splits + a.s) * 2] = M;
                p.part_ml[((int64_t)row * p.splits + a.s) * 2 + 1] = l;
            }
        }
        consumers_sync();
        if (sl) sl[kStATicket] = globaltimer();
        // Post this split's partial, then wait (bounded) until every split of
        // this KV head has posted this layer's: the head's counter only grows
        // (splits per layer per token), so no reset is needed between layers.
        if (tid == 0) {
            asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.tickets + a.g) : "memory");
            const unsigned int target =
                (x.epoch * (unsigned int)p.n_layers + (unsigned int)layer + 1u) * (unsigned int)p.splits;
            unsigned int v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p.tickets + a.g) : "memory");
            if ((int)(v - target) < 0) {
                const long long start = clock64(), budget = wait_budget(p.err);
                int spins = 0;
                do {
                    if ((++spins & 63) == 0) {
                        if (*x.abort || *reinterpret_cast<volatile int *>(p.err) != 0) {
                            *x.abort = 1;
                            break;
                        }
                        if (clock64() - start > budget) {
                            note_wait(x, p, 5, layer, (int)(target - v));
                            raise_abort(x, p, DEV_ERR_WAIT_FULL);
                            break;
                        }
                    }
                    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p.tickets + a.g) : "memory");
                } while ((int)(v - target) < 0);
            }
        }
        consumers_sync();
        if (sl) sl[kStAHeadWait] = globaltimer();
        // Merge: split s takes the head group's 32-element blocks s, s + splits,
        // ... (kRep * kD / 32 = 16 of them); one warp per block, lane = element.
        // Every split's (m, l) and partial value are loaded together (one L2
        // round trip each) and summed in split order; the block's bf16
        // outputs and their planar Q8_0 (k_quants.rs:676-706) are written.
        if (warp == 0) {
            for (int blk = a.s; blk < kRep * kD / 32; blk += p.splits) {
                const int h = blk / (kD / 32), d = (blk % (kD / 32)) * 32 + lane, row = a.g * kRep + h;
                const float *ml = p.part_ml + (int64_t)row * p.splits * 2;
                const float *po = p.part_o + (int64_t)row * p.splits * kD + d;
                // (m, l) of split s in lane s (splits <= 64: two per lane at most),
                // one load each; the maximum and the weights by shuffles
                float2 mlA = make_float2(-INFINITY, 0.0f), mlB = make_float2(-INFINITY, 0.0f);
                if (lane < p.splits) mlA = __ldcg(reinterpret_cast<const float2 *>(ml) + lane);
                if (lane + 32 < p.splits) mlB = __ldcg(reinterpret_cast<const float2 *>(ml) + lane + 32);
                float M = fmaxf(mlA.x, mlB.x);
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
                const float eA = (mlA.x == -INFINITY) ? 0.0f : exp2f(mlA.x - M);
                const float eB = (mlB.x == -INFINITY) ? 0.0f : exp2f(mlB.x - M);
                float den = 0.0f, acc = 0.0f;
#pragma unroll 8
                for (int sp = 0; sp < p.splits; ++sp) {
                    const float o = __ldcg(po + (int64_t)sp * kD);
                    const float e = __shfl_sync(0xffffffffu, sp < 32 ? eA : eB, sp & 31);
                    const float l = __shfl_sync(0xffffffffu, sp < 32 ? mlA.y : mlB.y, sp & 31);
                    den = fmaf(e, l, den);
                    acc = fmaf(e, o, acc);
                }
                const float v = bfr((den == 0.0f) ? 0.0f : acc / den);
                p.attn_out[row * kD + d] = __float2bfloat16_rn(v);
                float amax = fabsf(v);
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
                const float dq = __fdiv_rn(amax, 127.0f);
                const float id = (dq != 0.0f) ? __fdiv_rn(1.0f, dq) : 0.0f;
                const int q = sat_i8r(roundf(__fmul_rn(v, id)));
                int sum = q;
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
                const int gb = a.g * kRep * kD / 32 + blk;
                p.aq[gb * 32 + lane] = (int8_t)q;
                if (lane == 0) {
                    p.ad[gb] = __half2float(__float2half_rn(dq));
                    p.ac[gb] = 12582912.0f + 8.0f * (float)sum;
                }
            }
            if (sl && lane == 0) sl[kStAMerged] = globaltimer();
        }
    }
}

// h[r] = bf16(h[r] + bf16(v)) (transformers' residual add of two bf16
// tensors); the rounded linear output also goes to `out` (its trace copy).
__device__ __forceinline__ void residual(const MegaParams &p, __nv_bfloat16 *out, int r, float v) {
    const float y = bfr(v);
    out[r] = __float2bfloat16_rn(y);
    p.h[r] = __float2bfloat16_rn(__bfloat162float(__ldcg(p.h + r)) + y);
}

// Copy the staged activation tile (the linear's exact Q8_0 input: codes in
// logical order, then the widened scales and the offsets) to trace tile t
// (0: q/k/v input of the trace layer, 1: its gate/up input, 2: lm_head input).
__device__ __forceinline__ void trace_tile(const Ctx &x, const MegaParams &p, int t) {
    const int K = p.H, tid = threadIdx.x;
    uint8_t *dst = p.trace + (size_t)t * (K + K / 4);
    for (int i = tid; i < K; i += kCT) {
        const int bk = i / 32, e = i % 32;
        dst[i] = x.base[kXsOff + xchunk(bk >> 1, (bk & 1) * 2 + e / 16) + (e % 16)];
    }
    float *fd = reinterpret_cast<float *>(dst + K);
    for (int i = tid; i < K / 32; i += kCT) {
        fd[i] = reinterpret_cast<const float *>(x.base + kXdsOff)[i];
        fd[K / 32 + i] = reinterpret_cast<const float *>(x.base + kXcsOff)[i];
    }
}

// ---- the kernel ----------------------------------------------------------------

__global__ void __launch_bounds__(kThreads, 1) decode_mega_kernel(const MegaParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    Ctx x;
    x.base = smem;
    x.full = reinterpret_cast<uint64_t *>(smem);
    x.empty = x.full + kMaxSlots;
    x.xs = smem_u32(smem + kXsOff);
    x.xds = smem_u32(smem + kXdsOff);
    x.xcs = smem_u32(smem + kXcsOff);
    x.misc = reinterpret_cast<float *>(smem + kMiscOff);
    x.ring = smem_u32(smem + kRingOff);
    x.abort = reinterpret_cast<volatile int *>(x.misc + kBcastOff);
    x.G = gridDim.x;
    x.c = blockIdx.x;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nbar = 5 * p.n_layers + 1;
    const unsigned int epoch = *reinterpret_cast<volatile const unsigned int *>(p.epoch);
    x.bar_base = (unsigned long long)epoch * (unsigned long long)nbar * (unsigned long long)x.G;
    x.epoch = epoch;
    const int pos = *reinterpret_cast<volatile const int *>(p.pos);
    if (tid == 0) {
        for (int s = 0; s < p.nslots; ++s) {
            mbar_init(&x.full[s], 1);
            mbar_init(&x.empty[s], kAttnWarps);
        }
        fence_mbar_init();
        *x.abort = 0;
    }
    __syncthreads();
    if (pos < 0 || pos >= p.cap) {
        if (tid == 0) record_device_error(p.err, DEV_ERR_WAIT_FULL);
        return;
    }
    if (warp == kCW) {
        if (lane == 0) producer(x, p, pos);
        return;
    }
    const int G = x.G, c = x.c;
    const int QKV = (p.Hq + 2 * p.Hkv) * kD;
    // the shares are recomputed per phase (a few integer operations) rather
    // than kept live across the layer loop
    uint32_t item = 0;
    int b = 0;  // grid barriers passed
    bool ok = true;
    float *actv = x.misc + kActOff;
    unsigned long long *st = (p.stamps && p.n_layers > 1 && tid == 0) ? p.stamps + (size_t)c * kStamps : nullptr;
    if (st) st[kStStart] = globaltimer();
    for (int l = 0; l < p.n_layers && ok; ++l) {
        const MegaLayer L = p.layers[l];
        const bool tr = (l == p.trace_layer) && p.trace;
        unsigned long long *sl = (l == 1) ? st : nullptr;
        // ring order per layer: this CTA's first K/V tiles, q/k/v, the other
        // K/V tiles, then o, gate/up, down
        const Att at = att_share(p, c, pos);
        const int early = kv_early(p, at, lin_share(QKV, p.H, c, G, 4).items);
        const uint32_t kv0 = item;
        item += 2u * (uint32_t)early;
        // ---- Q: RMSNorm -> Q8_0, q/k/v rows
        if (l == 0) {
            int tok = __ldcg(p.tokens);
            if (tok < 0 || tok >= p.V) {  // an id outside the vocabulary: recorded, row 0 read instead
                if (tid == 0) record_device_error(p.err, DEV_ERR_WAIT_FULL);
                tok = 0;
            }
            const Lin so = lin_share(p.H, p.Hq * kD, c, G, 4);
            stage_rmsnorm(x, p, p.embed + (int64_t)tok * p.H, L.attn_norm, p.H, p.h, so.r0, so.r1);
        } else {
            ok = grid_wait(x, p, b++);
            if (!ok) break;
            if (sl) sl[kStQWait] = globaltimer();
            stage_rmsnorm(x, p, p.h, L.attn_norm, p.H, nullptr, 0, 0);
            if (sl) sl[kStQStaged] = globaltimer();
        }
        if (tr && c == 0) trace_tile(x, p, 0);
        consume_linear(x, p, lin_share(QKV, p.H, c, G, 4), item, [&](int ln, int r0, float v, int nr) {
            if ((ln & 3) == 0 && (ln >> 2) < nr) p.qkv_out[r0 + (ln >> 2)] = __float2bfloat16_rn(v);
        }, sl);
        if (l == 1 && p.stamps && lane == 0) p.stamps[(size_t)c * kStamps + kStQWarp0 + warp] = globaltimer();
        grid_arrive(x, p);
        if (sl) sl[kStQDone] = globaltimer();
        const uint32_t kv1 = item;  // where the later K/V tiles start
        item += 2u * (uint32_t)(at.tiles - early);
        // ---- A: attention
        ok = grid_wait(x, p, b++);
        if (!ok) break;
        if (sl) sl[kStAWait] = globaltimer();
        attention_phase(x, p, L, l, pos, kv0, kv1, early, sl);
        grid_arrive(x, p);
        if (sl) sl[kStADone] = globaltimer();
        // ---- O: o_proj + residual
        ok = grid_wait(x, p, b++);
        if (!ok) break;
        if (sl) sl[kStOWait] = globaltimer();
        stage_planar(x, p.aq, p.ad, p.ac, p.Hq * kD);
        consume_linear(x, p, lin_share(p.H, p.Hq * kD, c, G, 4), item, [&](int ln, int r0, float v, int nr) {
            if ((ln & 3) == 0 && (ln >> 2) < nr) residual(p, p.o_out, r0 + (ln >> 2), v);
        });
        grid_arrive(x, p);
        if (sl) sl[kStODone] = globaltimer();
        // ---- G: RMSNorm -> Q8_0, gate/up pairs -> act, act -> planar Q8_0
        ok = grid_wait(x, p, b++);
        if (!ok) break;
        if (sl) sl[kStGWait] = globaltimer();
        stage_rmsnorm(x, p, p.h, L.mlp_norm, p.H, nullptr, 0, 0);
        if (tr && c == 0) trace_tile(x, p, 1);
        const int g_r0 = gu_share(p.I, p.H, c, G).r0;
        consume_linear(x, p, gu_share(p.I, p.H, c, G), item, [&](int ln, int r0, float v, int nr) {
            // rows come in (gate, up) pairs: row 2j in lane 8j, row 2j + 1 in lane
            // 8j + 4; act = bf16(bf16(silu(g)) * u) with g and u rounded to bf16
            // first (transformers' LlamaMLP in bf16)
            const float u = __shfl_down_sync(0xffffffffu, v, 4);
            if ((ln & 7) == 0 && (ln >> 2) < nr) {
                const float gb = bfr(v), ub = bfr(u);
                actv[(r0 + (ln >> 2) - g_r0) >> 1] = bfr(bfr(gb / (1.0f + expf(-gb))) * ub);
            }
        });
        consumers_sync();
        // quantise this CTA's act blocks (one warp per 32-column block)
        {
            const Lin sg = gu_share(p.I, p.H, c, G);
            const int u0 = sg.r0 / 64, nu = (sg.r1 - sg.r0) / 64;
            for (int u = warp; u < nu; u += kCW) {
                const float v = actv[u * 32 + lane];
                float amax = fabsf(v);
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
                const float d = __fdiv_rn(amax, 127.0f);
                const float id = (d != 0.0f) ? __fdiv_rn(1.0f, d) : 0.0f;
                const int q = sat_i8r(roundf(__fmul_rn(v, id)));
                int sum = q;
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
                const int gb = u0 + u;
                p.gq[gb * 32 + lane] = (int8_t)q;
                p.act_out[gb * 32 + lane] = __float2bfloat16_rn(v);
                if (lane == 0) {
                    p.gd[gb] = __half2float(__float2half_rn(d));
                    p.gc[gb] = 12582912.0f + 8.0f * (float)sum;
                }
            }
        }
        grid_arrive(x, p);
        if (sl) sl[kStGDone] = globaltimer();
        // ---- D: down_proj + residual
        ok = grid_wait(x, p, b++);
        if (!ok) break;
        if (sl) sl[kStDWait] = globaltimer();
        stage_planar(x, p.gq, p.gd, p.gc, p.I);
        consume_linear(x, p, lin_share(p.H, p.I, c, G), item, [&](int ln, int r0, float v, int nr) {
            if ((ln & 3) == 0 && (ln >> 2) < nr) residual(p, p.down_out, r0 + (ln >> 2), v);
        });
        grid_arrive(x, p);
        if (sl) sl[kStDDone] = globaltimer();
    }
    if (!ok) return;
    // ---- F: final norm, lm_head, argmax
    ok = grid_wait(x, p, b++);
    if (!ok) return;
    stage_rmsnorm(x, p, p.h, p.final_norm, p.H, nullptr, 0, 0);
    float2 *arg = reinterpret_cast<float2 *>(x.misc + kArgOff);
    float best_v = -INFINITY;
    int best_i = 0x7fffffff;
    if (p.trace && c == 0) trace_tile(x, p, 2);
    consume_linear(x, p, lin_share(p.V, p.H, c, G), item, [&](int ln, int r0, float v, int nr) {
        if ((ln & 3) == 0 && (ln >> 2) < nr) {
            const int r = r0 + (ln >> 2);
            const float y = bfr(v);
            p.logits[r] = __float2bfloat16_rn(y);
            if (y > best_v || (y == best_v && r < best_i)) {
                best_v = y;
                best_i = r;
            }
        }
    });
    // the warp's best (value, first index) across its lanes
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best_v, off);
        const int oi = __shfl_xor_sync(0xffffffffu, best_i, off);
        if (ov > best_v || (ov == best_v && oi < best_i)) best_v = ov, best_i = oi;
    }
    if (lane == 0) arg[warp] = make_float2(best_v, __int_as_float(best_i));
    consumers_sync();
    if (tid == 0) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int w = 0; w < kCW; ++w) {
            const float v = arg[w].x;
            const int i = __float_as_int(arg[w].y);
            if (v > bv || (v == bv && i < bi)) bv = v, bi = i;
        }
        p.amax_part[c] = make_float2(bv, __int_as_float(bi));
    }
    grid_arrive(x, p);
    if (st) st[kStEnd] = globaltimer();
    if (c != 0) return;
    ok = grid_wait(x, p, b++);
    if (!ok) return;
    if (warp == 0) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int i = lane; i < G; i += 32) {
            const float2 e = __ldcg(p.amax_part + i);
            const int ei = __float_as_int(e.y);
            if (e.x > bv || (e.x == bv && ei < bi)) bv = e.x, bi = ei;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
            if (ov > bv || (ov == bv && oi < bi)) bv = ov, bi = oi;
        }
        if (lane == 0) {
            p.tokens[0] = bi;
            p.pos[0] = pos + 1;
            __threadfence();
            atomicAdd(p.epoch, 1u);
        }
    }
}

}  // namespace
}  // namespace tn

// ---- host side -------------------------------------------------------------------

namespace tn {
namespace {

struct MegaPlan {
    MegaParams p;  // tokens / pos / logits / trace filled per launch
    size_t sync_off = 0, sync_bytes = 0;
    uint8_t *ws = nullptr;
    int grid = 0;
    size_t smem = 0;
};

int64_t align256(int64_t v) { return (v + 255) & ~int64_t(255); }

int check_model(const tn_llama_q4_model *m, const std::string &op) {
    if (!m) return set_error(TN_ERR_INVALID, op + ": null model");
    const int L = m->layers, H = m->hidden, I = m->inter, Hq = m->heads, Hkv = m->kv_heads, D = m->head_dim,
              V = m->vocab;
    if (L <= 0 || H <= 0 || I <= 0 || Hq <= 0 || Hkv <= 0 || V <= 0 || m->capacity <= 0)
        return set_error(TN_ERR_SHAPE, op + ": every size must be positive");
    if (D != kD || Hq != kRep * Hkv)
        return set_error(TN_ERR_NOT_IMPLEMENTED, op + ": the persistent decode kernel takes head_dim 128 and 4 query "
                                                      "heads per key/value head (Llama-3-8B's shape family)");
    if (H % 256 != 0 || I % 256 != 0 || (Hq * D) % 256 != 0 || H / 16 > kCT || I > kMaxK || Hq * D > kMaxK)
        return set_error(TN_ERR_NOT_IMPLEMENTED, op + ": hidden and intermediate sizes must be multiples of 256 "
                                                      "(hidden <= 5632, intermediate <= 16384)");
    return TN_OK;
}

// Offsets of the workspace (bytes, 256-aligned) for this model on a grid of G CTAs.
void layout(const tn_llama_q4_model *m, int G, int splits, tn_llama_decode_layout *o) {
    const int64_t H = m->hidden, I = m->inter, Hq = m->heads, Hkv = m->kv_heads, D = m->head_dim;
    const int64_t QKV = (Hq + 2 * Hkv) * D, HD = Hq * D;
    int64_t off = 0;
    auto take = [&](int64_t bytes) {
        const int64_t at = off;
        off = align256(off + bytes);
        return at;
    };
    o->layers = take((int64_t)sizeof(MegaLayer) * m->layers);
    o->h = take(2 * H);
    o->qkv = take(2 * QKV);
    o->attn = take(2 * HD);
    o->act = take(2 * I);
    o->o_out = take(2 * H);
    o->down_out = take(2 * H);
    o->aq = take(HD);
    o->ad = take(4 * HD / 32);
    o->ac = take(4 * HD / 32);
    o->gq = take(I);
    o->gd = take(4 * I / 32);
    o->gc = take(4 * I / 32);
    o->part_o = take(4 * Hq * splits * D);
    o->part_ml = take(8 * Hq * splits);
    o->amax = take(8 * (int64_t)G);
    o->sync = take(((4 * Hkv + 7) & ~int64_t(7)) + 32);  // tickets [Hkv], barrier u64, epoch u32, diag int[4]
    o->total = off;
}

int grid_facts(int *G, int *splits, int *nslots, size_t *smem, int Hkv) {
    DeviceFacts f{};
    int st = device_facts(&f);
    if (st) return st;
    *G = f.sm_count;
    *splits = f.sm_count / Hkv < kMaxSplits ? f.sm_count / Hkv : kMaxSplits;
    int ns = (int)(((size_t)f.smem_optin - kRingOff) / kSlot);
    if (ns > kMaxSlots) ns = kMaxSlots;
    *nslots = ns / kCW * kCW;  // a multiple of the consumer warps (consume_linear)
    *smem = kRingOff + (size_t)(*nslots) * kSlot;
    return TN_OK;
}

}  // namespace
}  // namespace tn

extern "C" int tn_llama_decode_layout_of(const tn_llama_q4_model *m, tn_llama_decode_layout *out) {
    using namespace tn;
    const std::string op = "tn_llama_decode_layout_of";
    int st = check_model(m, op);
    if (st) return st;
    if (!out) return set_error(TN_ERR_INVALID, op + ": null output");
    int G, splits, nslots;
    size_t smem;
    st = grid_facts(&G, &splits, &nslots, &smem, m->kv_heads);
    if (st) return st;
    layout(m, G, splits < 1 ? 1 : splits, out);
    return TN_OK;
}

extern "C" int tn_llama_decode_plan(const tn_llama_q4_model *m, void *workspace, int64_t workspace_bytes,
                                    void **plan_out) {
    using namespace tn;
    const std::string op = "tn_llama_decode_plan";
    if (!plan_out) return set_error(TN_ERR_INVALID, op + ": null plan pointer");
    *plan_out = nullptr;
    int st = check_model(m, op);
    if (st) return st;
    if (!m->embed || !m->final_norm || !m->lm_head || !m->attn_norm || !m->qkv || !m->o || !m->mlp_norm ||
        !m->gate_up || !m->down || !m->k_cache || !m->v_cache || !m->inv_freq)
        return set_error(TN_ERR_INVALID, op + ": null pointer in the model description");
    int G, splits, nslots;
    size_t smem;
    st = grid_facts(&G, &splits, &nslots, &smem, m->kv_heads);
    if (st) return st;
    if (splits < 1) return set_error(TN_ERR_NOT_IMPLEMENTED, op + ": more key/value heads than SMs");
    if ((2 * m->inter / 64 + G - 1) / G > kMaxUnitsG)
        return set_error(TN_ERR_NOT_IMPLEMENTED, op + ": intermediate size too large for the grid");
    if (nslots < kCW) return set_error(TN_ERR_NOT_IMPLEMENTED, op + ": not enough shared memory for the weight ring");
    tn_llama_decode_layout lo{};
    layout(m, G, splits, &lo);
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255) != 0 || workspace_bytes < lo.total)
        return set_error(TN_ERR_INVALID, op + ": the workspace must be 256-byte aligned device memory of at least " +
                                             std::to_string(lo.total) + " bytes (tn_llama_decode_layout_of)");
    const int L = m->layers;
    std::vector<MegaLayer> layers((size_t)L);
    for (int l = 0; l < L; ++l) {
        layers[l].qkv = static_cast<const uint8_t *>(m->qkv[l]);
        layers[l].o = static_cast<const uint8_t *>(m->o[l]);
        layers[l].gate_up = static_cast<const uint8_t *>(m->gate_up[l]);
        layers[l].down = static_cast<const uint8_t *>(m->down[l]);
        layers[l].attn_norm = static_cast<const __nv_bfloat16 *>(m->attn_norm[l]);
        layers[l].mlp_norm = static_cast<const __nv_bfloat16 *>(m->mlp_norm[l]);
        layers[l].kc = static_cast<__nv_bfloat16 *>(m->k_cache[l]);
        layers[l].vc = static_cast<__nv_bfloat16 *>(m->v_cache[l]);
        const void *ptrs[] = {layers[l].qkv, layers[l].o, layers[l].gate_up, layers[l].down, layers[l].kc,
                              layers[l].vc, layers[l].attn_norm, layers[l].mlp_norm};
        for (const void *q : ptrs)
            if (!q || (reinterpret_cast<uintptr_t>(q) & 15) != 0)
                return set_error(TN_ERR_INVALID, op + ": layer " + std::to_string(l) +
                                                     ": weights, norms and caches must be non-null and 16-byte aligned");
    }
    uint8_t *b = static_cast<uint8_t *>(workspace);
    st = check_cuda(cudaMemcpy(b + lo.layers, layers.data(), sizeof(MegaLayer) * (size_t)L, cudaMemcpyHostToDevice),
                    op.c_str(), "cudaMemcpy");
    if (st) return st;
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        st = check_cuda(cudaFuncSetAttribute(decode_mega_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                        op.c_str(), "cudaFuncSetAttribute");
        if (st) return st;
        configured[dev] = true;
    }
    int per_sm = 0;
    st = check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_mega_kernel, kThreads, smem),
                    op.c_str(), "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    if (st) return st;
    if (per_sm < 1) return set_error(TN_ERR_NOT_IMPLEMENTED, op + ": the kernel does not fit on an SM");

    MegaPlan *pl = new MegaPlan();
    MegaParams &p = pl->p;
    p.layers = reinterpret_cast<const MegaLayer *>(b + lo.layers);
    p.n_layers = L;
    p.embed = static_cast<const __nv_bfloat16 *>(m->embed);
    p.final_norm = static_cast<const __nv_bfloat16 *>(m->final_norm);
    p.lm_head = static_cast<const uint8_t *>(m->lm_head);
    p.inv_freq = m->inv_freq;
    p.H = m->hidden, p.I = m->inter, p.Hq = m->heads, p.Hkv = m->kv_heads, p.V = m->vocab;
    p.eps = m->eps;
    p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)m->head_dim));
    p.cap = m->capacity;
    p.kv_hstride = m->capacity * m->head_dim;
    p.h = reinterpret_cast<__nv_bfloat16 *>(b + lo.h);
    p.qkv_out = reinterpret_cast<__nv_bfloat16 *>(b + lo.qkv);
    p.attn_out = reinterpret_cast<__nv_bfloat16 *>(b + lo.attn);
    p.act_out = reinterpret_cast<__nv_bfloat16 *>(b + lo.act);
    p.o_out = reinterpret_cast<__nv_bfloat16 *>(b + lo.o_out);
    p.down_out = reinterpret_cast<__nv_bfloat16 *>(b + lo.down_out);
    p.aq = reinterpret_cast<int8_t *>(b + lo.aq);
    p.ad = reinterpret_cast<float *>(b + lo.ad);
    p.ac = reinterpret_cast<float *>(b + lo.ac);
    p.gq = reinterpret_cast<int8_t *>(b + lo.gq);
    p.gd = reinterpret_cast<float *>(b + lo.gd);
    p.gc = reinterpret_cast<float *>(b + lo.gc);
    p.part_o = reinterpret_cast<float *>(b + lo.part_o);
    p.part_ml = reinterpret_cast<float *>(b + lo.part_ml);
    p.amax_part = reinterpret_cast<float2 *>(b + lo.amax);
    p.tickets = reinterpret_cast<int *>(b + lo.sync);
    p.bar = reinterpret_cast<unsigned long long *>(b + lo.sync + ((4 * (int64_t)m->kv_heads + 7) & ~int64_t(7)));
    p.epoch = reinterpret_cast<unsigned int *>(reinterpret_cast<uint8_t *>(p.bar) + 8);
    p.diag = reinterpret_cast<int *>(reinterpret_cast<uint8_t *>(p.bar) + 16);
    p.err = device_error_word();
    p.splits = splits;
    p.nslots = nslots;
    p.trace_layer = -1;
    p.trace = nullptr;
    p.stamps = nullptr;
    pl->ws = b;
    pl->sync_off = (size_t)lo.sync;
    pl->sync_bytes = (size_t)(lo.total - lo.sync);
    pl->grid = G;
    pl->smem = smem;
    *plan_out = pl;
    return TN_OK;
}

extern "C" int64_t tn_llama_decode_trace_bytes(const void *plan) {
    if (!plan) return 0;
    const tn::MegaParams &p = static_cast<const tn::MegaPlan *>(plan)->p;
    return 3 * (int64_t)(p.H + p.H / 4);
}

extern "C" int tn_llama_decode_token(void *plan, int *tokens, int *pos, void *logits, void *trace, int trace_layer,
                                     void *stream_) {
    using namespace tn;
    const std::string op = "tn_llama_decode_token";
    if (!plan || !tokens || !pos || !logits) return set_error(TN_ERR_INVALID, op + ": null argument");
    MegaPlan *pl = static_cast<MegaPlan *>(plan);
    MegaParams p = pl->p;
    p.tokens = tokens;
    p.pos = pos;
    p.logits = static_cast<__nv_bfloat16 *>(logits);
    p.trace = static_cast<uint8_t *>(trace);
    p.trace_layer = trace ? trace_layer : -1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)pl->grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = pl->smem;
    cfg.stream = tn::stream_of(stream_);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int st = check_cuda(cudaLaunchKernelEx(&cfg, decode_mega_kernel, p), op.c_str(), "cudaLaunchKernelEx");
    if (st) return st;
    __atomic_fetch_add(&counters().decode_token_launches, 1ull, __ATOMIC_RELAXED);
    return TN_OK;
}

extern "C" int tn_llama_decode_token_timeline(void *plan, int *tokens, int *pos, void *logits, uint64_t *stamps,
                                              void *stream_) {
    using namespace tn;
    if (!plan || !stamps) return set_error(TN_ERR_INVALID, "tn_llama_decode_token_timeline: null argument");
    MegaPlan *pl = static_cast<MegaPlan *>(plan);
    pl->p.stamps = reinterpret_cast<unsigned long long *>(stamps);
    const int st = tn_llama_decode_token(plan, tokens, pos, logits, nullptr, -1, stream_);
    pl->p.stamps = nullptr;
    return st;
}

extern "C" int tn_llama_decode_reset(void *plan, void *stream) {
    using namespace tn;
    if (!plan) return set_error(TN_ERR_INVALID, "tn_llama_decode_reset: null plan");
    MegaPlan *pl = static_cast<MegaPlan *>(plan);
    return check_cuda(cudaMemsetAsync(pl->ws + pl->sync_off, 0, pl->sync_bytes, tn::stream_of(stream)),
                      "tn_llama_decode_reset", "cudaMemsetAsync");
}

extern "C" int tn_llama_decode_plan_free(void *plan) {
    delete static_cast<tn::MegaPlan *>(plan);
    return TN_OK;
}
