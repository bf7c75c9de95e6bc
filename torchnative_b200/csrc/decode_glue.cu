// decode_glue.cu -- the element-wise and row-wise work between the two hot
// operators in one greedy decode token of a Llama-shaped model (the caller is
// transformers' LlamaForCausalLM: RMSNorm, rotary embedding + KV append,
// SiLU * up, argmax, embedding lookup), written to hand the next Q4_0 linear
// its activations already in planar Q8_0 form.
//
// Arithmetic follows transformers' Llama modules in bf16 storage:
//   RMSNorm  y = w * bf16(x32 * rsqrt(mean(x32^2) + eps))     (LlamaRMSNorm)
//   RoPE     q' = bf16(bf16(q*cos) + bf16(rot(q)*sin)), cos/sin = bf16(cos/sin(inv_freq*pos))
//   MLP      a = bf16(bf16(silu(g)) * u)
//   residual h = bf16(h + delta)
// and then the Q8_0 activation quantiser of k_quants.rs:676-706.
#include "q4_kernels.cuh"

namespace tn {
namespace {

__device__ __forceinline__ float bf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Rust `v as i8` after f32::round: saturate, NaN -> 0 (the Q8_0 writer).
__device__ __forceinline__ int sat_i8r(float v) {
    if (!(v == v)) return 0;
    if (v <= -128.0f) return -128;
    if (v >= 127.0f) return 127;
    return __float2int_rz(v);
}

// Quantise 32 consecutive values held by one warp (one per lane) to a Q8_0
// block in planar form: lane j writes code j; lane 0 writes scale and offset.
__device__ __forceinline__ void q8_block_warp(float v, int lane, int8_t *codes, float *scale, float *offset) {
    float amax = fabsf(v);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = (d != 0.0f) ? __fdiv_rn(1.0f, d) : 0.0f;
    const int q = sat_i8r(roundf(__fmul_rn(v, id)));
    codes[lane] = static_cast<int8_t>(q);
    int s = q;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) {
        *scale = __half2float(__float2half_rn(d));
        *offset = 12582912.0f + 8.0f * static_cast<float>(s);
    }
}

// h_out = bf16(h + delta) (delta optional), y = RMSNorm(h_out) * w, y -> Q8_0.
// One CTA of 256 threads per row; H % 32 == 0, H <= 8192.
__global__ void __launch_bounds__(256) add_rmsnorm_q8_kernel(const __nv_bfloat16 *__restrict__ h,
                                                             const __nv_bfloat16 *__restrict__ delta,
                                                             __nv_bfloat16 *__restrict__ h_out,
                                                             const __nv_bfloat16 *__restrict__ w, float eps, int H,
                                                             int8_t *codes, float *scales, float *offsets) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float xs[8192];
    __shared__ float red[8];
    const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const __nv_bfloat16 *hr = h + (int64_t)row * H;
    float ss = 0.0f;
    for (int i = tid; i < H; i += 256) {
        float x = __bfloat162float(hr[i]);
        if (delta) x = bf(x + __bfloat162float(delta[(int64_t)row * H + i]));
        if (h_out) h_out[(int64_t)row * H + i] = __float2bfloat16_rn(x);
        xs[i] = x;
        ss = fmaf(x, x, ss);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += red[i];
    const float r = rsqrtf(tot / (float)H + eps);
    const int nb = H / 32;
    for (int blk = warp; blk < nb; blk += 8) {
        const int i = blk * 32 + lane;
        const float y = bf(__bfloat162float(w[i]) * bf(xs[i] * r));
        q8_block_warp(y, lane, codes + (int64_t)row * H + blk * 32, scales + (int64_t)row * nb + blk,
                      offsets + (int64_t)row * nb + blk);
    }
}

// act = bf16(bf16(silu(g)) * u) from gate/up rows [B][2I] (gate first), -> Q8_0.
__global__ void __launch_bounds__(256) silu_mul_q8_kernel(const __nv_bfloat16 *__restrict__ gu, int I, int8_t *codes,
                                                          float *scales, float *offsets) {
    pdl_launch_dependents();
    pdl_wait();
    const int row = blockIdx.y, lane = threadIdx.x & 31;
    const int blk = blockIdx.x * 8 + (threadIdx.x >> 5), nb = I / 32;
    if (blk >= nb) return;
    const int i = blk * 32 + lane;
    const float g = __bfloat162float(gu[(int64_t)row * 2 * I + i]);
    const float u = __bfloat162float(gu[(int64_t)row * 2 * I + I + i]);
    const float s = bf(g / (1.0f + expf(-g)));
    q8_block_warp(bf(s * u), lane, codes + (int64_t)row * I + blk * 32, scales + (int64_t)row * nb + blk,
                  offsets + (int64_t)row * nb + blk);
}

// Rotary embedding of q and k (rotate_half convention) at position pos and the
// append of k, v to the cache slot pos. qkv rows are [q heads | k heads | v heads].
// Grid (Hq + Hkv, B), D/2 threads: one (head, pair i, i + D/2) per thread.
__global__ void rope_append_kernel(const __nv_bfloat16 *__restrict__ qkv, const float *__restrict__ inv_freq,
                                   const int *__restrict__ pos_dev, int pos_host, int Hq, int Hkv, int D,
                                   __nv_bfloat16 *__restrict__ q_out, __nv_bfloat16 *__restrict__ k_cache,
                                   __nv_bfloat16 *__restrict__ v_cache, int64_t cache_b_stride,
                                   int64_t cache_h_stride) {
    pdl_launch_dependents();
    pdl_wait();
    const int head = blockIdx.x, b = blockIdx.y, i = threadIdx.x, half = D / 2;
    const int pos = pos_dev ? *pos_dev : pos_host;
    const int W = (Hq + 2 * Hkv) * D;
    const __nv_bfloat16 *row = qkv + (int64_t)b * W;
    const float f = inv_freq[i] * (float)pos;
    const float c = bf(cosf(f)), s = bf(sinf(f));
    const bool is_q = head < Hq;
    const int src = is_q ? head * D : (Hq + (head - Hq)) * D;
    const float x1 = __bfloat162float(row[src + i]), x2 = __bfloat162float(row[src + i + half]);
    // q*cos + rotate_half(q)*sin, rotate_half(x) = (-x2, x1)
    const float y1 = bf(bf(x1 * c) + bf(-x2 * s));
    const float y2 = bf(bf(x2 * c) + bf(x1 * s));
    if (is_q) {
        __nv_bfloat16 *qo = q_out + ((int64_t)b * Hq + head) * D;
        qo[i] = __float2bfloat16_rn(y1);
        qo[i + half] = __float2bfloat16_rn(y2);
    } else {
        const int kh = head - Hq;
        __nv_bfloat16 *kc = k_cache + b * cache_b_stride + kh * cache_h_stride + (int64_t)pos * D;
        __nv_bfloat16 *vc = v_cache + b * cache_b_stride + kh * cache_h_stride + (int64_t)pos * D;
        kc[i] = __float2bfloat16_rn(y1);
        kc[i + half] = __float2bfloat16_rn(y2);
        const __nv_bfloat16 *vr = row + (Hq + Hkv + kh) * D;
        vc[i] = vr[i];
        vc[i + half] = vr[i + half];
    }
}

// Greedy pick (first index of the maximum, torch.argmax) per row, then the
// next token's embedding row; thread 0 of row 0 advances the position.
__global__ void __launch_bounds__(1024) argmax_embed_kernel(const __nv_bfloat16 *__restrict__ logits, int V,
                                                            int *__restrict__ tokens,
                                                            const __nv_bfloat16 *__restrict__ embed, int H,
                                                            __nv_bfloat16 *__restrict__ h, int *pos_dev) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float bv[32];
    __shared__ int bi[32];
    __shared__ int winner;
    const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const __nv_bfloat16 *lr = logits + (int64_t)row * V;
    float best = -INFINITY;
    int idx = 0x7fffffff;
    // 16-byte loads, kU of them in flight per thread before any compare (a
    // row is ~250 KB read by one CTA: latency, not bandwidth, bounds it)
    constexpr int kU = 8;
    const int nvec = ((reinterpret_cast<uintptr_t>(lr) & 15) == 0) ? V / 8 : 0;
    const uint4 *lv = reinterpret_cast<const uint4 *>(lr);
    for (int base = 0; base < nvec; base += kU * (int)blockDim.x) {
        uint4 r[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int j = base + u * (int)blockDim.x + tid;
            r[u] = j < nvec ? __ldcs(lv + j) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int j = base + u * (int)blockDim.x + tid;
            if (j >= nvec) break;
            const uint32_t w[4] = {r[u].x, r[u].y, r[u].z, r[u].w};
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float v = __uint_as_float((e & 1) ? (w[e >> 1] & 0xffff0000u) : (w[e >> 1] << 16));
                const int i = j * 8 + e;
                if (v > best || (v == best && i < idx)) best = v, idx = i;
            }
        }
    }
    for (int i = nvec * 8 + tid; i < V; i += blockDim.x) {
        const float v = __bfloat162float(lr[i]);
        if (v > best || (v == best && i < idx)) best = v, idx = i;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, off);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, off);
        if (ov > best || (ov == best && oi < idx)) best = ov, idx = oi;
    }
    if (lane == 0) bv[warp] = best, bi[warp] = idx;
    __syncthreads();
    if (warp == 0) {
        const int nw = blockDim.x / 32;
        best = lane < nw ? bv[lane] : -INFINITY;
        idx = lane < nw ? bi[lane] : 0x7fffffff;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, off);
            const int oi = __shfl_xor_sync(0xffffffffu, idx, off);
            if (ov > best || (ov == best && oi < idx)) best = ov, idx = oi;
        }
        if (lane == 0) {
            winner = idx;
            tokens[row] = idx;
        }
    }
    __syncthreads();
    const int tok = winner;
    for (int i = tid; i < H; i += blockDim.x) h[(int64_t)row * H + i] = embed[(int64_t)tok * H + i];
    if (row == 0 && tid == 0 && pos_dev) *pos_dev += 1;
}

__global__ void embed_kernel(const int *__restrict__ tokens, const __nv_bfloat16 *__restrict__ embed, int H,
                             __nv_bfloat16 *__restrict__ h) {
    pdl_launch_dependents();
    pdl_wait();
    const int row = blockIdx.x;
    const int tok = tokens[row];
    for (int i = threadIdx.x; i < H; i += blockDim.x) h[(int64_t)row * H + i] = embed[(int64_t)tok * H + i];
}

// Tensor-parallel gather layout fix: an all-gather of per-rank [rows][c]
// blocks lands as [G][rows][c]; the next layer reads [rows][G * c].
__global__ void tp_unshard_kernel(const uint16_t *__restrict__ src, uint16_t *__restrict__ dst, int G, int rows,
                                  int c) {
    pdl_launch_dependents();
    pdl_wait();
    const int64_t n = (int64_t)G * rows * c;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = i % c, r = (i / c) % rows, g = i / ((int64_t)c * rows);
        dst[r * (int64_t)G * c + g * c + j] = src[i];
    }
}

template <typename K, typename... Args>
int launch_pdl(K kernel, dim3 grid, dim3 block, cudaStream_t stream, const char *what, Args... args) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return check_cuda(cudaLaunchKernelEx(&cfg, kernel, args...), what, "cudaLaunchKernelEx");
}

}  // namespace
}  // namespace tn

using tn::launch_pdl;

extern "C" int tn_llama_add_rmsnorm_q8(const void *h, const void *delta, void *h_out, const void *weight, float eps,
                                       int64_t rows, int64_t H, int8_t *codes, float *scales, float *offsets,
                                       void *stream) {
    if (H % 32 != 0 || H > 8192 || rows < 0)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED, "tn_llama_add_rmsnorm_q8: hidden size must be a multiple of 32 "
                                                     "and at most 8192");
    if (rows == 0) return TN_OK;
    return launch_pdl(tn::add_rmsnorm_q8_kernel, dim3((unsigned)rows), dim3(256), tn::stream_of(stream),
                      "tn_llama_add_rmsnorm_q8", (const __nv_bfloat16 *)h, (const __nv_bfloat16 *)delta,
                      (__nv_bfloat16 *)h_out, (const __nv_bfloat16 *)weight, eps, (int)H, codes, scales, offsets);
}

extern "C" int tn_llama_silu_mul_q8(const void *gate_up, int64_t rows, int64_t I, int8_t *codes, float *scales,
                                    float *offsets, void *stream) {
    if (I % 32 != 0 || rows < 0)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED, "tn_llama_silu_mul_q8: intermediate size must be a multiple of 32");
    if (rows == 0) return TN_OK;
    const int nb = (int)(I / 32);
    return launch_pdl(tn::silu_mul_q8_kernel, dim3((unsigned)((nb + 7) / 8), (unsigned)rows), dim3(256),
                      tn::stream_of(stream), "tn_llama_silu_mul_q8", (const __nv_bfloat16 *)gate_up, (int)I, codes,
                      scales, offsets);
}

extern "C" int tn_llama_rope_append(const void *qkv, const float *inv_freq, const int *pos_dev, int64_t pos_host,
                                    int64_t B, int64_t Hq, int64_t Hkv, int64_t D, void *q_out, void *k_cache,
                                    void *v_cache, int64_t cache_b_stride, int64_t cache_h_stride, void *stream) {
    if (D % 2 != 0 || D > 1024 || B < 0)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED, "tn_llama_rope_append: head dimension must be even and <= 1024");
    if (B == 0) return TN_OK;
    return launch_pdl(tn::rope_append_kernel, dim3((unsigned)(Hq + Hkv), (unsigned)B), dim3((unsigned)(D / 2)),
                      tn::stream_of(stream), "tn_llama_rope_append", (const __nv_bfloat16 *)qkv, inv_freq, pos_dev,
                      (int)pos_host, (int)Hq, (int)Hkv, (int)D, (__nv_bfloat16 *)q_out, (__nv_bfloat16 *)k_cache,
                      (__nv_bfloat16 *)v_cache, cache_b_stride, cache_h_stride);
}

extern "C" int tn_llama_argmax_embed(const void *logits, int64_t rows, int64_t V, int *tokens, const void *embed,
                                     int64_t H, void *h, int *pos_dev, void *stream) {
    if (rows <= 0) return TN_OK;
    return launch_pdl(tn::argmax_embed_kernel, dim3((unsigned)rows), dim3(1024), tn::stream_of(stream),
                      "tn_llama_argmax_embed", (const __nv_bfloat16 *)logits, (int)V, tokens,
                      (const __nv_bfloat16 *)embed, (int)H, (__nv_bfloat16 *)h, pos_dev);
}

extern "C" int tn_llama_embed(const int *tokens, int64_t rows, const void *embed, int64_t H, void *h, void *stream) {
    if (rows <= 0) return TN_OK;
    return launch_pdl(tn::embed_kernel, dim3((unsigned)rows), dim3(256), tn::stream_of(stream), "tn_llama_embed",
                      tokens, (const __nv_bfloat16 *)embed, (int)H, (__nv_bfloat16 *)h);
}

extern "C" int tn_tp_unshard(const void *src, void *dst, int64_t G, int64_t rows, int64_t cols, void *stream) {
    if (G <= 0 || rows < 0 || cols < 0) return tn::set_error(TN_ERR_SHAPE, "tn_tp_unshard: negative size");
    if (rows == 0 || cols == 0) return TN_OK;
    if (!src || !dst || src == dst) return tn::set_error(TN_ERR_INVALID, "tn_tp_unshard: src and dst must be distinct");
    const int64_t n = G * rows * cols;
    const unsigned blocks = (unsigned)((n + 255) / 256 < 1184 ? (n + 255) / 256 : 1184);
    return launch_pdl(tn::tp_unshard_kernel, dim3(blocks), dim3(256), tn::stream_of(stream), "tn_tp_unshard",
                      (const uint16_t *)src, (uint16_t *)dst, (int)G, (int)rows, (int)cols);
}
