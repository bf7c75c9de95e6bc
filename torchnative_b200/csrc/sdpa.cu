// sdpa.cu -- tn_sdpa_flash_attention: the C-ABI door of
// aten._scaled_dot_product_flash_attention_for_cpu (torch_c/src/aten.rs:10092-10460)
// on a B200. Argument checks follow the reference's order and wording
// (aten.rs:10113-10172, 10226-10261, 17112-17122).
#include <cmath>

#include "sdpa_common.cuh"

namespace {

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" int tn_sdpa_flash_attention(const void *q, const void *k, const void *v, const void *attn_mask,
                                       int mask_dtype, const int64_t *mask_strides, void *out, float *lse, int dtype,
                                       int64_t B, int64_t Hq, int64_t Hkv, int64_t L, int64_t S, int64_t D,
                                       const int64_t *q_strides, const int64_t *k_strides, const int64_t *v_strides,
                                       int is_causal, double scale, void *stream_) {
    const std::string op = "aten._scaled_dot_product_flash_attention_for_cpu.default";
    cudaStream_t stream = tn::stream_of(stream_);
    __atomic_fetch_add(&tn::counters().sdpa_calls, 1ull, __ATOMIC_RELAXED);
    if (dtype == TN_F64)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": torch.float64 attention is not implemented on CUDA");
    if (dtype != TN_F32 && dtype != TN_BF16 && dtype != TN_F16)
        return tn::set_error(TN_ERR_SHAPE, "scaled_dot_product_attention_flash_attention: Expected data type in FP32, "
                                           "FP64, BF16, FP16, but got " +
                                               std::string(tn_dtype_name(dtype)) + " instead.");
    if (B < 0 || Hq < 0 || Hkv < 0 || L < 0 || S < 0 || D < 0)
        return tn::set_error(TN_ERR_SHAPE, op + ": negative size");
    if (D == 0 || S == 0)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED,
                             op + ": a zero key length or head dimension is not implemented in torch._C shim");
    if (B == 0 || Hq == 0 || L == 0) return TN_OK;
    if (Hkv == 0 || Hq % Hkv != 0)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED,
                             op + ": grouped-query attention with " + std::to_string(Hq) + " query heads and " +
                                 std::to_string(Hkv) +
                                 " key/value heads is not implemented in torch._C shim -- the head counts do not divide");
    if (D != 64 && D != 128)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED,
                             op + ": head dimension " + std::to_string(D) + " is not implemented on CUDA (64, 128)");
    if (attn_mask && mask_dtype != TN_F32 && mask_dtype != dtype)
        return tn::set_error(TN_ERR_SHAPE, "scaled_dot_product_attention_flash_attention: Attention mask is the same "
                                           "data type as query");
    if (!q || !k || !v || !out || !q_strides || !k_strides || !v_strides || (attn_mask && !mask_strides))
        return tn::set_error(TN_ERR_INVALID, op + ": null pointer");
    if (q_strides[3] != 1 || k_strides[3] != 1 || v_strides[3] != 1)
        return tn::set_error(TN_ERR_INVALID, op + ": the head dimension must have unit stride");
    const size_t es = tn_dtype_size(dtype);
    for (int i = 0; i < 3; ++i)
        if ((k_strides[i] * (int64_t)es) % 16 != 0 || (v_strides[i] * (int64_t)es) % 16 != 0)
            return tn::set_error(TN_ERR_INVALID, op + ": key/value strides must be multiples of 16 bytes");
    if (!aligned16(k) || !aligned16(v))
        return tn::set_error(TN_ERR_INVALID, op + ": key/value must be 16-byte aligned");
    if (B > 65535 || Hq > 65535 || S > (int64_t)1 << 30 || L > (int64_t)1 << 30)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": size beyond the kernel's grid limits");

    tn::DeviceFacts f{};
    int st = tn::device_facts(&f);
    if (st) return st;
    tn::SdpaParams p{};
    p.q = q;
    p.k = k;
    p.v = v;
    p.mask = attn_mask;
    p.out = out;
    p.lse = lse;
    for (int i = 0; i < 4; ++i) {
        p.qs[i] = q_strides[i];
        p.ks[i] = k_strides[i];
        p.vs[i] = v_strides[i];
        p.ms[i] = attn_mask ? mask_strides[i] : 0;
    }
    p.B = (int)B;
    p.Hq = (int)Hq;
    p.Hkv = (int)Hkv;
    p.L = (int)L;
    p.S = (int)S;
    p.D = (int)D;
    p.rep = (int)(Hq / Hkv);
    p.mask_dtype = mask_dtype;
    p.causal = is_causal ? 1 : 0;
    // Default 1/sqrt(D) in f64, then f32 (candle's affine casts its f64 multiplier).
    const double sc = (std::isnan(scale) || scale <= 0.0) ? 1.0 / std::sqrt((double)D) : scale;
    p.scale = (float)sc;
    p.err = tn::device_error_word();

    // Many query rows (prefill): the tcgen05 flash kernel, where it applies.
    const bool tma_ok = aligned16(q) && (q_strides[0] * 2) % 16 == 0 && (q_strides[1] * 2) % 16 == 0 &&
                        (q_strides[2] * 2) % 16 == 0;
    if (dtype != TN_F32 && D == 128 && !attn_mask && p.rep * L > 16 && tma_ok && aligned16(out))
        return L > 128 ? tn::launch_sdpa_prefill2(p, dtype, stream) : tn::launch_sdpa_prefill(p, dtype, stream);
    // Other calls with many query rows per head: the FP32-pipe flash kernel
    // (one pass over K/V per 64 query rows, where the split-KV kernel would
    // re-read K/V for every 8 rows).
    if (L > 16) return tn::launch_sdpa_prefill_simt(p, dtype, stream);
    st = tn::plan_sdpa_decode(p, f.sm_count, dtype);
    if (st) return st;
    void *ws = nullptr;
    st = tn::workspace(&ws, tn::sdpa_decode_workspace(p), stream, /*slot=*/1);
    if (st) return st;
    const int64_t rows = (int64_t)p.B * p.Hq * p.L;
    p.part_o = static_cast<float *>(ws);
    p.part_ml = p.part_o + rows * p.splits * p.D;
    if (p.L == 1 && p.row_groups == 1 && (int64_t)p.B * p.Hkv <= 32) {
        // one query row per head and few heads: the last CTA of each KV head
        // merges the splits (a zeroed ticket per head, reset by that CTA), no
        // combine launch. (With many (batch, head) pairs the separate combine
        // kernel spreads the merges wider and measures faster.)
        void *cnt = nullptr;
        st = tn::workspace_zeroed(&cnt, (size_t)p.B * p.Hkv * sizeof(int) + 256, stream, /*slot=*/3);
        if (st) return st;
        p.counters = static_cast<int *>(cnt);
    }
    return tn::launch_sdpa_decode(p, dtype, stream);
}

extern "C" int tn_sdpa_decode_cache(const void *q, const void *k_cache, const void *v_cache, void *out, float *lse,
                                    int dtype, int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t capacity,
                                    const int64_t *q_strides, const int64_t *k_strides, const int64_t *v_strides,
                                    const int *len_dev, int64_t len_add, double scale, void *stream_) {
    const std::string op = "tn_sdpa_decode_cache";
    cudaStream_t stream = tn::stream_of(stream_);
    __atomic_fetch_add(&tn::counters().sdpa_calls, 1ull, __ATOMIC_RELAXED);
    if (dtype != TN_F32 && dtype != TN_BF16 && dtype != TN_F16)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": dtype must be float32, bfloat16 or float16");
    if (D != 64 && D != 128)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": head dimension must be 64 or 128");
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0 || capacity <= 0 || !len_dev)
        return tn::set_error(TN_ERR_SHAPE, op + ": bad shape");
    if (q_strides[3] != 1 || k_strides[3] != 1 || v_strides[3] != 1 || !aligned16(k_cache) || !aligned16(v_cache))
        return tn::set_error(TN_ERR_INVALID, op + ": unit head-dim stride and 16-byte aligned caches required");
    tn::DeviceFacts f{};
    int st = tn::device_facts(&f);
    if (st) return st;
    tn::SdpaParams p{};
    p.q = q;
    p.k = k_cache;
    p.v = v_cache;
    p.out = out;
    p.lse = lse;
    for (int i = 0; i < 4; ++i) {
        p.qs[i] = q_strides[i];
        p.ks[i] = k_strides[i];
        p.vs[i] = v_strides[i];
    }
    p.B = (int)B;
    p.Hq = (int)Hq;
    p.Hkv = (int)Hkv;
    p.L = 1;
    p.S = (int)capacity;
    p.D = (int)D;
    p.rep = (int)(Hq / Hkv);
    p.mask_dtype = dtype;
    p.scale = (float)((std::isnan(scale) || scale <= 0.0) ? 1.0 / std::sqrt((double)D) : scale);
    p.S_dev = len_dev;
    p.S_add = (int)len_add;
    p.err = tn::device_error_word();
    st = tn::plan_sdpa_decode(p, f.sm_count, dtype);
    if (st) return st;
    void *ws = nullptr;
    st = tn::workspace(&ws, tn::sdpa_decode_workspace(p), stream, /*slot=*/2);
    if (st) return st;
    p.part_o = static_cast<float *>(ws);
    p.part_ml = p.part_o + (int64_t)p.B * p.Hq * p.splits * p.D;
    if (p.row_groups == 1 && (int64_t)p.B * p.Hkv <= 32) {  // in-kernel merge, as the flash op does
        void *cnt = nullptr;
        st = tn::workspace_zeroed(&cnt, (size_t)p.B * p.Hkv * sizeof(int) + 256, stream, /*slot=*/3);
        if (st) return st;
        p.counters = static_cast<int *>(cnt);
    }
    return tn::launch_sdpa_decode(p, dtype, stream);
}

extern "C" int tn_sdpa_decode_step(const void *qkv, const float *inv_freq, void *k_cache, void *v_cache, void *out,
                                   float *lse, int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t capacity,
                                   const int64_t *k_strides, const int64_t *v_strides, const int *pos_dev,
                                   double scale, void *stream_) {
    return tn_sdpa_decode_step_q8(qkv, inv_freq, k_cache, v_cache, out, lse, nullptr, nullptr, nullptr, B, Hq, Hkv,
                                  D, capacity, k_strides, v_strides, pos_dev, scale, stream_);
}

extern "C" int tn_sdpa_decode_step_q8(const void *qkv, const float *inv_freq, void *k_cache, void *v_cache,
                                      void *out, float *lse, int8_t *codes, float *scales, float *offsets,
                                      int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t capacity,
                                      const int64_t *k_strides, const int64_t *v_strides, const int *pos_dev,
                                      double scale, void *stream_) {
    const std::string op = "tn_sdpa_decode_step";
    if ((codes || scales || offsets) &&
        (!codes || !scales || !offsets || (reinterpret_cast<uintptr_t>(codes) & 3) != 0))
        return tn::set_error(TN_ERR_INVALID, op + ": planar Q8_0 output needs codes (4-byte aligned), scales and "
                                                  "offsets");
    cudaStream_t stream = tn::stream_of(stream_);
    __atomic_fetch_add(&tn::counters().sdpa_calls, 1ull, __ATOMIC_RELAXED);
    if (D != 64 && D != 128)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": head dimension must be 64 or 128");
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0 || Hq / Hkv > 8 || capacity <= 0 || B > 65535)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": needs Hq % Hkv == 0 and at most 8 query heads per KV head");
    if (!qkv || !inv_freq || !k_cache || !v_cache || !out || !pos_dev || !k_strides || !v_strides)
        return tn::set_error(TN_ERR_INVALID, op + ": null pointer");
    if (k_strides[3] != 1 || v_strides[3] != 1 || !aligned16(k_cache) || !aligned16(v_cache))
        return tn::set_error(TN_ERR_INVALID, op + ": unit head-dim stride and 16-byte aligned caches required");
    for (int i = 0; i < 3; ++i)
        if ((k_strides[i] * 2) % 16 != 0 || (v_strides[i] * 2) % 16 != 0)
            return tn::set_error(TN_ERR_INVALID, op + ": cache strides must be multiples of 16 bytes");
    tn::DeviceFacts f{};
    int st = tn::device_facts(&f);
    if (st) return st;
    tn::SdpaParams p{};
    p.k = k_cache;
    p.v = v_cache;
    p.out = out;
    p.lse = lse;
    for (int i = 0; i < 4; ++i) {
        p.ks[i] = k_strides[i];
        p.vs[i] = v_strides[i];
    }
    p.B = (int)B;
    p.Hq = (int)Hq;
    p.Hkv = (int)Hkv;
    p.L = 1;
    p.S = (int)capacity;
    p.D = (int)D;
    p.rep = (int)(Hq / Hkv);
    p.mask_dtype = TN_BF16;
    p.scale = (float)((std::isnan(scale) || scale <= 0.0) ? 1.0 / std::sqrt((double)D) : scale);
    p.S_dev = pos_dev;
    p.S_add = 1;
    p.qkv = static_cast<const __nv_bfloat16 *>(qkv);
    p.inv_freq = inv_freq;
    p.err = tn::device_error_word();
    st = tn::plan_sdpa_decode(p, f.sm_count, TN_BF16);
    if (st) return st;
    if (p.row_groups != 1) return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": internal: more than one row group");
    void *ws = nullptr;
    st = tn::workspace(&ws, tn::sdpa_decode_workspace(p), stream, /*slot=*/2);
    if (st) return st;
    p.part_o = static_cast<float *>(ws);
    p.part_ml = p.part_o + (int64_t)p.B * p.Hq * p.splits * p.D;
    void *cnt = nullptr;
    st = tn::workspace_zeroed(&cnt, (size_t)p.B * p.Hkv * sizeof(int) + 256, stream, /*slot=*/3);
    if (st) return st;
    p.counters = static_cast<int *>(cnt);
    p.q8_codes = codes;
    p.q8_scales = scales;
    p.q8_offs = offsets;
    return tn::launch_sdpa_decode(p, TN_BF16, stream);
}
