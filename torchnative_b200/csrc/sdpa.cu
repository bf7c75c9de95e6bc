// sdpa.cu -- tn_sdpa_flash_attention: the C-ABI door of
// aten._scaled_dot_product_flash_attention_for_cpu (torch_c/src/aten.rs:10092-10460).
#include "tn_common.cuh"

extern "C" int tn_sdpa_flash_attention(const void *q, const void *k, const void *v, const void *attn_mask,
                                       int mask_dtype, const int64_t *mask_strides, void *out, float *lse, int dtype,
                                       int64_t B, int64_t Hq, int64_t Hkv, int64_t L, int64_t S, int64_t D,
                                       const int64_t *q_strides, const int64_t *k_strides, const int64_t *v_strides,
                                       int is_causal, double scale, void *stream) {
    (void)q, (void)k, (void)v, (void)attn_mask, (void)mask_dtype, (void)mask_strides, (void)out, (void)lse;
    (void)dtype, (void)B, (void)Hq, (void)Hkv, (void)L, (void)S, (void)D, (void)q_strides, (void)k_strides;
    (void)v_strides, (void)is_causal, (void)scale, (void)stream;
    return tn::set_error(TN_ERR_NOT_IMPLEMENTED,
                         "aten._scaled_dot_product_flash_attention_for_cpu.default: not implemented on CUDA yet");
}
