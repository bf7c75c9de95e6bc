// sdpa_common.cuh -- shared definitions of the attention kernels.
#pragma once

#include "tn_common.cuh"

namespace tn {

// One attention call, as the kernels see it. Element strides in [b, h, t, d]
// order; the d stride is 1 for q, k, v.
struct SdpaParams {
    const void *q, *k, *v, *mask;
    void *out;
    float *lse;
    int64_t qs[4], ks[4], vs[4], ms[4];
    int B, Hq, Hkv, L, S, D;
    int rep;        // Hq / Hkv
    int mask_dtype; // TN_F32 or the input dtype
    int causal;
    float scale;
    // split-KV decode
    int rows;       // query rows per CTA (rep * L or a slice of it)
    int row_groups; // ceil(rep * L / rows)
    int splits;     // key splits per (b, kv head, row group)
    int keys_per_split;
    float *part_o;  // [B*Hq*L][splits][D] f32 unnormalised partial outputs
    float *part_ml; // [B*Hq*L][splits][2]  running max and sum
    const int *S_dev; // if set: the key count is min(*S_dev + S_add, S) (S is then the cache capacity)
    int S_add;
    // Fused decode step (bf16, L = 1, one row group): q and the new k, v come
    // from the q/k/v projection rows [B][(Hq + 2 Hkv) D]; q and k get the
    // rotary embedding at position S - 1 (inv_freq [D/2] f32) and k, v are
    // written to cache slot S - 1 before any key tile is read.
    const __nv_bfloat16 *qkv;
    const float *inv_freq;
    // If set, the last CTA of each (b, kv head) merges the splits itself
    // (counters start at zero and are left at zero).
    int *counters;
    // If set (decode step, L = 1): the merge also writes out as planar Q8_0
    // (codes [B][Hq D] int8, scales / offsets [B][Hq D / 32] f32), the bytes
    // tn_q8_0_quantize_planar writes for the bf16 output.
    int8_t *q8_codes;
    float *q8_scales, *q8_offs;
    int *err;
};

int launch_sdpa_decode(const SdpaParams &p, int dtype, cudaStream_t stream);
// Prefill on tcgen05 tensor cores: bf16/f16, D = 128, no additive mask, TMA-
// compatible q/k/v (16-byte aligned base and strides).
int launch_sdpa_prefill(const SdpaParams &p, int dtype, cudaStream_t stream);
// The same with two query tiles (256 rows) per CTA, for longer sequences.
int launch_sdpa_prefill2(const SdpaParams &p, int dtype, cudaStream_t stream);
// Prefill on the FP32 pipes: every dtype, D = 64 or 128, masks, any q strides;
// grid (ceil(L / 64), Hq, B).
int launch_sdpa_prefill_simt(const SdpaParams &p, int dtype, cudaStream_t stream);
size_t sdpa_decode_workspace(const SdpaParams &p);
int plan_sdpa_decode(SdpaParams &p, int sm_count, int dtype);

}  // namespace tn
