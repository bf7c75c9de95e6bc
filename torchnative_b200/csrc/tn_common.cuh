// tn_common.cuh -- shared pieces of the sm_100a kernels: status plumbing,
// mbarrier / bulk-copy PTX wrappers with bounded waits, small numeric helpers.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/torchnative_b200.h"

namespace tn {

// ---- host-side status ------------------------------------------------------

int set_error(int status, const std::string &msg);  // records msg for tn_last_error, returns status
int check_cuda(cudaError_t e, const char *op, const char *what);
int check_launch(const char *op);  // cudaGetLastError after a launch

// The stream a call runs on: the one it was given, or for NULL the current
// device's stream set by tn_stream_set (NULL: the legacy default stream).
cudaStream_t stream_of(void *stream);

struct Counters;
tn_counters &counters();

// Workspace from the caching allocator, grown on demand, one per (device, stream).
int workspace(void **ptr, size_t bytes, cudaStream_t stream, int slot);
// The same, zero-filled (stream-ordered) whenever it is (re)allocated; users
// that need zeros keep it zeroed themselves between calls.
int workspace_zeroed(void **ptr, size_t bytes, cudaStream_t stream, int slot);

// Device facts cached per device.
struct DeviceFacts {
    int sm_count;
    int cc_major, cc_minor;
    int64_t l2_bytes;
    int64_t smem_optin;
};
int device_facts(DeviceFacts *out);  // current device

// Device-side error word of the current device (set by a bounded wait that
// gave up); read by tn_device_status.
int *device_error_word();

// ---- device-side helpers -----------------------------------------------------

enum : int { DEV_ERR_NONE = 0, DEV_ERR_WAIT_FULL = 1, DEV_ERR_WAIT_EMPTY = 2, DEV_ERR_DRAIN = 3 };

// ~2^31 cycles (~1 s at 1.9 GHz) before a wait gives up: the default of the
// per-device budget (tn_set_wait_budget) that waits read next to the error
// word they were given.
constexpr long long kWaitBudgetCycles = 1ll << 31;

__device__ __forceinline__ long long wait_budget(const int *err) {
    return err ? *reinterpret_cast<const volatile long long *>(err + 2) : kWaitBudgetCycles;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: true when the phase with `parity` completed, false when the
// budget ran out (the caller records the error and stops using the pipeline).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    long long start = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - start > kWaitBudgetCycles) return false;
    }
    return true;
}

// One-dimensional bulk copy global -> shared, completing on an mbarrier.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Same with an L2 eviction hint (streamed-once data: evict_first).
__device__ __forceinline__ void bulk_g2s_hint(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Same, destination given as a 32-bit shared-window address.
__device__ __forceinline__ void bulk_g2s_hint_u32(uint32_t dst, const void *src, uint32_t bytes, uint64_t *bar,
                                                  uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            dst),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ void record_device_error(int *word, int code) {
    if (word) atomicCAS(word, 0, code);
}

// ---- tensor-parallel exchange regions (tp_comm.cu, and the GEMV epilogue
// that scatters its output rows straight into every rank's region) --------
//   [0, 4)                  epoch: steps this rank has completed
//   [64, 32768)             counters[slot][src]
//   [32768, 65536)          tickets[slot]: CTAs of this rank's producer kernel done
//   [65536, ...)            gathered activation rows; row-parallel partials as
//                           8-byte words {f32 value, tag = epoch * 256 + slot + 1}
constexpr int kTpMaxRanks = 8;
constexpr int kTpRedSlots = 256;  // reductions per step (the tag's slot field)
constexpr int64_t kTpEpochOff = 0, kTpCountOff = 64, kTpTicketOff = 32768, kTpDataOff = 65536;

__device__ __forceinline__ int ld_acquire_sys(const int *p) {
    int v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Bounded wait until counters[slot][g] >= target for every source rank g of
// this rank's region (one thread). False if it gave up (error recorded) or an
// earlier wait already had.
__device__ __forceinline__ bool tp_wait_counts(const uint8_t *local_base, int slot, int world, int target, int *err) {
    const int *cnt = reinterpret_cast<const int *>(local_base + kTpCountOff) + slot * world;
    for (int g = 0; g < world; ++g) {
        if (ld_acquire_sys(cnt + g) >= target) continue;
        if (err && *reinterpret_cast<volatile int *>(err) != 0) return false;
        const long long start = clock64(), budget = wait_budget(err);
        while (ld_acquire_sys(cnt + g) < target) {
            if (clock64() - start > budget) {
                record_device_error(err, DEV_ERR_WAIT_FULL);
                return false;
            }
        }
    }
    return true;
}

// Programmatic dependent launch: wait for the producer grid's memory, and let
// the next grid start its prologue.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

__device__ __forceinline__ void store_out(void *y, int dtype, int64_t idx, float v) {
    if (dtype == TN_F32)
        static_cast<float *>(y)[idx] = v;
    else if (dtype == TN_BF16)
        static_cast<__nv_bfloat16 *>(y)[idx] = __float2bfloat16_rn(v);
    else
        static_cast<__half *>(y)[idx] = __float2half_rn(v);
}

__device__ __forceinline__ float half_bits_to_f32(uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xffffu)));
}

}  // namespace tn

static inline size_t tn_dtype_size(int dtype) {
    switch (dtype) {
    case TN_F32: return 4;
    case TN_F16: return 2;
    case TN_BF16: return 2;
    case TN_F64: return 8;
    default: return 0;
    }
}

static inline const char *tn_dtype_name(int dtype) {
    switch (dtype) {
    case TN_F32: return "torch.float32";
    case TN_F16: return "torch.float16";
    case TN_BF16: return "torch.bfloat16";
    case TN_F64: return "torch.float64";
    default: return "an unknown dtype";
    }
}
