// tn_runtime.cu -- status/error plumbing, device facts, counters, the caching
// device allocator and per-stream workspaces behind the C ABI.
#include <atomic>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "tn_common.cuh"

namespace {

thread_local std::string g_last_error;

tn_counters g_counters{};

constexpr int kMaxDevices = 64;

struct FactsSlot {
    bool valid = false;
    tn::DeviceFacts facts{};
};
FactsSlot g_facts[kMaxDevices];
std::mutex g_facts_mu;

// Device-side words of each GPU: the error code set by kernels whose bounded
// waits gave up, and the wait budget (clock cycles) those waits allow. Kernels
// reach both through the `int *err` they are given (budget at err + 2).
struct DeviceWords {
    int err;
    int pad;
    long long wait_budget;
};
__device__ DeviceWords g_device_error = {0, 0, tn::kWaitBudgetCycles};
int *g_error_word[kMaxDevices] = {nullptr};

// The stream each device's calls run on when they are given none (the
// reference keeps one candle CudaStream per device); NULL = the legacy stream.
cudaStream_t g_current_stream[kMaxDevices] = {nullptr};

// ---- caching allocator -------------------------------------------------------

struct Block {
    void *ptr;
    size_t size;
    int device;
    cudaStream_t stream;
};

std::mutex g_alloc_mu;
std::multimap<std::tuple<int, cudaStream_t, size_t>, void *> g_free;  // (device, stream, size) -> ptr
std::map<void *, Block> g_live;
std::map<void *, Block> g_cached;
size_t g_allocated = 0, g_reserved = 0;

size_t round_size(size_t bytes) {
    if (bytes == 0) bytes = 1;
    if (bytes <= (1u << 20)) return (bytes + 511) & ~size_t(511);
    return (bytes + (2u << 20) - 1) & ~size_t((2u << 20) - 1);
}

// ---- workspaces ---------------------------------------------------------------

struct Workspace {
    void *ptr = nullptr;
    size_t size = 0;
};
std::mutex g_ws_mu;
std::map<std::tuple<int, cudaStream_t, int>, Workspace> g_ws;

}  // namespace

namespace tn {

int set_error(int status, const std::string &msg) {
    g_last_error = msg;
    if (status == TN_ERR_NOT_IMPLEMENTED) __atomic_fetch_add(&g_counters.refusals, 1ull, __ATOMIC_RELAXED);
    return status;
}

cudaStream_t stream_of(void *stream) {
    if (stream) return static_cast<cudaStream_t>(stream);
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    return g_current_stream[dev];
}

int check_cuda(cudaError_t e, const char *op, const char *what) {
    if (e == cudaSuccess) return TN_OK;
    int status = (e == cudaErrorMemoryAllocation) ? TN_ERR_OOM : TN_ERR_CUDA;
    return set_error(status, std::string(op) + ": " + what + " failed: " + cudaGetErrorName(e) + " (" +
                                 cudaGetErrorString(e) + ")");
}

int check_launch(const char *op) { return check_cuda(cudaGetLastError(), op, "kernel launch"); }

tn_counters &counters() { return g_counters; }

int device_facts(DeviceFacts *out) {
    int dev = 0;
    int st = check_cuda(cudaGetDevice(&dev), "tn_device_info", "cudaGetDevice");
    if (st) return st;
    if (dev < 0 || dev >= kMaxDevices) return set_error(TN_ERR_INVALID, "tn_device_info: device index out of range");
    std::lock_guard<std::mutex> lk(g_facts_mu);
    if (!g_facts[dev].valid) {
        DeviceFacts f{};
        cudaDeviceProp p;
        st = check_cuda(cudaGetDeviceProperties(&p, dev), "tn_device_info", "cudaGetDeviceProperties");
        if (st) return st;
        __atomic_fetch_add(&g_counters.resolves, 1ull, __ATOMIC_RELAXED);
        f.sm_count = p.multiProcessorCount;
        f.cc_major = p.major;
        f.cc_minor = p.minor;
        f.l2_bytes = p.l2CacheSize;
        f.smem_optin = (int64_t)p.sharedMemPerBlockOptin;
        g_facts[dev].facts = f;
        g_facts[dev].valid = true;
    }
    *out = g_facts[dev].facts;
    return TN_OK;
}

int *device_error_word() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    if (!g_error_word[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
        g_error_word[dev] = static_cast<int *>(p);
    }
    return g_error_word[dev];
}

int workspace_zeroed(void **ptr, size_t bytes, cudaStream_t stream, int slot) {
    int dev = 0;
    int st = check_cuda(cudaGetDevice(&dev), "workspace", "cudaGetDevice");
    if (st) return st;
    bool grew = false;
    {
        std::lock_guard<std::mutex> lk(g_ws_mu);
        Workspace &w = g_ws[std::make_tuple(dev, stream, slot)];
        grew = w.size < bytes;
    }
    st = workspace(ptr, bytes, stream, slot);
    if (st) return st;
    if (grew) return check_cuda(cudaMemsetAsync(*ptr, 0, bytes, stream), "workspace", "cudaMemsetAsync");
    return TN_OK;
}

int workspace(void **ptr, size_t bytes, cudaStream_t stream, int slot) {
    int dev = 0;
    int st = check_cuda(cudaGetDevice(&dev), "workspace", "cudaGetDevice");
    if (st) return st;
    std::lock_guard<std::mutex> lk(g_ws_mu);
    Workspace &w = g_ws[std::make_tuple(dev, stream, slot)];
    if (w.size < bytes) {
        if (w.ptr) {
            // Work queued on this stream may still read the old block.
            st = check_cuda(cudaStreamSynchronize(stream), "workspace", "cudaStreamSynchronize");
            if (st) return st;
            tn_free(w.ptr, stream);
            w.ptr = nullptr;
            w.size = 0;
        }
        size_t want = round_size(bytes);
        st = tn_alloc(&w.ptr, want, stream);
        if (st) return st;
        w.size = want;
    }
    *ptr = w.ptr;
    return TN_OK;
}

}  // namespace tn

extern "C" {

int tn_abi_version(void) { return TN_ABI_VERSION; }

const char *tn_last_error(void) { return g_last_error.c_str(); }

const char *tn_status_name(int status) {
    switch (status) {
    case TN_OK: return "TN_OK";
    case TN_ERR_NOT_IMPLEMENTED: return "TN_ERR_NOT_IMPLEMENTED";
    case TN_ERR_SHAPE: return "TN_ERR_SHAPE";
    case TN_ERR_INVALID: return "TN_ERR_INVALID";
    case TN_ERR_CUDA: return "TN_ERR_CUDA";
    case TN_ERR_OOM: return "TN_ERR_OOM";
    case TN_ERR_TIMEOUT: return "TN_ERR_TIMEOUT";
    default: return "TN_ERR_UNKNOWN";
    }
}

int tn_device_info(int device, int *sm_count, int *cc_major, int *cc_minor, int64_t *l2_bytes,
                   int64_t *smem_optin_per_block) {
    int prev = 0;
    int st = tn::check_cuda(cudaGetDevice(&prev), "tn_device_info", "cudaGetDevice");
    if (st) return st;
    if (device >= 0 && device != prev) {
        st = tn::check_cuda(cudaSetDevice(device), "tn_device_info", "cudaSetDevice");
        if (st) return st;
    }
    tn::DeviceFacts f{};
    st = tn::device_facts(&f);
    if (device >= 0 && device != prev) cudaSetDevice(prev);
    if (st) return st;
    if (sm_count) *sm_count = f.sm_count;
    if (cc_major) *cc_major = f.cc_major;
    if (cc_minor) *cc_minor = f.cc_minor;
    if (l2_bytes) *l2_bytes = f.l2_bytes;
    if (smem_optin_per_block) *smem_optin_per_block = f.smem_optin;
    if (f.cc_major != 10 || f.cc_minor != 0)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED,
                             "torchnative_b200: this library is built for sm_100a (B200); the device is sm_" +
                                 std::to_string(f.cc_major) + std::to_string(f.cc_minor));
    return TN_OK;
}

int tn_device_status(int reset) {
    int *w = tn::device_error_word();
    if (!w) return tn::set_error(TN_ERR_CUDA, "tn_device_status: no device error word");
    int st = tn::check_cuda(cudaDeviceSynchronize(), "tn_device_status", "cudaDeviceSynchronize");
    if (st) return st;
    int v = 0;
    st = tn::check_cuda(cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost), "tn_device_status", "read");
    if (st) return st;
    if (reset && v) {
        int zero = 0;
        cudaMemcpy(w, &zero, sizeof(int), cudaMemcpyHostToDevice);
    }
    if (v)
        return tn::set_error(TN_ERR_TIMEOUT, "torchnative_b200: a kernel's bounded wait gave up (device code " +
                                                 std::to_string(v) + ")");
    return TN_OK;
}

int tn_set_wait_budget(int64_t cycles, int64_t *previous) {
    int *w = tn::device_error_word();
    if (!w) return tn::set_error(TN_ERR_CUDA, "tn_set_wait_budget: no device words");
    long long *b = reinterpret_cast<long long *>(w + 2);
    long long old = 0;
    int st = tn::check_cuda(cudaMemcpy(&old, b, sizeof(old), cudaMemcpyDeviceToHost), "tn_set_wait_budget", "read");
    if (st) return st;
    if (previous) *previous = old;
    if (cycles <= 0) cycles = tn::kWaitBudgetCycles;
    long long v = cycles;
    return tn::check_cuda(cudaMemcpy(b, &v, sizeof(v), cudaMemcpyHostToDevice), "tn_set_wait_budget", "write");
}

int tn_stream_set(int device, void *stream) {
    if (device < 0 || device >= kMaxDevices) return tn::set_error(TN_ERR_INVALID, "tn_stream_set: bad device index");
    g_current_stream[device] = static_cast<cudaStream_t>(stream);
    return TN_OK;
}

int tn_stream_get(int device, void **stream) {
    if (device < 0 || device >= kMaxDevices || !stream)
        return tn::set_error(TN_ERR_INVALID, "tn_stream_get: bad device index or null out-pointer");
    *stream = g_current_stream[device];
    return TN_OK;
}

int tn_alloc(void **ptr, size_t bytes, void *stream_) {
    if (!ptr) return tn::set_error(TN_ERR_INVALID, "tn_alloc: null out-pointer");
    cudaStream_t stream = tn::stream_of(stream_);
    int dev = 0;
    int st = tn::check_cuda(cudaGetDevice(&dev), "tn_alloc", "cudaGetDevice");
    if (st) return st;
    size_t size = round_size(bytes);
    std::lock_guard<std::mutex> lk(g_alloc_mu);
    auto it = g_free.find(std::make_tuple(dev, stream, size));
    if (it != g_free.end()) {
        void *p = it->second;
        g_free.erase(it);
        Block b = g_cached[p];
        g_cached.erase(p);
        g_live[p] = b;
        g_allocated += size;
        *ptr = p;
        return TN_OK;
    }
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, size);
    if (e == cudaErrorMemoryAllocation && !g_cached.empty()) {
        cudaGetLastError();
        cudaDeviceSynchronize();
        for (auto &kv : g_cached) cudaFree(kv.first), g_reserved -= kv.second.size;
        g_cached.clear();
        g_free.clear();
        e = cudaMalloc(&p, size);
    }
    st = tn::check_cuda(e, "tn_alloc", "cudaMalloc");
    if (st) return st;
    g_live[p] = Block{p, size, dev, stream};
    g_allocated += size;
    g_reserved += size;
    __atomic_fetch_add(&g_counters.bytes_allocated, (uint64_t)size, __ATOMIC_RELAXED);
    *ptr = p;
    return TN_OK;
}

int tn_free(void *ptr, void *stream_) {
    (void)stream_;
    if (!ptr) return TN_OK;
    std::lock_guard<std::mutex> lk(g_alloc_mu);
    auto it = g_live.find(ptr);
    if (it == g_live.end()) return tn::set_error(TN_ERR_INVALID, "tn_free: pointer was not allocated by tn_alloc");
    Block b = it->second;
    g_live.erase(it);
    g_allocated -= b.size;
    g_cached[ptr] = b;
    g_free.emplace(std::make_tuple(b.device, b.stream, b.size), ptr);
    return TN_OK;
}

int tn_empty_cache(void) {
    std::lock_guard<std::mutex> lk(g_alloc_mu);
    if (g_cached.empty()) return TN_OK;
    int st = tn::check_cuda(cudaDeviceSynchronize(), "tn_empty_cache", "cudaDeviceSynchronize");
    if (st) return st;
    for (auto &kv : g_cached) {
        cudaFree(kv.first);
        g_reserved -= kv.second.size;
    }
    g_cached.clear();
    g_free.clear();
    return TN_OK;
}

int tn_memory_stats(size_t *allocated_bytes, size_t *reserved_bytes) {
    std::lock_guard<std::mutex> lk(g_alloc_mu);
    if (allocated_bytes) *allocated_bytes = g_allocated;
    if (reserved_bytes) *reserved_bytes = g_reserved;
    return TN_OK;
}

int tn_get_counters(tn_counters *out) {
    if (!out) return tn::set_error(TN_ERR_INVALID, "tn_get_counters: null out-pointer");
    *out = g_counters;
    return TN_OK;
}

int tn_reset_counters(void) {
    g_counters = tn_counters{};
    return TN_OK;
}

}  // extern "C"

// ---- tensor maps -------------------------------------------------------------

#include "tc05.cuh"

namespace tn {

namespace {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder(int *status) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    if (!encode) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q{};
        cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) {
            *status = set_error(TN_ERR_CUDA, "tensor map: cuTensorMapEncodeTiled is not available from the driver");
            return nullptr;
        }
        encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    return encode;
}

}  // namespace

int encode_map_4d_b16(CUtensorMap *map, const void *base, const uint64_t dims[4], const uint64_t strides_bytes[3],
                      uint32_t box_rows) {
    int st = TN_OK;
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder(&st);
    if (!encode) return st;
    cuuint64_t gdim[4] = {dims[0], dims[1], dims[2], dims[3]};
    cuuint64_t gstride[3] = {strides_bytes[0], strides_bytes[1], strides_bytes[2]};
    cuuint32_t box[4] = {64, box_rows, 1, 1};
    cuuint32_t estride[4] = {1, 1, 1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void *>(base), gdim, gstride, box, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(TN_ERR_INVALID, "tensor map: cuTensorMapEncodeTiled failed with CUresult " + std::to_string((int)r));
    return TN_OK;
}

int encode_map_2d(CUtensorMap *map, const void *base, int elem_bytes, uint64_t inner, uint64_t outer,
                  uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, bool swizzle128) {
    int st = TN_OK;
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder(&st);
    if (!encode) return st;
    const CUtensorMapDataType dt = elem_bytes == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                   : elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16
                                                     : CU_TENSOR_MAP_DATA_TYPE_UINT32;
    cuuint64_t gdim[2] = {inner, outer};
    cuuint64_t gstride[1] = {row_stride_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estride[2] = {1, 1};
    CUresult r = encode(map, dt, 2, const_cast<void *>(base), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(TN_ERR_INVALID, "tensor map: cuTensorMapEncodeTiled (2-D) failed with CUresult " +
                                             std::to_string((int)r));
    return TN_OK;
}

}  // namespace tn
