// tp_comm.cu -- the per-layer all-gather of tensor-parallel decode over peer
// memory (NVLink / NVSwitch), replacing a library collective for messages of
// a few KB where launch and protocol latency, not bandwidth, set the cost.
//
// Every rank owns one exchange region (cudaMalloc'd, shared with the other
// ranks through CUDA IPC handles, plain peer mappings -- no multicast):
//   [0, 4)             epoch: steps this rank has completed (tn_tp_step_end)
//   [64, 32768)        counters[slot][src]: for this kernel's gathers, CTAs of
//                      rank src that finished writing this rank's copy of
//                      gather `slot`; for gathers fused into a GEMV's epilogue
//                      (q4_gemv.cu), launches of rank src that finished
//   [32768, 65536)     tickets[slot]: the fused producer's finished CTAs
//   [65536, ...)       the gathered activation rows and the row-parallel
//                      GEMV's tagged partials (q4_gemv.cu), at caller-chosen
//                      offsets
// One gather: every rank stores its [rows][cols] slice straight into every
// rank's region (row r, columns [rank * cols, (rank + 1) * cols) of a
// [rows][dst_row_stride] buffer), fences system-wide and adds 1 to its counter
// in every region; CTA 0 then waits until all G sources have reached
// (epoch + 1) * CTAs in its own region. Each slot is used once per step and
// consecutive gathers use different buffers, so a rank that runs ahead can
// only ever write a buffer its peers have finished reading. The wait is
// bounded (~1 s); on expiry the kernel records a device error (read by
// tn_device_status) and returns.
#include <cstring>

#include "tn_common.cuh"

namespace tn {
namespace {

constexpr int64_t kEpochOff = kTpEpochOff, kCountOff = kTpCountOff, kDataOff = kTpDataOff;
constexpr int kMaxRanks = kTpMaxRanks;

struct Bases {
    uint8_t *p[kMaxRanks];
};

__global__ void __launch_bounds__(256) tp_allgather_kernel(Bases bases, int rank, int world, const uint8_t *local,
                                                           int64_t local_row_bytes, int rows, int64_t row_bytes,
                                                           int64_t dst_offset, int64_t dst_row_bytes, int slot,
                                                           int vec16, int *err) {
    pdl_launch_dependents();
    pdl_wait();
    const int tid = threadIdx.x;
    const int epoch = ld_acquire_sys(reinterpret_cast<const int *>(bases.p[rank] + kEpochOff));
    const int64_t col0 = (int64_t)rank * row_bytes;
    // push this rank's slice into every rank's region
    if (vec16) {
        const int64_t per_row = row_bytes / 16, n = (int64_t)rows * per_row;
        for (int64_t i = blockIdx.x * (int64_t)blockDim.x + tid; i < n; i += (int64_t)gridDim.x * blockDim.x) {
            const int64_t r = i / per_row, c = (i % per_row) * 16;
            const uint4 v = *reinterpret_cast<const uint4 *>(local + r * local_row_bytes + c);
            for (int g = 0; g < world; ++g)
                *reinterpret_cast<uint4 *>(bases.p[g] + kDataOff + dst_offset + r * dst_row_bytes + col0 + c) = v;
        }
    } else {
        const int64_t per_row = row_bytes / 2, n = (int64_t)rows * per_row;
        for (int64_t i = blockIdx.x * (int64_t)blockDim.x + tid; i < n; i += (int64_t)gridDim.x * blockDim.x) {
            const int64_t r = i / per_row, c = (i % per_row) * 2;
            const uint16_t v = *reinterpret_cast<const uint16_t *>(local + r * local_row_bytes + c);
            for (int g = 0; g < world; ++g)
                *reinterpret_cast<uint16_t *>(bases.p[g] + kDataOff + dst_offset + r * dst_row_bytes + col0 + c) = v;
        }
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence_system();
        for (int g = 0; g < world; ++g)
            atomicAdd_system(reinterpret_cast<int *>(bases.p[g] + kCountOff) + slot * world + rank, 1);
    }
    if (blockIdx.x != 0 || tid >= world) return;
    // CTA 0: one thread per source rank waits for that rank's CTAs
    const int target = (epoch + 1) * (int)gridDim.x;
    const int *cnt = reinterpret_cast<const int *>(bases.p[rank] + kCountOff) + slot * world + tid;
    if (ld_acquire_sys(cnt) >= target) return;
    // after one wait has given up (a rank gone), later gathers fail fast
    if (err && *reinterpret_cast<volatile int *>(err) != 0) return;
    const long long start = clock64(), budget = wait_budget(err);
    while (ld_acquire_sys(cnt) < target) {
        if (clock64() - start > budget) {
            record_device_error(err, DEV_ERR_WAIT_FULL);
            return;
        }
    }
}

__global__ void tp_step_end_kernel(int *epoch) {
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x == 0) atomicAdd(epoch, 1);
}

}  // namespace
}  // namespace tn

extern "C" {

int tn_tp_region_alloc(size_t bytes, void **base, void *ipc_handle) {
    if (!base || !ipc_handle) return tn::set_error(TN_ERR_INVALID, "tn_tp_region_alloc: null pointer");
    const size_t total = bytes + (size_t)tn::kDataOff;
    void *p = nullptr;
    int st = tn::check_cuda(cudaMalloc(&p, total), "tn_tp_region_alloc", "cudaMalloc");
    if (st) return st;
    st = tn::check_cuda(cudaMemset(p, 0, total), "tn_tp_region_alloc", "cudaMemset");
    if (st) {
        cudaFree(p);
        return st;
    }
    cudaIpcMemHandle_t h;
    st = tn::check_cuda(cudaIpcGetMemHandle(&h, p), "tn_tp_region_alloc", "cudaIpcGetMemHandle");
    if (st) {
        cudaFree(p);
        return st;
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == TN_IPC_HANDLE_BYTES, "IPC handle size");
    memcpy(ipc_handle, &h, sizeof(h));
    *base = p;
    return TN_OK;
}

int tn_tp_region_open(const void *ipc_handle, void **peer_base) {
    if (!ipc_handle || !peer_base) return tn::set_error(TN_ERR_INVALID, "tn_tp_region_open: null pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    return tn::check_cuda(cudaIpcOpenMemHandle(peer_base, h, cudaIpcMemLazyEnablePeerAccess), "tn_tp_region_open",
                          "cudaIpcOpenMemHandle");
}

int tn_tp_region_close(void *peer_base) {
    return tn::check_cuda(cudaIpcCloseMemHandle(peer_base), "tn_tp_region_close", "cudaIpcCloseMemHandle");
}

int tn_tp_region_free(void *base) { return tn::check_cuda(cudaFree(base), "tn_tp_region_free", "cudaFree"); }

int64_t tn_tp_region_data_offset(void) { return tn::kDataOff; }

int tn_tp_allgather(void *const *bases, int rank, int world, const void *local, int64_t local_row_stride,
                    int64_t rows, int64_t cols, int64_t dst_offset, int64_t dst_row_stride, int slot, void *stream) {
    const char *op = "tn_tp_allgather";
    if (world < 1 || world > tn::kMaxRanks || rank < 0 || rank >= world)
        return tn::set_error(TN_ERR_INVALID, std::string(op) + ": rank/world out of range (at most 8 ranks)");
    if (rows < 0 || cols < 0 || local_row_stride < cols || dst_row_stride < world * cols || slot < 0 ||
        (int64_t)(slot + 1) * world * 4 > tn::kTpTicketOff - tn::kCountOff)
        return tn::set_error(TN_ERR_SHAPE, std::string(op) + ": bad shape, stride or slot");
    if (!bases || !local) return tn::set_error(TN_ERR_INVALID, std::string(op) + ": null pointer");
    tn::Bases b{};
    for (int g = 0; g < world; ++g) {
        if (!bases[g]) return tn::set_error(TN_ERR_INVALID, std::string(op) + ": null region base");
        b.p[g] = static_cast<uint8_t *>(bases[g]);
    }
    const int64_t row_bytes = cols * 2, n = rows * cols * 2;
    const uintptr_t al = reinterpret_cast<uintptr_t>(local) | (uintptr_t)(local_row_stride * 2) |
                         (uintptr_t)(dst_offset) | (uintptr_t)(dst_row_stride * 2) | (uintptr_t)row_bytes |
                         (uintptr_t)(rank * row_bytes);
    const int vec16 = (al & 15) == 0;
    int ctas = (int)((n + 8191) / 8192);
    ctas = ctas < 1 ? 1 : (ctas > 64 ? 64 : ctas);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ctas);
    cfg.blockDim = dim3(256);
    cfg.stream = tn::stream_of(stream);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return tn::check_cuda(cudaLaunchKernelEx(&cfg, tn::tp_allgather_kernel, b, rank, world,
                                             static_cast<const uint8_t *>(local), local_row_stride * 2, (int)rows,
                                             row_bytes, dst_offset, dst_row_stride * 2, slot, vec16,
                                             tn::device_error_word()),
                          op, "cudaLaunchKernelEx");
}

int tn_tp_step_end(void *local_base, void *stream) {
    if (!local_base) return tn::set_error(TN_ERR_INVALID, "tn_tp_step_end: null region base");
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(1);
    cfg.stream = tn::stream_of(stream);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return tn::check_cuda(cudaLaunchKernelEx(&cfg, tn::tp_step_end_kernel,
                                             reinterpret_cast<int *>(static_cast<uint8_t *>(local_base) +
                                                                     tn::kEpochOff)),
                          "tn_tp_step_end", "cudaLaunchKernelEx");
}

}  // extern "C"
