// q4_noalloc.cu -- tn_q4_0_linear_noalloc: the Q4_0 linear with its scratch in
// a fixed device array instead of the caching allocator.
//
// Who needs it: a host that must not let a library allocate device memory on
// its hot path -- an engine that plans every byte of HBM up front and hands
// out slices of its own arena, code that records work into a CUDA graph under
// the global capture mode (where cudaMalloc is an error), or a latency-bound
// loop that cannot afford cudaMalloc's implicit synchronisation. Such a caller
// passes inputs and outputs it owns; the activation blocks this linear needs in
// between live in `g_q8_scratch` below.
//
// The array is a file-scope __device__ variable, so every GPU that loads this
// library holds its kNoallocScratchBytes (320 KB) until the process exits. Host
// code cannot use the symbol as an address: on the host `g_q8_scratch` names a
// shadow object, not device memory. The device address is looked up once per
// device with cudaGetSymbolAddress, with that device current, on the first call
// made on that device; make that first call before any stream capture begins.
// The cached address belongs to the CUDA context that was current at that first
// call: after cudaDeviceReset, or when another context is made current on the
// same device, the cache is stale, so those hosts must not use this entry
// point across such a change.
//
// Every call shares the one array and leaves its contents behind. Nothing in it
// has to start at zero: each call's quantiser writes every code, scale and
// offset the following GEMV reads. Two calls whose work overlaps on the GPU
// (different streams, no ordering between them) race on the array.
#include <mutex>

#include "q4_kernels.cuh"

namespace {

constexpr int64_t kRowsMax = TN_NOALLOC_MAX_ROWS;  // activation rows per call
constexpr int64_t kInMax = TN_NOALLOC_MAX_IN;      // in_features per call
constexpr size_t kCodesBytes = (size_t)kRowsMax * kInMax;
constexpr size_t kScaleBytes = (size_t)kRowsMax * (kInMax / 32) * 4;
constexpr size_t kNoallocScratchBytes = kCodesBytes + 2 * kScaleBytes;

static __device__ __align__(256) uint8_t g_q8_scratch[kNoallocScratchBytes];

constexpr int kMaxDevices = 64;
uint8_t *g_scratch_addr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mu;

// Device address of g_q8_scratch on the current device (looked up once).
int scratch_address(uint8_t **out) {
    int dev = 0;
    int st = tn::check_cuda(cudaGetDevice(&dev), "tn_q4_0_linear_noalloc", "cudaGetDevice");
    if (st) return st;
    if (dev < 0 || dev >= kMaxDevices)
        return tn::set_error(TN_ERR_INVALID, "tn_q4_0_linear_noalloc: device index out of range");
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!g_scratch_addr[dev]) {
        void *p = nullptr;
        st = tn::check_cuda(cudaGetSymbolAddress(&p, g_q8_scratch), "tn_q4_0_linear_noalloc",
                            "cudaGetSymbolAddress(g_q8_scratch)");
        if (st) return st;
        g_scratch_addr[dev] = static_cast<uint8_t *>(p);
    }
    *out = g_scratch_addr[dev];
    return TN_OK;
}

}  // namespace

extern "C" int tn_q4_0_linear_noalloc(const void *x, int x_dtype, int64_t x_row_stride, const void *w_blob,
                                      const float *bias, void *y, int y_dtype, int64_t M, int64_t N, int64_t K,
                                      void *stream_) {
    const std::string op = "tn_q4_0_linear_noalloc";
    cudaStream_t stream = tn::stream_of(stream_);
    if (x_dtype != TN_F32 && x_dtype != TN_BF16 && x_dtype != TN_F16)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": the activation must be torch.float32, torch.bfloat16 or "
                                                          "torch.float16, got " +
                                                          tn_dtype_name(x_dtype));
    if (y_dtype != TN_F32 && y_dtype != TN_BF16 && y_dtype != TN_F16)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": unsupported output dtype " + tn_dtype_name(y_dtype));
    if (M < 0 || N < 0 || K < 0 || K % 32 != 0)
        return tn::set_error(TN_ERR_SHAPE, op + ": a q4_0 row is whole 32-element blocks (K % 32 == 0)");
    if (M > kRowsMax || K > kInMax)
        return tn::set_error(TN_ERR_SHAPE, op + ": M = " + std::to_string(M) + ", K = " + std::to_string(K) +
                                               " exceed its fixed scratch (M <= " + std::to_string(kRowsMax) +
                                               ", K <= " + std::to_string(kInMax) +
                                               "); call tn_q4_0_linear, which allocates");
    __atomic_fetch_add(&tn::counters().q4_linear_calls, 1ull, __ATOMIC_RELAXED);
    if (M == 0 || N == 0) return TN_OK;
    if (K == 0) return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": in_features == 0 is not implemented");
    if (!x || !w_blob || !y) return tn::set_error(TN_ERR_INVALID, op + ": null device pointer");
    if (x_row_stride < K) return tn::set_error(TN_ERR_INVALID, op + ": activation row stride smaller than in_features");
    if ((reinterpret_cast<uintptr_t>(w_blob) & 1) != 0)
        return tn::set_error(TN_ERR_INVALID, op + ": the q4_0 blob must be at least 2-byte aligned");
    const int chunk = tn::q4_gemv_max_rows(K);
    if (chunk <= 0)
        return tn::set_error(TN_ERR_NOT_IMPLEMENTED, op + ": in_features " + std::to_string(K) +
                                                         " is too large for the decode kernel's shared memory");

    uint8_t *scratch = nullptr;
    int st = scratch_address(&scratch);
    if (st) return st;
    // Same planar layout as tn_q4_0_linear's workspace, carved from the array:
    // codes [M][K] int8, then scales [M][K/32] and offsets [M][K/32] f32.
    const int64_t nb = K / 32;
    int8_t *xq = reinterpret_cast<int8_t *>(scratch);
    float *xd = reinterpret_cast<float *>(scratch + kCodesBytes);
    float *xc = reinterpret_cast<float *>(scratch + kCodesBytes + kScaleBytes);
    st = tn::launch_q8_planar(x, x_dtype, x_row_stride, xq, xd, xc, M, nb, K, stream);
    if (st) return st;
    const size_t ysz = tn_dtype_size(y_dtype);
    for (int64_t m0 = 0; m0 < M; m0 += chunk) {
        const int mc = (int)((M - m0) < chunk ? (M - m0) : chunk);
        st = tn::launch_q4_gemv_q8(static_cast<const uint8_t *>(w_blob), xq + m0 * K, xd + m0 * nb, xc + m0 * nb, K,
                                   bias, static_cast<uint8_t *>(y) + (size_t)m0 * N * ysz, y_dtype, N, mc, N, K, 0,
                                   stream);
        if (st) return st;
    }
    return TN_OK;
}
