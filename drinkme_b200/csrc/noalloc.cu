// dm_gemv_noalloc: the fused decode + GEMV for callers that cannot allocate
// device memory when they call it.
//
// dm_gemv's sip kernel needs scratch: stream-K partial sums and per-tile
// arrival counters (plus a bf16 split buffer for fp32 activations). dm_gemv
// takes it from buffers the tensor handle allocated at load time. This entry
// point takes it from one fixed array in the library's device memory
// instead, so the call itself never allocates. It is for callers such as a
// serving engine that has handed all free HBM to its own pool (KV cache,
// activations) before decoding starts, or a decode loop that must not call
// cudaMalloc because it can synchronise the device: they load their tensors
// once, then run every GEMV through here with no allocator involved.
//
// The array is a file-scope static __device__ object, so every GPU that
// loads the library holds it until the process exits. Host code cannot pass
// the array's name to a kernel (on the host it is a stand-in, not a device
// address): the first call on each device looks its address up with
// cudaGetSymbolAddress, with that device current, and caches it. That first
// call should come before any CUDA-graph capture on the device. The cached
// address assumes the device's primary context lives until the process
// exits: after cudaDeviceReset (or any teardown of that context) the cache is
// stale, and this entry point must not be called again in the process.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <string>

#include "dm_internal.h"

namespace {

// The limits of the static scratch (about 1.45 MiB per GPU):
constexpr int64_t kNoAllocMaxWorkers = 1024;  // stream-K workers (CTAs) of one launch: 148 on a B200
constexpr int64_t kNoAllocMaxTiles = 16384;   // 16-row tiles: tensors (or row shards) of up to 262,144 rows
constexpr int64_t kNoAllocMaxCols = 32768;    // columns of a staged activation row (fp32 split, unaligned bf16)

constexpr size_t kPartialBytes = (size_t)kNoAllocMaxWorkers * 2 * 128 * sizeof(float);
constexpr size_t kCounterBytes = (size_t)kNoAllocMaxTiles * sizeof(int);
constexpr size_t kSplitBytes = (size_t)6 * kNoAllocMaxCols * sizeof(uint16_t);
constexpr size_t kScratchBytes = kPartialBytes + kCounterBytes + kSplitBytes;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_lock;
void *g_scratch_addr[kMaxDevices] = {nullptr};

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

// The device address of the static scratch on `device` (current). Looked up
// once per device and cached.
int scratch_address(int device, unsigned char **out, std::string &msg) {
    if (device < 0 || device >= kMaxDevices) {
        msg = "dm_gemv_noalloc: device ordinal " + std::to_string(device) + " outside 0.." +
              std::to_string(kMaxDevices - 1);
        return DM_EINVAL;
    }
    std::lock_guard<std::mutex> lk(g_lock);
    if (!g_scratch_addr[device]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) {
            msg = std::string("cudaGetSymbolAddress(no-alloc scratch): ") + cudaGetErrorString(e);
            return DM_ECUDA;
        }
        g_scratch_addr[device] = p;
    }
    *out = static_cast<unsigned char *>(g_scratch_addr[device]);
    return DM_OK;
}

int fail(char *err, size_t len, int code, const std::string &msg) {
    dm::set_error(err, len, msg);
    return code;
}

}  // namespace

extern "C" int dm_gemv_noalloc(const dm_tensor *t, const void *x, int32_t x_dtype, int64_t M, const void *bias,
                               void *out, int32_t out_dtype, void *stream, char *err, size_t err_len) {
    if (!t || !x || !out) return fail(err, err_len, DM_EINVAL, "dm_gemv_noalloc: null pointer");
    if (M < 1 || M > DM_MC_MAX)
        return fail(err, err_len, DM_EINVAL,
                    "radix gemv_mc: M=" + std::to_string(M) + " outside 1.." + std::to_string(DM_MC_MAX));
    if ((x_dtype != DM_BF16 && x_dtype != DM_F32) || (out_dtype != DM_BF16 && out_dtype != DM_F32))
        return fail(err, err_len, DM_EINVAL, "dm_gemv_noalloc: dtype must be DM_BF16 or DM_F32");
    if ((reinterpret_cast<uintptr_t>(x) & (x_dtype == DM_F32 ? 3u : 1u)) != 0)
        return fail(err, err_len, DM_EINVAL, "dm_gemv_noalloc: activations not aligned to their element size");
    DeviceGuard guard(t->device);
    std::string msg;
    const uint16_t *b16 = reinterpret_cast<const uint16_t *>(bias);
    const int of32 = out_dtype == DM_F32;
    if (!t->L.fast_sip) {
        // the general kernel keeps its sums in registers: no scratch to place
        int rc = dm::launch_gemv_generic(t, x, x_dtype == DM_F32, M, b16, out, of32, stream, msg);
        if (rc) dm::set_error(err, err_len, msg);
        return rc;
    }
    if (t->L.tiles > kNoAllocMaxTiles)
        return fail(err, err_len, DM_EINVAL,
                    "dm_gemv_noalloc: " + std::to_string(t->L.rows) + " rows exceed the static scratch's " +
                        std::to_string(kNoAllocMaxTiles * dm::kUnitRows) + " (use dm_gemv)");
    // fp32 activations are split, and bf16 ones off a 16-byte boundary copied,
    // into the array's staging part before the kernel reads them
    const bool staged = x_dtype == DM_F32 || (reinterpret_cast<uintptr_t>(x) & 15) != 0;
    if (staged && t->L.C > kNoAllocMaxCols)
        return fail(err, err_len, DM_EINVAL,
                    "dm_gemv_noalloc: " + std::string(x_dtype == DM_F32 ? "fp32" : "unaligned bf16") +
                        " activations of " + std::to_string(t->L.C) + " columns exceed the static scratch's " +
                        std::to_string(kNoAllocMaxCols) + " (use dm_gemv)");
    unsigned char *base = nullptr;
    int rc = scratch_address(t->device, &base, msg);
    if (rc) return fail(err, err_len, rc, msg);
    float *partials = reinterpret_cast<float *>(base);
    int *counters = reinterpret_cast<int *>(base + kPartialBytes);
    uint16_t *xstage = reinterpret_cast<uint16_t *>(base + kPartialBytes + kCounterBytes);
    // the array keeps the last call's contents: the arrival counters start at zero
    cudaError_t e = cudaMemsetAsync(counters, 0, (size_t)t->L.tiles * sizeof(int), (cudaStream_t)stream);
    if (e != cudaSuccess)
        return fail(err, err_len, DM_ECUDA, std::string("cudaMemsetAsync(counters): ") + cudaGetErrorString(e));
    rc = dm::gemv_sip_rows(t, x, x_dtype == DM_F32, M, b16, out, of32, xstage, (int64_t)6 * kNoAllocMaxCols, partials,
                           counters, kNoAllocMaxWorkers, stream, msg);
    if (rc) dm::set_error(err, err_len, msg);
    return rc;
}
