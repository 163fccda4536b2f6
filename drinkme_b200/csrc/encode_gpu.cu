// The pack encoder on the GPU: uint16 BF16 bit patterns already in device
// memory -> pack format 1 radix arrays, byte-identical to the host encoder
// (encode.cpp) and so to the reference's writers (src/drinkme/codec/radix.py:
// 77-136 `pack_array`; radix_native.cpp:57-166 `plan` / `encode`).
//
// Plan: a histogram of the exponents (per-warp shared-memory counters, then
// one global add per bin and CTA); the host orders the palette (256 bins)
// exactly as encode.cpp does; a warp per block counts the weights that leave
// at each tier, which gives every block's word count; the host adds them up
// into the directory. Encode: a CTA per block builds the block's words in
// shared memory — the literal plane (sign | mantissa byte per weight), each
// nonterminal tier's codes over the weights still active (OR-ed into place,
// a field may straddle two words), the stable compaction of the escaped
// weights by a CTA-wide prefix sum, the terminal exponents — then writes them
// out. Every weight's work is independent of the others' except through the
// compaction order, which keeps the pack's order.
#include <cuda_runtime.h>

#include <algorithm>
#include <string>
#include <vector>

#include "dm_internal.h"

namespace dm {
namespace {

constexpr int kHistThreads = 256;
constexpr int kEncThreads = 256;

struct EncTables {
    uint16_t rank[256];  // exponent -> palette rank (covered when absent)
    uint8_t exit[256];   // exponent -> the tier whose code is not its escape (nw - 1: terminal)
    int32_t widths[8];
    int32_t nw;
};

__host__ __device__ inline int64_t cw(int64_t count, int64_t width) { return (count * width + 31) / 32; }

__global__ void exp_histogram_kernel(const uint16_t *bits, int64_t n, unsigned long long *hist) {
    __shared__ uint32_t h[kHistThreads / 32][256];  // one histogram per warp: fewer collisions on hot bins
    const int warp = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < (kHistThreads / 32) * 256; i += blockDim.x) (&h[0][0])[i] = 0u;
    __syncthreads();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        atomicAdd(&h[warp][(bits[i] >> 7) & 0xFF], 1u);
    __syncthreads();
    for (int e = threadIdx.x; e < 256; e += blockDim.x) {
        uint32_t s = 0;
        for (int w = 0; w < kHistThreads / 32; ++w) s += h[w][e];
        if (s) atomicAdd(&hist[e], (unsigned long long)s);
    }
}

// A warp per block: the words the block takes (radix_native.cpp plan's count).
__global__ void block_words_kernel(const uint16_t *bits, int64_t R, int64_t C, int64_t NB, int32_t B,
                                   EncTables T, uint32_t *words) {
    const int64_t blk = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (blk >= R * NB) return;
    const int64_t r = blk / NB, c0 = (blk % NB) * B;
    const int64_t n = min((int64_t)B, C - c0);
    const uint16_t *src = bits + r * C + c0;
    uint32_t cnt[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int64_t i = lane; i < n; i += 32) {
        const uint32_t e = T.exit[(src[i] >> 7) & 0xFF];
#pragma unroll
        for (int t = 0; t < 8; ++t) cnt[t] += e == (uint32_t)t ? 1u : 0u;
    }
#pragma unroll
    for (int t = 0; t < 8; ++t)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) cnt[t] += __shfl_xor_sync(0xffffffffu, cnt[t], o);
    if (lane == 0) {
        int64_t total = cw(n, 8), active = n;
        for (int t = 0; t < T.nw - 1; ++t) {
            total += cw(active, T.widths[t]);
            active -= cnt[t];
        }
        total += cw(active, 8);
        words[blk] = (uint32_t)total;
    }
}

// OR a `w`-bit field into word stream `ow` at bit `bit`.
__device__ __forceinline__ void put_field(uint32_t *ow, uint64_t bit, uint32_t v, uint32_t w) {
    const uint32_t lo = (uint32_t)(bit & 31);
    const uint64_t wi = bit >> 5;
    atomicOr(&ow[wi], v << lo);
    if (lo + w > 32) atomicOr(&ow[wi + 1], v >> (32 - lo));
}

// Exclusive prefix sum of one value per thread over the CTA (kEncThreads);
// *total gets the sum. Every thread of the CTA calls it.
__device__ __forceinline__ uint32_t cta_exclusive_scan(uint32_t v, uint32_t *warp_sums, uint32_t *total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
        uint32_t s = lane < kEncThreads / 32 ? warp_sums[lane] : 0u;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        if (lane < kEncThreads / 32) warp_sums[lane] = s;  // inclusive
    }
    __syncthreads();
    const uint32_t before = (warp > 0 ? warp_sums[warp - 1] : 0u) + x - v;
    *total = warp_sums[kEncThreads / 32 - 1];
    __syncthreads();  // warp_sums is reused by the next call
    return before;
}

// A CTA per block: the block's words (radix_native.cpp encode).
__global__ void __launch_bounds__(kEncThreads) encode_block_kernel(const uint16_t *bits, int64_t R, int64_t C,
                                                                    int64_t NB, int32_t B, EncTables T,
                                                                    const uint32_t *offsets, uint32_t *data,
                                                                    int32_t max_words, int *bad) {
    extern __shared__ __align__(16) uint32_t sm[];
    __shared__ uint32_t warp_sums[kEncThreads / 32];
    uint32_t *ow = sm;                                             // [max_words] the block's words
    uint16_t *act = reinterpret_cast<uint16_t *>(ow + max_words);  // [B] active weights, pack order
    uint16_t *nxt = act + B;                                       // [B] the next tier's
    uint16_t *rk = nxt + B;                                        // [B] palette rank per weight
    uint8_t *ex = reinterpret_cast<uint8_t *>(rk + B);             // [B] exponent per weight
    const int64_t blk = blockIdx.x;
    const int64_t r = blk / NB, c0 = (blk % NB) * B;
    const int32_t n = (int32_t)min((int64_t)B, C - c0);
    const uint16_t *src = bits + r * C + c0;
    const int64_t avail = (int64_t)offsets[blk + 1] - (int64_t)offsets[blk];
    if (avail > max_words) {  // the directory does not match these bits (uniform over the CTA)
        if (threadIdx.x == 0) atomicExch(bad, 1);
        return;
    }
    for (int64_t i = threadIdx.x; i < avail; i += blockDim.x) ow[i] = 0u;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const uint32_t v = src[i];
        const uint32_t e = (v >> 7) & 0xFF;
        atomicOr(&ow[i >> 2], ((v & 0x7Fu) | ((v >> 8) & 0x80u)) << (8 * (i & 3)));
        ex[i] = (uint8_t)e;
        rk[i] = T.rank[e];
        act[i] = (uint16_t)i;
    }
    __syncthreads();
    int64_t pos = cw(n, 8);
    int32_t active = n, base = 0;
    for (int t = 0; t < T.nw - 1; ++t) {
        const uint32_t w = (uint32_t)T.widths[t], esc = (1u << w) - 1u;
        if (pos + cw(active, w) > avail) {
            if (threadIdx.x == 0) atomicExch(bad, 1);
            return;
        }
        // thread k takes active positions [j0, j1): codes in place, then its
        // escaped weights at its offset among the CTA's, in order
        const int32_t per = (active + kEncThreads - 1) / kEncThreads;
        const int32_t j0 = min(active, (int32_t)threadIdx.x * per), j1 = min(active, j0 + per);
        uint32_t kept = 0;
        for (int32_t j = j0; j < j1; ++j) {
            const uint32_t code = min((uint32_t)(rk[act[j]] - base), esc);
            put_field(ow + pos, (uint64_t)j * w, code, w);
            kept += code == esc ? 1u : 0u;
        }
        uint32_t total;
        uint32_t o = cta_exclusive_scan(kept, warp_sums, &total);
        for (int32_t j = j0; j < j1; ++j) {
            const uint16_t i = act[j];
            if ((uint32_t)(rk[i] - base) >= esc) nxt[o++] = i;
        }
        __syncthreads();
        for (int32_t j = threadIdx.x; j < (int32_t)total; j += blockDim.x) act[j] = nxt[j];
        __syncthreads();
        pos += cw(active, w);
        active = (int32_t)total;
        base += (int32_t)esc;
    }
    if (pos + cw(active, 8) != avail) {
        if (threadIdx.x == 0) atomicExch(bad, 1);
        return;
    }
    for (int32_t j = threadIdx.x; j < active; j += blockDim.x) put_field(ow + pos, (uint64_t)j * 8, ex[act[j]], 8);
    __syncthreads();
    uint32_t *out = data + offsets[blk];
    for (int64_t i = threadIdx.x; i < avail; i += blockDim.x) out[i] = ow[i];
}

struct Guard {
    int prev = -1;
    explicit Guard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (dev >= 0 && prev != dev) cudaSetDevice(dev);
    }
    ~Guard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

int device_of(const void *p, int *dev, std::string &msg) {
    cudaPointerAttributes at{};
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess || at.type != cudaMemoryTypeDevice) {
        cudaGetLastError();
        msg = "expected device memory";
        return DM_EINVAL;
    }
    *dev = at.device;
    return DM_OK;
}

int tables_of(const uint8_t *palette, int32_t covered, const int32_t *widths, int32_t nw, EncTables &T) {
    for (int e = 0; e < 256; ++e) T.rank[e] = (uint16_t)covered;
    for (int k = 0; k < covered; ++k) T.rank[palette[k]] = (uint16_t)k;
    for (int e = 0; e < 256; ++e) {
        int base = 0, tier = nw - 1;
        for (int t = 0; t < nw - 1; ++t) {
            const int esc = (1 << widths[t]) - 1;
            if (T.rank[e] < base + esc) {
                tier = t;
                break;
            }
            base += esc;
        }
        T.exit[e] = (uint8_t)tier;
    }
    for (int t = 0; t < 8; ++t) T.widths[t] = t < nw ? widths[t] : 0;
    T.nw = nw;
    return 0;
}

int cuda_err(cudaError_t e, const char *what, std::string &msg) {
    msg = std::string(what) + ": " + cudaGetErrorString(e);
    return DM_ECUDA;
}

}  // namespace
}  // namespace dm

extern "C" int dm_pack_plan_device(const uint16_t *d_bits, int64_t R, int64_t C, const int32_t *widths, int32_t nw,
                                   int32_t B, uint8_t *host_palette, uint32_t *host_offsets, uint64_t *nwords,
                                   void *stream, char *err, size_t err_len) {
    std::string msg;
    int32_t covered;
    if (!d_bits || !widths || !host_palette || !host_offsets || !nwords) {
        dm::set_error(err, err_len, "dm_pack_plan_device: null pointer");
        return DM_EINVAL;
    }
    if (dm::check_pack_params(R, C, widths, nw, B, &covered, msg)) {
        dm::set_error(err, err_len, msg);
        return DM_EINVAL;
    }
    int dev = 0;
    if (int rc = dm::device_of(d_bits, &dev, msg)) {
        dm::set_error(err, err_len, "dm_pack_plan_device: the bits must be " + msg);
        return rc;
    }
    dm::Guard g(dev);
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t NB = (C + B - 1) / B, nblk = R * NB;
    if (nblk > (int64_t)INT32_MAX * 4) {
        dm::set_error(err, err_len, "dm_pack_plan_device: too many blocks");
        return DM_EINVAL;
    }
    unsigned long long *d_hist = nullptr;
    uint32_t *d_words = nullptr;
    cudaError_t e;
    int rc = DM_OK;
    if ((e = cudaMallocAsync((void **)&d_hist, 256 * sizeof(unsigned long long), s)) != cudaSuccess ||
        (e = cudaMallocAsync((void **)&d_words, (size_t)nblk * sizeof(uint32_t), s)) != cudaSuccess) {
        rc = dm::cuda_err(e, "cudaMallocAsync", msg);
    }
    std::vector<uint64_t> hist(256);
    dm::EncTables T{};
    std::vector<uint32_t> words((size_t)nblk);
    if (!rc) {
        const int64_t n = R * C;
        const int grid = (int)std::min<int64_t>(148 * 8, (n + dm::kHistThreads * 8 - 1) / (dm::kHistThreads * 8));
        cudaMemsetAsync(d_hist, 0, 256 * sizeof(unsigned long long), s);
        dm::exp_histogram_kernel<<<std::max(grid, 1), dm::kHistThreads, 0, s>>>(d_bits, n, d_hist);
        if ((e = cudaMemcpyAsync(hist.data(), d_hist, 256 * sizeof(uint64_t), cudaMemcpyDeviceToHost, s)) !=
                cudaSuccess ||
            (e = cudaStreamSynchronize(s)) != cudaSuccess)
            rc = dm::cuda_err(e, "dm_pack_plan_device: histogram", msg);
    }
    if (!rc) {
        dm::palette_from_histogram(hist.data(), covered, host_palette, T.rank);
        dm::tables_of(host_palette, covered, widths, nw, T);
        const int per_cta = 8;  // warps per CTA, a block each
        const int64_t grid = (nblk + per_cta - 1) / per_cta;
        dm::block_words_kernel<<<(unsigned)grid, 32 * per_cta, 0, s>>>(d_bits, R, C, NB, B, T, d_words);
        if ((e = cudaMemcpyAsync(words.data(), d_words, (size_t)nblk * sizeof(uint32_t), cudaMemcpyDeviceToHost, s)) !=
                cudaSuccess ||
            (e = cudaStreamSynchronize(s)) != cudaSuccess)
            rc = dm::cuda_err(e, "dm_pack_plan_device: block words", msg);
    }
    if (d_hist) cudaFreeAsync(d_hist, s);
    if (d_words) cudaFreeAsync(d_words, s);
    if (!rc) {
        uint64_t acc = 0;
        host_offsets[0] = 0;
        for (int64_t b = 0; b < nblk; ++b) {
            acc += words[(size_t)b];
            if (acc > UINT32_MAX) {
                msg = "radix payload exceeds the uint32 word directory";
                rc = DM_EINVAL;
                break;
            }
            host_offsets[b + 1] = (uint32_t)acc;
        }
        *nwords = acc;
    }
    if (rc) dm::set_error(err, err_len, msg);
    return rc;
}

extern "C" int dm_pack_encode_device(const uint16_t *d_bits, int64_t R, int64_t C, const int32_t *widths,
                                     int32_t nw, int32_t B, const uint8_t *host_palette, const uint32_t *host_offsets,
                                     uint32_t *d_data, uint64_t nwords, void *stream, char *err, size_t err_len) {
    std::string msg;
    int32_t covered;
    if (!d_bits || !widths || !host_palette || !host_offsets || !d_data) {
        dm::set_error(err, err_len, "dm_pack_encode_device: null pointer");
        return DM_EINVAL;
    }
    if (dm::check_pack_params(R, C, widths, nw, B, &covered, msg)) {
        dm::set_error(err, err_len, msg);
        return DM_EINVAL;
    }
    const int64_t NB = (C + B - 1) / B, nblk = R * NB;
    if (host_offsets[0] != 0 || host_offsets[nblk] != nwords) {
        dm::set_error(err, err_len, "directory endpoints");
        return DM_EINVAL;
    }
    if (nblk > (int64_t)INT32_MAX) {
        dm::set_error(err, err_len, "dm_pack_encode_device: too many blocks");
        return DM_EINVAL;
    }
    int dev = 0, ddev = 0;
    if (dm::device_of(d_bits, &dev, msg) || dm::device_of(d_data, &ddev, msg) || dev != ddev) {
        dm::set_error(err, err_len, "dm_pack_encode_device: the bits and the data must be device memory of one GPU");
        return DM_EINVAL;
    }
    dm::Guard g(dev);
    cudaStream_t s = (cudaStream_t)stream;
    dm::EncTables T{};
    dm::tables_of(host_palette, covered, widths, nw, T);
    const int32_t max_words = (int32_t)dm::block_words_most(B, widths, nw);
    const size_t smem = (size_t)max_words * 4 + (size_t)B * (3 * 2 + 1);
    uint32_t *d_off = nullptr;
    int *d_bad = nullptr;
    cudaError_t e;
    int rc = DM_OK;
    if ((e = cudaMallocAsync((void **)&d_off, (size_t)(nblk + 1) * sizeof(uint32_t), s)) != cudaSuccess ||
        (e = cudaMallocAsync((void **)&d_bad, sizeof(int), s)) != cudaSuccess)
        rc = dm::cuda_err(e, "cudaMallocAsync", msg);
    int bad = 0;
    if (!rc) {
        cudaMemcpyAsync(d_off, host_offsets, (size_t)(nblk + 1) * sizeof(uint32_t), cudaMemcpyHostToDevice, s);
        cudaMemsetAsync(d_bad, 0, sizeof(int), s);
        if ((e = cudaFuncSetAttribute(dm::encode_block_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem)) != cudaSuccess)
            rc = dm::cuda_err(e, "cudaFuncSetAttribute", msg);
    }
    if (!rc) {
        dm::encode_block_kernel<<<(unsigned)nblk, dm::kEncThreads, smem, s>>>(d_bits, R, C, NB, B, T, d_off, d_data,
                                                                             max_words, d_bad);
        if ((e = cudaGetLastError()) != cudaSuccess ||
            (e = cudaMemcpyAsync(&bad, d_bad, sizeof(int), cudaMemcpyDeviceToHost, s)) != cudaSuccess ||
            (e = cudaStreamSynchronize(s)) != cudaSuccess)
            rc = dm::cuda_err(e, "dm_pack_encode_device", msg);
    }
    if (d_off) cudaFreeAsync(d_off, s);
    if (d_bad) cudaFreeAsync(d_bad, s);
    if (!rc && bad) {
        msg = "terminal stream mismatch: the directory does not match these bits";
        rc = DM_EINVAL;
    }
    if (rc) dm::set_error(err, err_len, msg);
    return rc;
}
