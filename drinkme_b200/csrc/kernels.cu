// The general kernels: any tier widths (2..8 tiers), any block size, ragged
// rows. One warp walks one row-block; a weight's rank inside each later
// tier's stream comes from a warp ballot over the weights that escaped the
// tier before it (the reference's scheduled decoder,
// src/drinkme/codec/radix_kernel_gpu.py:70-99, as SIMT: per 32-weight chunk,
// one ballot + popc per tier).
//
// Also here: the gulp schedule over the original pack layout
// (radix_ops.prepare_schedule), the fp32 activation split the sip kernel
// reads, and the raw bf16 GEMV (radix_ops.gemv_narrow and the raw lm_head).
#include <cuda_runtime.h>

#include <algorithm>
#include <string>

#include "dm_device.cuh"
#include "dm_internal.h"

namespace dm {

struct GenericParams {
    const uint8_t *data;
    const uint32_t *unit16;
    int64_t rows, C, NB;
    int32_t B, nw;
    int32_t widths[8];
    uint8_t palette[256];
};

__device__ __forceinline__ uint32_t lanemask_lt() {
    uint32_t m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

__device__ __forceinline__ int cwd(int count, int width) { return (count * width + 31) / 32; }

// One row-block's streams, walked 32 weights at a time by a warp.
struct BlockWalker {
    const uint32_t *s;
    int n;
    int start[8];  // word offset of every nonterminal tier's stream, then the terminal's
    int run[8];    // per later tier: codes consumed so far (the next rank)

    __device__ void init(const GenericParams &p, const uint32_t *stream, int nweights) {
        s = stream;
        n = nweights;
        int pos = cwd(n, 8), cnt = n;
        for (int t = 0; t < p.nw - 1; ++t) {
            const int w = p.widths[t];
            const uint32_t esc = (1u << w) - 1u;
            start[t] = pos;
            run[t] = 0;
            if (t < p.nw - 2) {  // how many of this tier's codes escape: the next tier's count
                int next = 0;
                for (int b = 0; b < cnt; b += 32) {
                    int i = b + (threadIdx.x & 31);
                    bool e = i < cnt && field(s + pos, (uint32_t)i, (uint32_t)w) == esc;
                    next += __popc(__ballot_sync(0xffffffffu, e));
                }
                pos += cwd(cnt, w);
                cnt = next;
            } else {
                pos += cwd(cnt, w);
            }
        }
        start[p.nw - 1] = pos;
        run[p.nw - 1] = 0;
    }

    // The bf16 bits of weight c0 + lane (0 for lanes past n).
    __device__ uint32_t chunk(const GenericParams &p, int c0) {
        const int lane = threadIdx.x & 31;
        const int i = c0 + lane;
        const bool act = i < n;
        uint32_t lit = act ? field(s, (uint32_t)i, 8) : 0u;
        uint32_t ex = 0;
        bool reach = act;  // this weight's exponent is still undecided
        int base = 0;
        for (int t = 0; t < p.nw - 1; ++t) {
            const int w = p.widths[t];
            const uint32_t esc = (1u << w) - 1u;
            int rank;
            if (t == 0) {
                rank = i;
            } else {
                uint32_t bal = __ballot_sync(0xffffffffu, reach);
                rank = run[t] + __popc(bal & lanemask_lt());
                run[t] += __popc(bal);
            }
            uint32_t code = reach ? field(s + start[t], (uint32_t)rank, (uint32_t)w) : 0u;
            bool next = reach && code == esc;
            if (reach && !next) ex = p.palette[base + code];
            reach = next;
            base += (int)esc;
        }
        {
            const int T = p.nw - 1;
            uint32_t bal = __ballot_sync(0xffffffffu, reach);
            int rank = run[T] + __popc(bal & lanemask_lt());
            run[T] += __popc(bal);
            if (reach) ex = field(s + start[T], (uint32_t)rank, 8);
        }
        return (lit & 0x7Fu) | ((lit >> 7) << 15) | (ex << 7);
    }
};

__device__ __forceinline__ const uint32_t *row_block_stream(const GenericParams &p, int64_t r, int64_t b,
                                                            int *words) {
    int64_t u = (r / kUnitRows) * p.NB + b;
    const uint8_t *unit = p.data + (size_t)p.unit16[u] * 16;
    const RowEntry *hdr = reinterpret_cast<const RowEntry *>(unit);
    RowEntry e = hdr[r % kUnitRows];
    *words = e.words;
    return reinterpret_cast<const uint32_t *>(unit + (size_t)e.off16 * 16);
}

__global__ void __launch_bounds__(128) decode_generic_kernel(GenericParams p, uint16_t *out) {
    const int64_t warp = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
    if (warp >= p.rows * p.NB) return;
    const int64_t r = warp / p.NB, b = warp % p.NB;
    int words;
    const uint32_t *s = row_block_stream(p, r, b, &words);
    const int n = (int)((p.C - b * p.B) < p.B ? (p.C - b * p.B) : p.B);
    BlockWalker w;
    w.init(p, s, n);
    uint16_t *dst = out + r * p.C + b * p.B;
    for (int c0 = 0; c0 < n; c0 += 32) {
        uint32_t bits = w.chunk(p, c0);
        int i = c0 + (threadIdx.x & 31);
        if (i < n) dst[i] = (uint16_t)bits;
    }
}

// The same walk over a pack as stored (pack format 1: the block directory and
// the word stream, no device layout): a warp per block. For verification and
// for callers that hold a pack in device memory as it is.
__global__ void __launch_bounds__(128) decode_pack_kernel(GenericParams p, const uint32_t *words,
                                                          const uint32_t *offsets, uint16_t *out) {
    const int64_t warp = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
    if (warp >= p.rows * p.NB) return;
    const int64_t r = warp / p.NB, b = warp % p.NB;
    const uint32_t *s = words + offsets[warp];
    const int n = (int)((p.C - b * p.B) < p.B ? (p.C - b * p.B) : p.B);
    BlockWalker w;
    w.init(p, s, n);
    uint16_t *dst = out + r * p.C + b * p.B;
    for (int c0 = 0; c0 < n; c0 += 32) {
        uint32_t bits = w.chunk(p, c0);
        int i = c0 + (threadIdx.x & 31);
        if (i < n) dst[i] = (uint16_t)bits;
    }
}

// One warp per output row: every block of the row decoded and contracted with
// up to 8 activation rows, fp32 accumulate per lane, a fixed butterfly
// reduction, then bias in fp32 and one rounding. Column m's arithmetic does
// not depend on M.
__global__ void __launch_bounds__(128) gemv_generic_kernel(GenericParams p, const void *x, int x_f32, int M,
                                                           const uint16_t *bias, void *out, int out_f32) {
    const int64_t r = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
    if (r >= p.rows) return;
    const int lane = threadIdx.x & 31;
    float acc[kMaxVirtualRows];
#pragma unroll
    for (int m = 0; m < kMaxVirtualRows; ++m) acc[m] = 0.f;
    for (int64_t b = 0; b < p.NB; ++b) {
        int words;
        const uint32_t *s = row_block_stream(p, r, b, &words);
        const int n = (int)((p.C - b * p.B) < p.B ? (p.C - b * p.B) : p.B);
        BlockWalker w;
        w.init(p, s, n);
        for (int c0 = 0; c0 < n; c0 += 32) {
            float wv = bf16_bits_to_f32(w.chunk(p, c0));
            int i = c0 + lane;
            if (i < n) {
                int64_t col = b * p.B + i;
#pragma unroll
                for (int m = 0; m < kMaxVirtualRows; ++m) {
                    if (m < M) {
                        float xv = x_f32 ? reinterpret_cast<const float *>(x)[m * p.C + col]
                                         : bf16_bits_to_f32(reinterpret_cast<const uint16_t *>(x)[m * p.C + col]);
                        acc[m] = fmaf(xv, wv, acc[m]);
                    }
                }
            }
        }
    }
#pragma unroll
    for (int m = 0; m < kMaxVirtualRows; ++m) {
        float v = acc[m];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        acc[m] = v;
    }
    if (lane == 0) {
        const float bv = bias ? bf16_bits_to_f32(bias[r]) : 0.f;
#pragma unroll
        for (int m = 0; m < kMaxVirtualRows; ++m) {
            if (m < M) {
                float y = acc[m] + bv;
                if (out_f32)
                    reinterpret_cast<float *>(out)[m * p.rows + r] = y;
                else
                    reinterpret_cast<uint16_t *>(out)[m * p.rows + r] = f32_to_bf16_bits(y);
            }
        }
    }
}

struct SchedParams {
    const uint32_t *data;
    const uint32_t *offsets;
    int64_t nwords, C, nblocks;
    int32_t B, nw;
    int32_t widths[8];
};

__device__ __forceinline__ uint32_t field_bounded(const uint32_t *data, int64_t nwords, int64_t wbase, uint32_t index,
                                                  uint32_t width) {
    int64_t bit = (int64_t)index * width, wi = wbase + (bit >> 5);
    uint32_t lo = (uint32_t)(bit & 31);
    uint32_t a = wi < nwords ? data[wi] : 0u, b = wi + 1 < nwords ? data[wi + 1] : 0u;
    uint32_t v = a >> lo;
    if (lo + width > 32) v |= b << (32 - lo);
    return v & ((1u << width) - 1u);
}

// radix_kernel_gpu._prepare_schedule (radix_kernel_gpu.py:45-66): per block,
// byte (k-1) of a uint16 = word length of nonterminal tier k (k >= 1).
__global__ void __launch_bounds__(128) schedule_kernel(SchedParams p, uint16_t *out) {
    const int64_t blk = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
    if (blk >= p.nblocks) return;
    const int64_t NB = (p.C + p.B - 1) / p.B;
    const int n = (int)((p.C - (blk % NB) * p.B) < p.B ? (p.C - (blk % NB) * p.B) : p.B);
    int64_t pos = (int64_t)p.offsets[blk] + cwd(n, 8);
    int cnt = n;
    uint32_t header = 0;
    for (int t = 0; t < p.nw - 1; ++t) {
        const int w = p.widths[t];
        const uint32_t esc = (1u << w) - 1u;
        const int words = cwd(cnt, w);
        if (t > 0) header |= (uint32_t)words << ((t - 1) * 8);
        if (t < p.nw - 2) {
            int next = 0;
            for (int b = 0; b < cnt; b += 32) {
                int i = b + (threadIdx.x & 31);
                bool e = i < cnt && field_bounded(p.data, p.nwords, pos, (uint32_t)i, (uint32_t)w) == esc;
                next += __popc(__ballot_sync(0xffffffffu, e));
            }
            cnt = next;
        }
        pos += words;
    }
    if ((threadIdx.x & 31) == 0) out[blk] = (uint16_t)header;
}

// fp32 activations [M, C] -> bf16 rows [3M, C]: hi, mid, lo with
// x = hi + mid + lo to within 2^-26 |x| (each piece is the round-to-nearest
// bf16 of what the pieces before it left), so a bf16 x bf16 MMA over the
// three pieces is an fp32-accurate product with x.
__global__ void split_f32_kernel(const float *x, int64_t C, int64_t M, uint16_t *out) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= M * C) return;
    int64_t m = i / C, c = i % C;
    float v = x[i];
    uint16_t h = f32_to_bf16_bits(v);
    float r1 = v - bf16_bits_to_f32(h);
    uint16_t md = f32_to_bf16_bits(r1);
    float r2 = r1 - bf16_bits_to_f32(md);
    uint16_t lo = f32_to_bf16_bits(r2);
    out[(3 * m + 0) * C + c] = h;
    out[(3 * m + 1) * C + c] = md;
    out[(3 * m + 2) * C + c] = lo;
}

// Raw bf16 GEMV: one warp per output row, 16-byte loads along the row, MM
// activation rows (1..8) per pass over the weights, a fixed butterfly
// reduction.
template <int XF32, int MM>
__global__ void __launch_bounds__(256) gemv_raw_kernel(const uint16_t *w, int64_t R, int64_t C, const void *x,
                                                       const uint16_t *bias, void *out, int out_f32, int vec) {
    constexpr int M = MM;
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = (int64_t)gridDim.x * 8;
    for (int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); r < R; r += nwarps) {
        const uint16_t *row = w + r * C;
        float acc[MM];
#pragma unroll
        for (int m = 0; m < MM; ++m) acc[m] = 0.f;
        if (vec) {  // C % 8 == 0 and 16-byte aligned weight and activations: 16-byte loads
            // 16 weights of the row at c times the activations, in c order
            auto step = [&](int64_t c, uint4 wv) {
                const uint32_t wp[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                for (int m = 0; m < MM; ++m) {
                    float xs[8];
                    if (XF32) {
                        const float4 *xp =
                            reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(x) + m * C + c);
                        const float4 a = __ldg(xp), b = __ldg(xp + 1);
                        xs[0] = a.x; xs[1] = a.y; xs[2] = a.z; xs[3] = a.w;
                        xs[4] = b.x; xs[5] = b.y; xs[6] = b.z; xs[7] = b.w;
                    } else {
                        const uint4 xv =
                            __ldg(reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(x) + m * C + c));
                        const uint32_t xp[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            xs[2 * k] = __uint_as_float(xp[k] << 16);
                            xs[2 * k + 1] = __uint_as_float(xp[k] & 0xFFFF0000u);
                        }
                    }
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        acc[m] = fmaf(xs[2 * k], __uint_as_float(wp[k] << 16), acc[m]);
                        acc[m] = fmaf(xs[2 * k + 1], __uint_as_float(wp[k] & 0xFFFF0000u), acc[m]);
                    }
                }
            };
            // four 16-byte weight loads in flight per lane (streamed: the
            // weights are read once, the activations stay cached)
            int64_t c = (int64_t)lane * 8;
            for (; c + 3 * 256 < C; c += 4 * 256) {
                const uint4 w0 = __ldcs(reinterpret_cast<const uint4 *>(row + c));
                const uint4 w1 = __ldcs(reinterpret_cast<const uint4 *>(row + c + 256));
                const uint4 w2 = __ldcs(reinterpret_cast<const uint4 *>(row + c + 512));
                const uint4 w3 = __ldcs(reinterpret_cast<const uint4 *>(row + c + 768));
                step(c, w0);
                step(c + 256, w1);
                step(c + 512, w2);
                step(c + 768, w3);
            }
            for (; c < C; c += 256) step(c, __ldcs(reinterpret_cast<const uint4 *>(row + c)));
        } else {
            for (int64_t c = lane; c < C; c += 32) {
                float wf = bf16_bits_to_f32(row[c]);
#pragma unroll
                for (int m = 0; m < MM; ++m) {
                    const float xv = XF32 ? reinterpret_cast<const float *>(x)[m * C + c]
                                          : bf16_bits_to_f32(reinterpret_cast<const uint16_t *>(x)[m * C + c]);
                    acc[m] = fmaf(xv, wf, acc[m]);
                }
            }
        }
#pragma unroll
        for (int m = 0; m < MM; ++m) {
            float v = acc[m];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            acc[m] = v;
        }
        if (lane == 0) {
            const float bv = bias ? bf16_bits_to_f32(bias[r]) : 0.f;
#pragma unroll
            for (int m = 0; m < MM; ++m) {
                const float y = acc[m] + bv;
                if (out_f32)
                    reinterpret_cast<float *>(out)[m * R + r] = y;
                else
                    reinterpret_cast<uint16_t *>(out)[m * R + r] = f32_to_bf16_bits(y);
            }
        }
    }
}

static GenericParams generic_params(const dm_tensor *t) {
    GenericParams p{};
    p.data = t->d_data;
    p.unit16 = t->d_unit16;
    p.rows = t->L.rows;
    p.C = t->L.C;
    p.NB = t->L.NB;
    p.B = t->L.B;
    p.nw = t->L.nw;
    for (int i = 0; i < 8; ++i) p.widths[i] = t->L.widths[i];
    for (int i = 0; i < 256; ++i) p.palette[i] = t->L.palette[i];
    return p;
}

static int cuda_check(cudaError_t e, const char *what, std::string &msg) {
    if (e == cudaSuccess) return DM_OK;
    msg = std::string(what) + ": " + cudaGetErrorString(e);
    return DM_ECUDA;
}

// The general kernels walk each block's tier-0 codes as the pack's plain
// 3-bit stream; a sip fast-path layout holds them as code planes instead
// (layout.cpp: sip_code_planes), which these kernels must never read.
static bool plain_streams(const dm_tensor *t, const char *who, std::string &msg) {
    if (!t->L.fast_sip) return true;
    msg = std::string(who) + ": a sip fast-path layout (code planes) is served by the sip kernels only";
    return false;
}

int launch_decode_generic(const dm_tensor *t, uint16_t *out, void *stream, std::string &msg) {
    if (!plain_streams(t, "decode_generic_kernel", msg)) return DM_EINVAL;
    GenericParams p = generic_params(t);
    int64_t warps = p.rows * p.NB;
    int64_t blocks = (warps + 3) / 4;
    decode_generic_kernel<<<(unsigned)blocks, 128, 0, (cudaStream_t)stream>>>(p, out);
    return cuda_check(cudaGetLastError(), "decode_generic_kernel", msg);
}

int launch_decode_pack(const uint8_t *palette, size_t npal, int64_t R, int64_t C, const int32_t *widths, int32_t nw,
                       int32_t B, const uint32_t *words, const uint32_t *offsets, uint16_t *out, void *stream,
                       std::string &msg) {
    GenericParams p{};
    p.rows = R;
    p.C = C;
    p.B = B;
    p.NB = (C + B - 1) / B;
    p.nw = nw;
    for (int i = 0; i < nw && i < 8; ++i) p.widths[i] = widths[i];
    for (size_t i = 0; i < npal && i < 256; ++i) p.palette[i] = palette[i];
    const int64_t warps = R * p.NB;
    if (warps == 0) return DM_OK;
    decode_pack_kernel<<<(unsigned)((warps + 3) / 4), 128, 0, (cudaStream_t)stream>>>(p, words, offsets, out);
    return cuda_check(cudaGetLastError(), "decode_pack_kernel", msg);
}

int launch_gemv_generic(const dm_tensor *t, const void *x, int x_f32, int64_t M, const uint16_t *bias, void *out,
                        int out_f32, void *stream, std::string &msg) {
    if (!plain_streams(t, "gemv_generic_kernel", msg)) return DM_EINVAL;
    GenericParams p = generic_params(t);
    int64_t blocks = (p.rows + 3) / 4;
    gemv_generic_kernel<<<(unsigned)blocks, 128, 0, (cudaStream_t)stream>>>(p, x, x_f32, (int)M, bias, out, out_f32);
    return cuda_check(cudaGetLastError(), "gemv_generic_kernel", msg);
}

int launch_prepare_schedule(const uint32_t *data, size_t nwords, const uint32_t *offsets, int64_t C,
                            const int32_t *widths, int32_t nw, int32_t B, int64_t nblocks, uint16_t *out,
                            void *stream, std::string &msg) {
    SchedParams p{};
    p.data = data;
    p.offsets = offsets;
    p.nwords = (int64_t)nwords;
    p.C = C;
    p.nblocks = nblocks;
    p.B = B;
    p.nw = nw;
    for (int i = 0; i < nw && i < 8; ++i) p.widths[i] = widths[i];
    if (nblocks == 0) return DM_OK;
    schedule_kernel<<<(unsigned)((nblocks + 3) / 4), 128, 0, (cudaStream_t)stream>>>(p, out);
    return cuda_check(cudaGetLastError(), "schedule_kernel", msg);
}

int launch_split_f32(const float *x, int64_t C, int64_t M, uint16_t *out, void *stream, std::string &msg) {
    int64_t n = M * C;
    split_f32_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(x, C, M, out);
    return cuda_check(cudaGetLastError(), "split_f32_kernel", msg);
}

// bf16 activations at any 2-byte alignment -> a 16-byte aligned copy (the
// sip kernel stages activations with bulk copies, whose source must be
// 16-byte aligned).
__global__ void copy_u16_kernel(const uint16_t *__restrict__ src, int64_t n, uint16_t *__restrict__ dst) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = src[i];
}

int launch_copy_u16(const uint16_t *src, int64_t n, uint16_t *dst, void *stream, std::string &msg) {
    if (n <= 0) return DM_OK;
    const int64_t blocks = std::min<int64_t>((n + 255) / 256, 1184);
    copy_u16_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(src, n, dst);
    return cuda_check(cudaGetLastError(), "copy_u16_kernel", msg);
}

int launch_gemv_raw(const void *w, int64_t R, int64_t C, const void *x, int x_f32, int64_t M, const uint16_t *bias,
                    void *out, int out_f32, void *stream, std::string &msg) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    using Kern = void (*)(const uint16_t *, int64_t, int64_t, const void *, const uint16_t *, void *, int, int);
    static const Kern kernels[2][8] = {
        {gemv_raw_kernel<0, 1>, gemv_raw_kernel<0, 2>, gemv_raw_kernel<0, 3>, gemv_raw_kernel<0, 4>,
         gemv_raw_kernel<0, 5>, gemv_raw_kernel<0, 6>, gemv_raw_kernel<0, 7>, gemv_raw_kernel<0, 8>},
        {gemv_raw_kernel<1, 1>, gemv_raw_kernel<1, 2>, gemv_raw_kernel<1, 3>, gemv_raw_kernel<1, 4>,
         gemv_raw_kernel<1, 5>, gemv_raw_kernel<1, 6>, gemv_raw_kernel<1, 7>, gemv_raw_kernel<1, 8>}};
    if (M < 1 || M > 8) {
        msg = "gemv_raw: 1..8 activation rows";
        return DM_EINVAL;
    }
    // one wave: as many blocks as stay resident on every SM (the blocks loop
    // over rows), no second partial wave
    const Kern kern = kernels[x_f32 ? 1 : 0][M - 1];
    static int resident[2][8] = {};
    int &per_sm = resident[x_f32 ? 1 : 0][M - 1];
    if (per_sm == 0 && cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, 0) != cudaSuccess)
        per_sm = 4;
    const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((R + 7) / 8, (int64_t)sms * std::max(per_sm, 1)));
    // the 16-byte loads need whole 8-weight groups per row and 16-byte aligned
    // weight and activation rows; anything else takes the scalar loop
    const int vec = (C % 8 == 0) && ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(x)) & 15) == 0;
    kern<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const uint16_t *>(w), R, C, x, bias, out, out_f32, vec);
    return cuda_check(cudaGetLastError(), "gemv_raw_kernel", msg);
}

}  // namespace dm
