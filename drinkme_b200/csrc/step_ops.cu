// The small fused operations of a batch-1 decode step around the packed
// Linears (decode_step.DecodeStack; the reference runs transformers' own
// modules there, src/drinkme/serving/cudagraph.py captures them): one
// launch each for the residual add + RMSNorm, the per-head q/k RMSNorm +
// rotary embedding + KV-cache write, grouped-query decode attention over
// the cache (split over the sequence, then combined) and SiLU(gate) * up.
// Every launch reads the position from device memory, so a captured graph
// serves every step. bf16 storage, fp32 arithmetic. Every launch is a
// programmatic dependent launch both ways: each kernel is scheduled while its
// predecessor finishes and waits for it on the device before reading, and
// lets its own successor start early (a sip GEMV stages its first weights
// while these run and waits for them before it reads their output).
#include <cuda_runtime.h>

#include <cmath>
#include <string>

#include "dm_device.cuh"
#include "dm_internal.h"

namespace dm {
namespace {

// Cache rows per attention CTA: a warp walks its chunk's rows in order, so
// the chunk bounds the serial work (32: at position 896 the 8B step took
// 6.77 ms with 128-row chunks).
constexpr int kAttnChunk = 32;

__device__ __forceinline__ float bf(uint16_t b) { return bf16_bits_to_f32(b); }
__device__ __forceinline__ uint16_t to_bf(float f) { return f32_to_bf16_bits(f); }

__device__ __forceinline__ float block_sum(float v, float *red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
    if (l == 0) red[w] = v;
    __syncthreads();
    float s = 0.f;
    for (int i = 0; i < nw; ++i) s += red[i];
    __syncthreads();
    return s;
}

// h <- h + delta (rounded to bf16, as an in-place bf16 add), then
// out = h * rsqrt(mean(h^2) + eps) * w; one CTA, one row.
// Rows of up to kNormReg * blockDim elements keep each thread's elements in
// registers, all of a thread's loads in flight at once (each is an L2 round
// trip), the norm weights fetched before the wait for the predecessor; the
// sum runs in the same element order either way.
constexpr int kNormReg = 8;
__global__ void add_rmsnorm_kernel(uint16_t *h, const uint16_t *delta, const uint16_t *w, uint16_t *out, int n,
                                   float eps) {
    pdl_launch_dependents();  // the next GEMV may stage its weights meanwhile
    __shared__ float red[32];
    const int bd = blockDim.x, t = threadIdx.x;
    const bool regs = n <= kNormReg * bd;
    uint16_t wv[kNormReg];
    if (regs) {
#pragma unroll
        for (int k = 0; k < kNormReg; ++k)
            if (t + k * bd < n) wv[k] = w[t + k * bd];  // a constant: no need to wait for it
    }
    pdl_wait();  // launched early: the producer of this kernel's inputs has finished
    float ss = 0.f, xs[kNormReg];
    if (regs) {
        uint16_t hv[kNormReg], dv[kNormReg];
#pragma unroll
        for (int k = 0; k < kNormReg; ++k)
            if (t + k * bd < n) {
                hv[k] = h[t + k * bd];
                if (delta) dv[k] = delta[t + k * bd];
            }
#pragma unroll
        for (int k = 0; k < kNormReg; ++k)
            if (t + k * bd < n) {
                float x = bf(hv[k]);
                if (delta) {
                    x = bf(to_bf(x + bf(dv[k])));
                    h[t + k * bd] = to_bf(x);
                }
                xs[k] = x;
                ss += x * x;
            }
    } else {
        for (int i = t; i < n; i += bd) {
            float x = bf(h[i]);
            if (delta) {
                x = bf(to_bf(x + bf(delta[i])));
                h[i] = to_bf(x);
            }
            ss += x * x;
        }
    }
    const float r = rsqrtf(block_sum(ss, red) / (float)n + eps);
    __syncthreads();
    if (regs) {
#pragma unroll
        for (int k = 0; k < kNormReg; ++k)
            if (t + k * bd < n) out[t + k * bd] = to_bf(bf(to_bf(xs[k] * r)) * bf(wv[k]));
    } else {
        for (int i = t; i < n; i += bd) out[i] = to_bf(bf(to_bf(bf(h[i]) * r)) * bf(w[i]));
    }
}

// A warp per head of the fused q|k|v row: q and k heads get RMSNorm over
// the head (weights qn / kn) and the rotary embedding at *pos (pairs i,
// i + hd/2); q goes to q_out, k and v to row *pos of the layer's caches
// [max_len][nkv][hd].
__global__ void qk_norm_rope_cache_kernel(const uint16_t *qkv, const uint16_t *qn, const uint16_t *kn,
                                          const float *cosv, const float *sinv, const int64_t *pos, uint16_t *q_out,
                                          uint16_t *kc, uint16_t *vc, int nh, int nkv, int hd, float eps) {
    pdl_launch_dependents();  // the next GEMV may stage its weights meanwhile
    pdl_wait();               // launched early: the producer of this kernel's inputs has finished
    const int head = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (head >= nh + 2 * nkv) return;
    const int64_t p = *pos;
    const uint16_t *src = qkv + (int64_t)head * hd;
    if (head >= nh + nkv) {  // v: copied into the cache row
        uint16_t *dst = vc + (p * nkv + (head - nh - nkv)) * hd;
        for (int i = lane; i < hd; i += 32) dst[i] = src[i];
        return;
    }
    const bool isq = head < nh;
    const uint16_t *wn = isq ? qn : kn;
    const int half = hd / 2;
    float ss = 0.f;
    for (int i = lane; i < hd; i += 32) {
        const float x = bf(src[i]);
        ss += x * x;
    }
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float r = rsqrtf(ss / (float)hd + eps);
    uint16_t *dst = isq ? q_out + (int64_t)head * hd : kc + (p * nkv + (head - nh)) * hd;
    for (int i = lane; i < half; i += 32) {
        // the normed values rounded to bf16 first, as the module stores them
        const float x1 = bf(to_bf(bf(to_bf(bf(src[i]) * r)) * bf(wn[i])));
        const float x2 = bf(to_bf(bf(to_bf(bf(src[i + half]) * r)) * bf(wn[i + half])));
        const float c = cosv[p * half + i], s = sinv[p * half + i];
        dst[i] = to_bf(x1 * c - x2 * s);
        dst[i + half] = to_bf(x2 * c + x1 * s);
    }
}

// The online softmax of one query head (this warp; lane l holds elements
// 4l .. 4l + 3 of q, already scaled) over cache rows [r0, r1) of kv head g:
// the rows are taken in order, one at a time, as a plain loop would, but
// the keys and values of sixteen rows are loaded before their arithmetic (the
// rows were just written: each load is an L2 round trip, which a row-by-row
// loop would wait for once per row).
__device__ __forceinline__ void attend_rows(const float qv[4], const uint16_t *kc, const uint16_t *vc, int64_t r0,
                                            int64_t r1, int nkv, int g, int hd, int lane, float &m, float &l,
                                            float acc[4]) {
    constexpr int kAhead = 16;
    for (int64_t rb = r0; rb < r1; rb += kAhead) {
        uint2 kk[kAhead], vv[kAhead];
#pragma unroll
        for (int u = 0; u < kAhead; ++u) {
            const int64_t r = rb + u < r1 ? rb + u : r1 - 1;  // in bounds; unused past r1
            kk[u] = *reinterpret_cast<const uint2 *>(kc + (r * nkv + g) * hd + lane * 4);
            vv[u] = *reinterpret_cast<const uint2 *>(vc + (r * nkv + g) * hd + lane * 4);
        }
#pragma unroll
        for (int u = 0; u < kAhead; ++u) {
            if (rb + u >= r1) break;
            const float k4[4] = {bf(kk[u].x & 0xffffu), bf(kk[u].x >> 16), bf(kk[u].y & 0xffffu), bf(kk[u].y >> 16)};
            const float v4[4] = {bf(vv[u].x & 0xffffu), bf(vv[u].x >> 16), bf(vv[u].y & 0xffffu), bf(vv[u].y >> 16)};
            float s = 0.f;
            for (int e = 0; e < 4; ++e) s += qv[e] * k4[e];
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            const float mn = fmaxf(m, s);
            const float a = __expf(m - mn), b = __expf(s - mn);
            for (int e = 0; e < 4; ++e) acc[e] = acc[e] * a + b * v4[e];
            l = l * a + b;
            m = mn;
        }
    }
}

// Split decode attention: CTA (kv head g, chunk j) covers cache rows
// [32 j, 32 j + 32) below *pos + 1; a warp per query head of the group
// keeps a running max, sum and weighted value sum, written to
// part[head][j] = {m, l, acc[hd]}.
__global__ void attn_split_kernel(const uint16_t *q, const uint16_t *kc, const uint16_t *vc, const int64_t *pos,
                                  float *part, int nh, int nkv, int hd, int nchunks, float scale) {
    pdl_launch_dependents();  // the next GEMV may stage its weights meanwhile
    pdl_wait();               // launched early: the producer of this kernel's inputs has finished
    const int g = blockIdx.x, j = blockIdx.y, lane = threadIdx.x & 31, wq = threadIdx.x >> 5;
    const int grp = nh / nkv;
    if (wq >= grp) return;
    const int head = g * grp + wq;
    const int64_t live = *pos + 1;
    const int64_t r0 = (int64_t)j * kAttnChunk, r1 = min(live, r0 + kAttnChunk);
    float qv[4], acc[4];
    const int per = hd / 32;  // 4 at hd = 128
    for (int e = 0; e < per; ++e) {
        qv[e] = bf(q[(int64_t)head * hd + lane * per + e]) * scale;
        acc[e] = 0.f;
    }
    float m = -INFINITY, l = 0.f;
    attend_rows(qv, kc, vc, r0, r1, nkv, g, hd, lane, m, l, acc);
    float *out = part + ((int64_t)head * nchunks + j) * (hd + 2);
    if (lane == 0) {
        out[0] = m;
        out[1] = l;
    }
    for (int e = 0; e < per; ++e) out[2 + lane * per + e] = acc[e];
}

// The partial softmaxes {m, l, acc[hd]} of chunks [0, used) of one head
// combined by one warp (lane l owns elements 4l .. 4l + 3) into the head's
// bf16 output: the chunks folded in order with a running maximum, the
// partials of eight chunks loaded at once (L2 round trips). Both attention
// routes combine through this function, so their results are the same bits.
__device__ __forceinline__ void combine_chunks(const float *ph, int used, int hd, int lane, uint16_t *outp) {
    float M = -INFINITY, L = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
    for (int c0 = 0; c0 < used; c0 += 8) {
        float mc[8], lc[8], ac[8][4];
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (c0 + u < used) {
                const float *pc = ph + (int64_t)(c0 + u) * (hd + 2);
                mc[u] = __ldcg(pc);
                lc[u] = __ldcg(pc + 1);
                for (int e = 0; e < 4; ++e) ac[u][e] = __ldcg(pc + 2 + lane * 4 + e);
            }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            if (c0 + u >= used) break;
            if (lc[u] == 0.f) continue;
            const float Mn = fmaxf(M, mc[u]);
            const float so = __expf(M - Mn), sn = __expf(mc[u] - Mn);
            L = L * so + lc[u] * sn;
            for (int e = 0; e < 4; ++e) o[e] = o[e] * so + ac[u][e] * sn;
            M = Mn;
        }
    }
    for (int e = 0; e < 4; ++e) outp[lane * 4 + e] = to_bf(o[e] / L);
}

// A warp per query head: the chunks' partial softmaxes combined.
__global__ void attn_combine_kernel(const float *part, const int64_t *pos, uint16_t *out, int nh, int hd,
                                    int nchunks) {
    pdl_launch_dependents();  // the next GEMV may stage its weights meanwhile
    pdl_wait();               // launched early: the producer of this kernel's inputs has finished
    const int head = blockIdx.x, lane = threadIdx.x;
    const int used = (int)min((int64_t)nchunks, (*pos + kAttnChunk) / kAttnChunk);
    combine_chunks(part + (int64_t)head * nchunks * (hd + 2), used, hd, lane, out + (int64_t)head * hd);
}

// The whole attention block of a layer in one launch: CTA (kv head g, chunk
// j), a warp per query head of the group. Each warp norms and rotates its q
// head from the fused q|k|v row; the CTA whose chunk holds *pos also norms
// and rotates k and writes k and v into row *pos of the caches first; every
// CTA with live rows then runs its chunk of the split attention; the last
// CTA of kv head g to finish (a counter of the live chunks, which it resets)
// combines the chunks for the group. With one live chunk (*pos < 32) that
// chunk's CTA writes the result itself.
__global__ void attn_block_kernel(const uint16_t *qkv, const uint16_t *qn, const uint16_t *kn, const float *cosv,
                                  const float *sinv, const int64_t *pos, uint16_t *kc, uint16_t *vc, float *part,
                                  unsigned int *count, uint16_t *out, int nh, int nkv, int hd, int nchunks, float eps,
                                  float scale) {
    pdl_launch_dependents();
    __shared__ int last;
    const int g = blockIdx.x, j = blockIdx.y, lane = threadIdx.x & 31, wq = threadIdx.x >> 5;
    const int grp = nh / nkv, half = hd / 2, per = hd / 32;
    // what does not depend on the kernel before this one, fetched before the
    // wait for it: the position (advanced between steps, before the step's
    // first kernel), the norm weights and the rotary row of this lane's
    // elements
    const int64_t p = *pos, live = p + 1;
    // chunks past the live rows have nothing to do: they leave at once and
    // are not counted (the count below waits for the live chunks)
    const int used = (int)min((int64_t)nchunks, (p + kAttnChunk) / kAttnChunk);
    if (j >= used) return;
    float wq4[4], wk4[4], c4[4], s4[4];
    for (int e = 0; e < per; ++e) {
        const int idx = lane * per + e, i = idx < half ? idx : idx - half;
        wq4[e] = bf(qn[idx]);
        wk4[e] = bf(kn[idx]);
        c4[e] = cosv[p * half + i];
        s4[e] = sinv[p * half + i];
    }
    pdl_wait();
    // rotate-half pairs: lane l holds elements l*per .. l*per+3; the partner
    // of element e is e +- hd/2, held by lane (l +- 16)
    auto norm_rope = [&](const uint16_t *src, const float wn[4], float v[4]) {
        // the sum of squares in qk_norm_rope_cache_kernel's order (lane l
        // adds elements l, l + 32, ...), so that the bits match it
        float ss = 0.f;
        for (int i = lane; i < hd; i += 32) {
            const float x = bf(src[i]);
            ss += x * x;
        }
        for (int e = 0; e < per; ++e) v[e] = bf(src[lane * per + e]);
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float r = rsqrtf(ss / (float)hd + eps);
        for (int e = 0; e < per; ++e) v[e] = bf(to_bf(bf(to_bf(v[e] * r)) * wn[e]));
        // rotate-half: the partner of element e (lane l) sits in lane l ^ 16
        float o4[4];
        for (int e = 0; e < per; ++e) {
            const int idx = lane * per + e;
            const float partner = __shfl_xor_sync(0xffffffffu, v[e], 16);
            const float c = c4[e], sn = s4[e];
            o4[e] = idx < half ? v[e] * c - partner * sn : v[e] * c + partner * sn;
        }
        for (int e = 0; e < per; ++e) v[e] = bf(to_bf(o4[e]));
    };
    const int head = g * grp + wq;
    float qv[4];
    norm_rope(qkv + (int64_t)head * hd, wq4, qv);
    const int64_t r0 = (int64_t)j * kAttnChunk, r1 = min(live, r0 + kAttnChunk);
    if (p >= r0 && p < r0 + kAttnChunk && wq == 0) {  // this chunk holds the new row
        float kv4[4];
        norm_rope(qkv + (int64_t)(nh + g) * hd, wk4, kv4);
        uint16_t *kd = kc + (p * nkv + g) * hd, *vd = vc + (p * nkv + g) * hd;
        const uint16_t *vs = qkv + (int64_t)(nh + nkv + g) * hd;
        for (int e = 0; e < per; ++e) {
            kd[lane * per + e] = to_bf(kv4[e]);
            vd[lane * per + e] = vs[lane * per + e];
        }
    }
    __syncthreads();
    float acc[4] = {0.f, 0.f, 0.f, 0.f}, m = -INFINITY, l = 0.f;
    for (int e = 0; e < per; ++e) qv[e] *= scale;
    attend_rows(qv, kc, vc, r0, r1, nkv, g, hd, lane, m, l, acc);
    if (used == 1) {
        // one live chunk: its softmax is the result — the combine's
        // arithmetic over one chunk, written directly (same bits), with no
        // partials, fence, count or combine
        const float a = __expf(m - fmaxf(-INFINITY, m));
        float o4[4] = {0.f, 0.f, 0.f, 0.f}, L = 0.f;
        L += a * l;
        for (int e = 0; e < per; ++e) o4[e] += a * acc[e];
        for (int e = 0; e < per; ++e) out[(int64_t)head * hd + lane * per + e] = to_bf(o4[e] / L);
        return;
    }
    float *pp = part + ((int64_t)head * nchunks + j) * (hd + 2);
    if (lane == 0) {
        pp[0] = m;
        pp[1] = l;
    }
    for (int e = 0; e < per; ++e) pp[2 + lane * per + e] = acc[e];
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned int old = atomicAdd(count + g, 1u);
        last = old == (unsigned int)(used - 1);
        if (last) count[g] = 0u;  // for the next launch
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    combine_chunks(part + (int64_t)head * nchunks * (hd + 2), used, hd, lane, out + (int64_t)head * hd);
}

__global__ void silu_mul_kernel(const uint16_t *gu, uint16_t *out, int n) {
    pdl_launch_dependents();  // the next GEMV may stage its weights meanwhile
    pdl_wait();               // launched early: the producer of this kernel's inputs has finished
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float g = bf(gu[i]), u = bf(gu[n + i]);
    out[i] = to_bf(g / (1.f + __expf(-g)) * u);
}

int launched(const char *what, std::string &msg) {
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) return DM_OK;
    msg = std::string(what) + ": " + cudaGetErrorString(e);
    return DM_ECUDA;
}

// Every launch here lets the kernel start while its predecessor finishes
// (programmatic dependent launch; the kernel waits for it on the device
// before reading anything).
template <typename... Params, typename... Args>
cudaError_t launch_pdl(void (*kern)(Params...), dim3 grid, dim3 block, void *stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<Params>(args)...);
}

}  // namespace
}  // namespace dm

extern "C" int dm_step_add_rmsnorm(void *h, const void *delta, const void *w, void *out, int64_t n, float eps,
                                   void *stream, char *err, size_t err_len) {
    if (!h || !w || !out || n < 1 || n > (1 << 20)) {
        dm::set_error(err, err_len, "dm_step_add_rmsnorm: bad arguments");
        return DM_EINVAL;
    }
    dm::launch_pdl(dm::add_rmsnorm_kernel, dim3(1), dim3(1024), stream, (uint16_t *)h, (const uint16_t *)delta,
                   (const uint16_t *)w, (uint16_t *)out, (int)n, eps);
    std::string msg;
    int rc = dm::launched("add_rmsnorm_kernel", msg);
    if (rc) dm::set_error(err, err_len, msg);
    return rc;
}

extern "C" int dm_step_qk_rope_cache(const void *qkv, const void *qn, const void *kn, const float *cosv,
                                     const float *sinv, const int64_t *pos, void *q_out, void *kcache, void *vcache,
                                     int32_t nh, int32_t nkv, int32_t hd, float eps, void *stream, char *err,
                                     size_t err_len) {
    if (!qkv || !qn || !kn || !cosv || !sinv || !pos || !q_out || !kcache || !vcache || nh < 1 || nkv < 1 ||
        nh % nkv || hd != 128) {
        dm::set_error(err, err_len, "dm_step_qk_rope_cache: bad arguments (head_dim 128)");
        return DM_EINVAL;
    }
    const int heads = nh + 2 * nkv, per = 4;
    dm::launch_pdl(dm::qk_norm_rope_cache_kernel, dim3((heads + per - 1) / per), dim3(32 * per), stream,
                   (const uint16_t *)qkv, (const uint16_t *)qn, (const uint16_t *)kn, cosv, sinv, pos,
                   (uint16_t *)q_out, (uint16_t *)kcache, (uint16_t *)vcache, nh, nkv, hd, eps);
    std::string msg;
    int rc = dm::launched("qk_norm_rope_cache_kernel", msg);
    if (rc) dm::set_error(err, err_len, msg);
    return rc;
}

extern "C" int64_t dm_step_attention_workspace_bytes(int32_t nh, int32_t hd, int64_t max_len) {
    const int64_t nchunks = (max_len + dm::kAttnChunk - 1) / dm::kAttnChunk;
    return (int64_t)nh * nchunks * (hd + 2) * 4;
}

extern "C" int dm_step_attention(const void *q, const void *kcache, const void *vcache, const int64_t *pos,
                                 int64_t max_len, void *out, float *work, int32_t nh, int32_t nkv, int32_t hd,
                                 void *stream, char *err, size_t err_len) {
    if (!q || !kcache || !vcache || !pos || !out || !work || nh < 1 || nkv < 1 || nh % nkv || hd != 128 ||
        nh / nkv > 32 || max_len < 1) {
        dm::set_error(err, err_len, "dm_step_attention: bad arguments (head_dim 128, up to 32 heads per kv head)");
        return DM_EINVAL;
    }
    const int nchunks = (int)((max_len + dm::kAttnChunk - 1) / dm::kAttnChunk);
    cudaStream_t s = (cudaStream_t)stream;
    dm::launch_pdl(dm::attn_split_kernel, dim3(nkv, nchunks), dim3(32 * (nh / nkv)), s, (const uint16_t *)q,
                   (const uint16_t *)kcache, (const uint16_t *)vcache, pos, work, nh, nkv, hd, nchunks,
                   1.0f / sqrtf((float)hd));
    dm::launch_pdl(dm::attn_combine_kernel, dim3(nh), dim3(32), s, (const float *)work, pos, (uint16_t *)out, nh,
                   hd, nchunks);
    std::string msg;
    int rc = dm::launched("attention kernels", msg);
    if (rc) dm::set_error(err, err_len, msg);
    return rc;
}

extern "C" int64_t dm_step_attention_block_workspace_bytes(int32_t nh, int32_t nkv, int32_t hd, int64_t max_len) {
    return (dm_step_attention_workspace_bytes(nh, hd, max_len) + 255) / 256 * 256 + (int64_t)nkv * 4;
}

extern "C" int dm_step_attention_block(const void *qkv, const void *qn, const void *kn, const float *cos_table,
                                       const float *sin_table, const int64_t *pos, void *kcache, void *vcache,
                                       int64_t max_len, void *out, void *work, int32_t nh, int32_t nkv, int32_t hd,
                                       float eps, void *stream, char *err, size_t err_len) {
    if (!qkv || !qn || !kn || !cos_table || !sin_table || !pos || !kcache || !vcache || !out || !work || nh < 1 ||
        nkv < 1 || nh % nkv || hd != 128 || nh / nkv > 32 || max_len < 1) {
        dm::set_error(err, err_len, "dm_step_attention_block: bad arguments (head_dim 128, up to 32 heads per kv head)");
        return DM_EINVAL;
    }
    const int nchunks = (int)((max_len + dm::kAttnChunk - 1) / dm::kAttnChunk);
    float *part = reinterpret_cast<float *>(work);
    unsigned int *count = reinterpret_cast<unsigned int *>(
        reinterpret_cast<uint8_t *>(work) + (dm_step_attention_workspace_bytes(nh, hd, max_len) + 255) / 256 * 256);
    dm::launch_pdl(dm::attn_block_kernel, dim3(nkv, nchunks), dim3(32 * (nh / nkv)), stream, (const uint16_t *)qkv,
                   (const uint16_t *)qn, (const uint16_t *)kn, cos_table, sin_table, pos, (uint16_t *)kcache,
                   (uint16_t *)vcache, part, count, (uint16_t *)out, nh, nkv, hd, nchunks, eps,
                   1.0f / sqrtf((float)hd));
    std::string msg;
    int rc = dm::launched("attn_block_kernel", msg);
    if (rc) dm::set_error(err, err_len, msg);
    return rc;
}

extern "C" int dm_step_silu_mul(const void *gu, void *out, int64_t n, void *stream, char *err, size_t err_len) {
    if (!gu || !out || n < 1 || n > INT32_MAX) {
        dm::set_error(err, err_len, "dm_step_silu_mul: bad arguments");
        return DM_EINVAL;
    }
    dm::launch_pdl(dm::silu_mul_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), stream, (const uint16_t *)gu,
                   (uint16_t *)out, (int)n);
    std::string msg;
    int rc = dm::launched("silu_mul_kernel", msg);
    if (rc) dm::set_error(err, err_len, msg);
    return rc;
}
