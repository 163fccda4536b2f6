// The sip fast path on sm_100a: fused radix decode + GEMV for 1..8
// activation rows, 1024-weight blocks, rows of whole blocks.
//
// Reference: the M=1 `_gemv` + `_finish` (src/drinkme/codec/radix_kernel_gpu.py:
// 683-718) and the multi-column `_gemv_mc` (radix_ops.py:92-164) with the
// lean sip decoder (radix_kernel_gpu.py:103-235). The result contract is
// theirs: fp32 accumulate, the bias added in fp32, one rounding; each
// activation row's result independent of the others.
//
// Design (B200-first):
//   * A CTA = 1 producer warp + NC consumer warps. Each consumer warp is a
//     WORKER owning a contiguous range of units (8 rows x 1 block column,
//     see layout.cpp); the units of all workers of the grid cover the tensor
//     in tile-major order, split evenly (stream-K).
//   * The producer stages each unit with ONE 1-D bulk copy (the TMA engine)
//     plus one 2 KB bulk copy per activation row of the unit's block column,
//     into a per-worker ring of shared-memory slots, completing an mbarrier.
//   * A consumer decodes its unit straight into MMA operands: the weights
//     are the B operand (n = 8 output rows) of mma.m16n8k16 bf16 with fp32
//     accumulate, the activations the A operand (rows 0..7 = up to 8
//     activation rows, rows 8..15 zero). Lane (g, t) decodes row g of the
//     unit at k = 64q + 16t + [0, 16) for q = 0..15.
//   * Decode is byte-parallel: the 3-bit tier-0 codes are spread into
//     nibbles with three AND + IMAD steps (the IMADs run on the FMA pipe,
//     idle otherwise), then one PRMT per 4 weights looks four exponents up
//     in an 8-byte table, and two LOP3 + two PRMT merge sign, exponent and
//     mantissa into the bf16 pairs of the MMA operand. The table's escape
//     entry makes a weight whose code is 7 decode to exactly +0.
//   * Escaped weights (about 2% of a N(0, 0.02) tensor) are added back as
//     fp32 corrections: the loader's escape index lists each block's escape
//     positions; lane (g, t) handles every fourth escape of row g.
//   * A worker accumulates a tile's units in registers (each unit's MMA chain
//     starts from zero; unit sums are added in unit order). A tile covered
//     by one worker is written directly; a tile split across workers goes
//     through scratch: each contributor writes its partial, the last to
//     arrive (an atomic counter that it resets) sums them in worker order and
//     writes the output. Every sum has a fixed order, so results are
//     deterministic and activation row m of an M-row call is bitwise the M=1
//     call on row m.
#include <cuda_runtime.h>

#include <algorithm>
#include <string>

#include "dm_device.cuh"
#include "dm_internal.h"

namespace dm {

struct SipArgs {
    const uint8_t *data;
    const uint32_t *unit16;
    int64_t units, rows, NB;
    uint32_t th0, th1, tl0, tl1;  // exponent lookup tables (high / low part)
    const uint16_t *x;            // virtual activation rows [Mv][x_stride] bf16
    int64_t x_stride;
    int32_t Mv, nsplit, M_out;
    const uint16_t *bias;
    void *out;
    int32_t out_f32;
    float *partials;
    int *counters;
    int *err;
    int32_t slot_bytes, x_off, spw, nc, workers;
};

constexpr int kMaxConsumers = 8;

__device__ __forceinline__ int64_t range_start(int64_t w, int64_t U, int64_t W) { return (w * U) / W; }
__device__ __forceinline__ int64_t worker_of(int64_t u, int64_t U, int64_t W) { return ((u + 1) * W + U - 1) / U - 1; }

// 8 three-bit codes (bits 0..23 of v, upper bits zero) -> nibble k holds code
// k in its bits 0..2 with bit 3 clear: a PRMT selector per 4 codes.
__device__ __forceinline__ uint32_t spread_codes(uint32_t v) {
    uint32_t x = v;
    x += 15u * (x & 0x00FFF000u);  // codes 4..7 up by 4 bits
    x += 3u * (x & 0x0FC00FC0u);   // codes 2,3 and 6,7 up by 2
    x += (x & 0x38383838u);        // codes 1,3,5,7 up by 1
    return x;
}

// Four weights: literal word L (4 literal bytes), selector S (4 codes in
// nibbles) -> two bf16 pairs {w0, w1}, {w2, w3}.
__device__ __forceinline__ void decode4(uint32_t L, uint32_t S, uint32_t th0, uint32_t th1, uint32_t tl0,
                                        uint32_t tl1, uint32_t &p01, uint32_t &p23) {
    const uint32_t eh = __byte_perm(th0, th1, S);  // exponent >> 1 (0x80 marks an escape)
    const uint32_t el = __byte_perm(tl0, tl1, S);  // (exponent & 1) << 7 (0x7F for an escape)
    // high byte: bit 7 = sign unless escaped, bits 0..6 = exponent >> 1
    const uint32_t hi = lop3<0x64>(L, eh, 0x80808080u);
    // low byte: bit 7 = exponent & 1, bits 0..6 = mantissa unless escaped
    const uint32_t lo = lop3<0x98>(L, el, 0x80808080u);
    p01 = __byte_perm(lo, hi, 0x5140);
    p23 = __byte_perm(lo, hi, 0x7362);
}

__device__ void store_outputs(const SipArgs &a, int64_t tile, const float (*P)[kMaxVirtualRows]) {
    const int lane = threadIdx.x & 31;
    for (int o = lane; o < kUnitRows * a.M_out; o += 32) {
        const int r = o % kUnitRows, m = o / kUnitRows;
        const int64_t row = tile * kUnitRows + r;
        if (row >= a.rows) continue;
        float y = P[r][m * a.nsplit];
        for (int s = 1; s < a.nsplit; ++s) y += P[r][m * a.nsplit + s];
        if (a.bias) y += bf16_bits_to_f32(a.bias[row]);
        if (a.out_f32)
            reinterpret_cast<float *>(a.out)[m * a.rows + row] = y;
        else
            reinterpret_cast<uint16_t *>(a.out)[m * a.rows + row] = f32_to_bf16_bits(y);
    }
}

__global__ void __launch_bounds__(32 * (1 + kMaxConsumers), 1) sip_gemv_kernel(SipArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nslots = a.nc * a.spw;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)nslots * a.slot_bytes);
    uint64_t *empty = full + nslots;
    float *xch = reinterpret_cast<float *>(empty + nslots);  // [nc][8][8] exchange per consumer
    if (threadIdx.x == 0) {
        for (int s = 0; s < nslots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_fence_init();
    }
    __syncthreads();
    const int64_t U = a.units, W = a.workers, NB = a.NB;

    if (warp == 0) {
        // ---------------------------------------------------- producer --
        if (lane == 0) {
            bool ok = true;
            int64_t issued[kMaxConsumers];
            for (int c = 0; c < a.nc; ++c) issued[c] = 0;
            for (int64_t round = 0; ok; ++round) {
                bool any = false;
                for (int c = 0; c < a.nc && ok; ++c) {
                    const int64_t w = (int64_t)blockIdx.x * a.nc + c;
                    const int64_t u0 = range_start(w, U, W), u1 = range_start(w + 1, U, W);
                    if (u0 + round >= u1) continue;
                    any = true;
                    const int64_t u = u0 + round;
                    const int slot = c * a.spw + (int)(round % a.spw);
                    const int64_t use = round / a.spw;
                    if (use > 0 && !mbar_wait(&empty[slot], (uint32_t)((use - 1) & 1), a.err, kErrWaitEmpty)) {
                        ok = false;
                        break;
                    }
                    const uint32_t q0 = a.unit16[u], q1 = a.unit16[u + 1];
                    const uint32_t ubytes = (q1 - q0) * 16u;
                    uint8_t *dst = smem + (size_t)slot * a.slot_bytes;
                    mbar_arrive_expect_tx(&full[slot], ubytes + (uint32_t)a.Mv * 2048u);
                    bulk_g2s(dst, a.data + (size_t)q0 * 16, ubytes, &full[slot]);
                    const int64_t b = u % NB;
                    for (int v = 0; v < a.Mv; ++v)
                        bulk_g2s(dst + a.x_off + v * kXRowStride, a.x + v * a.x_stride + b * 1024, 2048u,
                                 &full[slot]);
                    issued[c] = round + 1;
                }
                if (!any) break;
            }
            // drain: every copy this producer issued lands before the CTA exits
            for (int c = 0; c < a.nc; ++c) {
                for (int k = 0; k < a.spw; ++k) {
                    // the last round that used slot (c, k)
                    int64_t last = -1;
                    for (int64_t r = issued[c] - 1; r >= 0 && r >= issued[c] - a.spw; --r)
                        if (r % a.spw == k) { last = r; break; }
                    if (last < 0) continue;
                    const int slot = c * a.spw + k;
                    mbar_wait(&full[slot], (uint32_t)((last / a.spw) & 1), a.err, kErrWaitDrain);
                }
            }
        }
        return;
    }

    // ------------------------------------------------------- consumers --
    const int c = warp - 1;
    const int64_t w = (int64_t)blockIdx.x * a.nc + c;
    const int64_t u0 = range_start(w, U, W), u1 = range_start(w + 1, U, W);
    const int g = lane >> 2, t = lane & 3;
    const uint32_t th0 = a.th0, th1 = a.th1, tl0 = a.tl0, tl1 = a.tl1;
    const int Mv = a.Mv;
    float (*X)[kMaxVirtualRows] = reinterpret_cast<float (*)[kMaxVirtualRows]>(xch + c * 64);

    float acc0 = 0.f, acc1 = 0.f;  // D[batch g][rows 2t, 2t+1], summed over the tile's units
    float corr[kMaxVirtualRows];   // row g's escape corrections per virtual activation row
#pragma unroll
    for (int v = 0; v < kMaxVirtualRows; ++v) corr[v] = 0.f;
    int64_t tile = u0 / NB;
    const int64_t first_tile = u0 / NB, last_tile = (u1 - 1) / NB;

    auto flush = [&](int64_t tl) {
        // corrections: sum over the row's four lanes, then hand each to the
        // lane holding D[batch][row]
#pragma unroll
        for (int v = 0; v < kMaxVirtualRows; ++v) {
            float s = corr[v];
            s += __shfl_xor_sync(0xffffffffu, s, 1);
            s += __shfl_xor_sync(0xffffffffu, s, 2);
            corr[v] = s;
        }
        __syncwarp();
        if (t == 0) {
#pragma unroll
            for (int v = 0; v < kMaxVirtualRows; ++v) X[g][v] = corr[v];
        }
        __syncwarp();
        float y0 = 0.f, y1 = 0.f;
        if (g < Mv) {
            y0 = acc0 + X[2 * t][g];
            y1 = acc1 + X[2 * t + 1][g];
        }
        __syncwarp();
        // the tile's partial P[row][virtual row]
#pragma unroll
        for (int v = 0; v < kMaxVirtualRows; ++v) X[g][v] = 0.f;
        __syncwarp();
        if (g < Mv) {
            X[2 * t][g] = y0;
            X[2 * t + 1][g] = y1;
        }
        __syncwarp();
        const bool whole = tl * NB >= u0 && (tl + 1) * NB <= u1;
        if (whole) {
            store_outputs(a, tl, X);
        } else {
            const int slot = (tl == first_tile) ? 0 : 1;
            float *mine = a.partials + (w * 2 + slot) * 64;
            mine[lane] = X[lane / 8][lane % 8];
            mine[lane + 32] = X[4 + lane / 8][lane % 8];
            __threadfence();
            __syncwarp();
            int last = 0;
            if (lane == 0) {
                const int64_t wf = worker_of(tl * NB, U, W), wl = worker_of((tl + 1) * NB - 1, U, W);
                const int n = (int)(wl - wf + 1);
                const int old = atomicAdd(&a.counters[tl], 1);
                last = (old == n - 1);
                if (last) {
                    __threadfence();
                    a.counters[tl] = 0;
                }
            }
            last = __shfl_sync(0xffffffffu, last, 0);
            if (last) {
                __threadfence();
                const int64_t wf = worker_of(tl * NB, U, W), wl = worker_of((tl + 1) * NB - 1, U, W);
                float s0 = 0.f, s1 = 0.f;
                for (int64_t j = wf; j <= wl; ++j) {
                    const int64_t j0 = range_start(j, U, W);
                    const int sj = (tl == j0 / NB) ? 0 : 1;
                    const float *pp = a.partials + (j * 2 + sj) * 64;
                    s0 += __ldcg(pp + lane);
                    s1 += __ldcg(pp + lane + 32);
                }
                __syncwarp();
                X[lane / 8][lane % 8] = s0;
                X[4 + lane / 8][lane % 8] = s1;
                __syncwarp();
                store_outputs(a, tl, X);
            }
        }
        __syncwarp();
        acc0 = acc1 = 0.f;
#pragma unroll
        for (int v = 0; v < kMaxVirtualRows; ++v) corr[v] = 0.f;
    };

    bool ok = true;
    for (int64_t u = u0; u < u1; ++u) {
        const int64_t k = u - u0;
        const int slot = c * a.spw + (int)(k % a.spw);
        if (!mbar_wait(&full[slot], (uint32_t)((k / a.spw) & 1), a.err, kErrWaitFull)) {
            ok = false;
            break;
        }
        const int64_t ut = u / NB;
        if (ut != tile) {
            flush(tile);
            tile = ut;
        }
        const uint8_t *base = smem + (size_t)slot * a.slot_bytes;
        const RowEntry e = reinterpret_cast<const RowEntry *>(base)[g];
        const uint8_t *lit = base + (size_t)e.off16 * 16;
        const uint32_t *tier0 = reinterpret_cast<const uint32_t *>(lit + 1024);
        const uint8_t *xs = base + a.x_off;
        const uint8_t *xg = xs + g * kXRowStride;
        const uint32_t sh = (t & 1) ? 16u : 0u;
        float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll 2
        for (int q = 0; q < 16; ++q) {
            const uint4 L = *reinterpret_cast<const uint4 *>(lit + 64 * q + 16 * t);
            const int wi = (192 * q + 48 * t) >> 5;
            const uint32_t w0 = tier0[wi], w1 = tier0[wi + 1];
            const uint32_t lo32 = __funnelshift_r(w0, w1, sh);
            const uint32_t hi = w1 >> sh;
            const uint32_t xa = spread_codes(lo32 & 0x00FFFFFFu);
            const uint32_t xb = spread_codes(__funnelshift_r(lo32, hi, 24) & 0x00FFFFFFu);
            uint32_t b0[4], b1[4];
            decode4(L.x, xa, th0, th1, tl0, tl1, b0[0], b1[0]);
            decode4(L.y, xa >> 16, th0, th1, tl0, tl1, b0[1], b1[1]);
            decode4(L.z, xb, th0, th1, tl0, tl1, b0[2], b1[2]);
            decode4(L.w, xb >> 16, th0, th1, tl0, tl1, b0[3], b1[3]);
            uint4 X0 = make_uint4(0, 0, 0, 0), X1 = make_uint4(0, 0, 0, 0);
            if (g < Mv) {
                X0 = *reinterpret_cast<const uint4 *>(xg + 128 * q + 32 * t);
                X1 = *reinterpret_cast<const uint4 *>(xg + 128 * q + 32 * t + 16);
            }
            mma_bf16_16816(d0, d1, d2, d3, X0.x, 0u, X0.y, 0u, b0[0], b1[0]);
            mma_bf16_16816(d0, d1, d2, d3, X0.z, 0u, X0.w, 0u, b0[1], b1[1]);
            mma_bf16_16816(d0, d1, d2, d3, X1.x, 0u, X1.y, 0u, b0[2], b1[2]);
            mma_bf16_16816(d0, d1, d2, d3, X1.z, 0u, X1.w, 0u, b0[3], b1[3]);
        }
        // escapes of row g: every fourth one, from lane t
        const int ne = e.nesc;
        if (ne) {
            const uint8_t *term = lit + 1408;
            const uint16_t *idx = reinterpret_cast<const uint16_t *>(lit + (((uint32_t)e.words * 4u + 15u) & ~15u));
            for (int j = t; j < ne; j += 4) {
                const uint32_t pos = idx[j];
                const uint32_t ex = term[j];
                const uint32_t lb = lit[pos];
                const float wv = __uint_as_float(((lb & 0x80u) << 24) | (ex << 23) | ((lb & 0x7Fu) << 16));
#pragma unroll
                for (int v = 0; v < kMaxVirtualRows; ++v) {
                    if (v < Mv) {
                        const uint32_t xb16 = *reinterpret_cast<const uint16_t *>(xs + v * kXRowStride + pos * 2);
                        corr[v] = fmaf(bf16_bits_to_f32(xb16), wv, corr[v]);
                    }
                }
            }
        }
        acc0 += d0;
        acc1 += d1;
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
    }
    if (ok && u1 > u0) flush(tile);
    (void)last_tile;
}

// Shared-memory plan for a launch: slot size, slots per consumer, consumers.
int sip_shared_bytes(const dm_tensor *t, int Mv, int *slot_bytes, int *spw, int *nc) {
    const int unit = (t->L.max_unit_bytes + 127) & ~127;
    const int sb = unit + Mv * kXRowStride;
    const int budget = 227 * 1024;
    for (int c = kMaxConsumers; c >= 1; c /= 2) {
        for (int s = 3; s >= 2; --s) {
            int need = c * s * (sb + 16) + c * 64 * 4 + 128;
            if (need <= budget) {
                *slot_bytes = sb;
                *spw = s;
                *nc = c;
                return need;
            }
        }
    }
    return -1;
}

int launch_gemv_sip(const dm_tensor *t, const uint16_t *xv, int64_t x_stride, int Mv, int nsplit, int M_out,
                    const uint16_t *bias, void *out, int out_f32, void *stream, std::string &msg) {
    int slot_bytes = 0, spw = 0, nc = 0;
    int smem = sip_shared_bytes(t, Mv, &slot_bytes, &spw, &nc);
    if (smem < 0) {
        msg = "sip kernel: a unit does not fit in shared memory";
        return DM_EINVAL;
    }
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(sip_gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) {
            msg = std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e);
            return DM_ECUDA;
        }
        attr_set = true;
    }
    const dm::TensorLayout &L = t->L;
    // one CTA per SM; every worker (consumer warp) owns at least one unit
    int64_t grid, workers;
    if (L.units >= (int64_t)t->sms * nc) {
        grid = t->sms;
    } else {
        grid = std::min<int64_t>(t->sms, L.units);
        nc = (int)std::max<int64_t>(1, std::min<int64_t>(nc, L.units / grid));
    }
    workers = grid * nc;
    if (workers > t->S.max_workers) {
        msg = "sip kernel: scratch sized for fewer workers";
        return DM_EINVAL;
    }
    SipArgs a{};
    a.data = t->d_data;
    a.unit16 = t->d_unit16;
    a.units = L.units;
    a.rows = L.rows;
    a.NB = L.NB;
    uint8_t th[8], tl[8];
    for (int c = 0; c < 7; ++c) {
        th[c] = (uint8_t)(L.palette[c] >> 1);
        tl[c] = (uint8_t)((L.palette[c] & 1u) << 7);
    }
    th[7] = 0x80;  // escape marker: zeroes the sign in the high byte
    tl[7] = 0x7F;  // escape: zeroes the mantissa in the low byte
    a.th0 = th[0] | (th[1] << 8) | (th[2] << 16) | ((uint32_t)th[3] << 24);
    a.th1 = th[4] | (th[5] << 8) | (th[6] << 16) | ((uint32_t)th[7] << 24);
    a.tl0 = tl[0] | (tl[1] << 8) | (tl[2] << 16) | ((uint32_t)tl[3] << 24);
    a.tl1 = tl[4] | (tl[5] << 8) | (tl[6] << 16) | ((uint32_t)tl[7] << 24);
    a.x = xv;
    a.x_stride = x_stride;
    a.Mv = Mv;
    a.nsplit = nsplit;
    a.M_out = M_out;
    a.bias = bias;
    a.out = out;
    a.out_f32 = out_f32;
    a.partials = t->S.partials;
    a.counters = t->S.counters;
    a.err = t->S.err;
    a.slot_bytes = slot_bytes;
    a.x_off = (t->L.max_unit_bytes + 127) & ~127;
    a.spw = spw;
    a.nc = nc;
    a.workers = (int32_t)workers;
    sip_gemv_kernel<<<(unsigned)grid, 32 * (1 + nc), smem, (cudaStream_t)stream>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        msg = std::string("sip_gemv_kernel: ") + cudaGetErrorString(e);
        return DM_ECUDA;
    }
    return DM_OK;
}

}  // namespace dm
