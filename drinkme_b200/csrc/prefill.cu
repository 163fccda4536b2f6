// The prefill path on sm_100a: Y[M, rows] = X[M, C] @ W^T for M >= 9
// activation rows (a prefill chunk) with W a sip tensor, the weights decoded
// into shared memory and contracted on the 5th-generation tensor cores
// (tcgen05.mma, fp32 accumulators in tensor memory).
//
// Reference: the dense arm (radix_kernel_gpu.py:615-636 `_dense`, swap.py:
// 361-378) decodes the whole weight to HBM, then runs one bf16 GEMM. The
// result contract is the same: fp32 accumulate, the bias added in fp32, one
// rounding; here the decoded weight never leaves the SM.
//
// Design:
//   * One CTA per 128 weight rows (the MMA's N), covering up to 512
//     activation rows in up to four 128-row token tiles (the MMA's M), one
//     fp32 accumulator per token tile in tensor memory (128 lanes x 128
//     columns each). The K loop runs over 64-wide windows.
//   * Decode warps 0-7: threads i and 128 + i own weight row i of the CTA,
//     taking alternate windows. Per window a thread reads the row's 64
//     literal bytes and 64 tier-0 codes (six words) straight from HBM (its
//     next window's prefetched into registers while it decodes), decodes
//     them with the GEMV's byte-parallel table lookups into bf16, and writes
//     the 128-byte K-major row of the B tile in the 128-byte swizzled layout
//     the tensor core reads (16-byte chunk c at c XOR (row mod 8)); escaped
//     weights take their terminal exponent from the escape index and are
//     patched in place. A fence makes the generic writes visible to the
//     tensor core's (async) reads; the warps then arrive on the stage's
//     barrier.
//   * Warp 8 stages the activation window of every token tile with one bulk
//     copy: a pre-pass (x_swizzle_kernel) wrote X window-major in the same
//     swizzled layout, so each window is one contiguous block.
//   * Warp 9 allocates the tensor memory; one of its threads issues the MMAs
//     (kind::f16, bf16 x bf16 -> fp32, M = 128, N = 128, K = 16) and commits
//     each window's MMAs to the barriers that free its stages.
//   * Epilogue: warps 0-3 read the accumulators (tcgen05.ld, thread = token
//     row, 32 weight rows per load), add the bias in fp32, round once, store.
//   * Every wait is bounded (the device error word records a wait that gave
//     up); the tensor memory is freed on every path.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <string>

#include "dm_device.cuh"
#include "dm_internal.h"

namespace dm {

namespace {

constexpr int kPfRows = 128;         // weight rows per CTA (MMA N)
constexpr int kPfTok = 128;          // activation rows per token tile (MMA M)
constexpr int kPfMaxTiles = 4;       // token tiles per pass (512 tensor-memory columns)
constexpr int kPfBStages = 4;        // decoded weight windows in flight
constexpr int kPfAStages = 2;        // activation windows in flight
constexpr int kPfWin = 64;           // K per window (one 128-byte swizzle row of bf16)
constexpr int kPfDecWarps = 8;       // two threads per weight row, alternate windows
constexpr int kPfActWarp = kPfDecWarps, kPfMmaWarp = kPfDecWarps + 1;
constexpr int kPfThreads = (kPfDecWarps + 2) * 32;
constexpr int kBTile = kPfRows * 128;          // 16 KB
constexpr int kPfEsc = 64;                     // escapes per row block staged in shared memory
constexpr int kATile = kPfTok * 128;           // 16 KB per token tile

// Shared-memory matrix descriptor of a 128-byte-swizzled K-major tile whose
// 8-row groups are 1024 bytes apart (rows 128 bytes): start address,
// leading byte offset 16 (unused with swizzling), stride byte offset 1024,
// descriptor version 1 (sm_100), layout type 2 = SWIZZLE_128B.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
    return (uint64_t)((smem_addr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor of kind::f16: fp32 accumulate (bits 4-5 = 1), A and
// B bf16 (bits 7-9, 10-12 = 1), both K-major, N >> 3 at bits 17-22, M >> 4 at
// bits 24-28.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kPfRows >> 3) << 17) |
                            ((uint32_t)(kPfTok >> 4) << 24);

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        :
        : "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(kIdesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_load32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// The selectors of 16 codes (quarter t of a quad) from the unit's code
// planes (the GEMV's code_selectors): v = plane word 4q + t, P = bit-2 word
// 64 + 2q + t / 2.
__device__ __forceinline__ void selectors16(uint32_t v, uint32_t P, int t, uint32_t &s0, uint32_t &s1) {
    const uint32_t rl = (t & 1) ? 0u : 2u, rh = (t & 1) ? 31u : 1u;
    s0 = (v & 0x33333333u) | (__funnelshift_l(P, P, rl) & 0x44444444u);
    s1 = ((v >> 2) & 0x33333333u) | (__funnelshift_l(P, P, rh) & 0x44444444u);
}

// Four weights -> two bf16 pairs (the GEMV's decode4).
__device__ __forceinline__ void dec4(uint32_t L, uint32_t S, uint32_t th0, uint32_t th1, uint32_t tl0, uint32_t tl1,
                                     uint32_t &p01, uint32_t &p23) {
    const uint32_t eh = __byte_perm(th0, th1, S);
    const uint32_t el = __byte_perm(tl0, tl1, S);
    const uint32_t hi = lop3<0x64>(L, eh, 0x80808080u);
    const uint32_t lo = lop3<0x98>(L, el, 0x80808080u);
    p01 = __byte_perm(lo, hi, 0x5140);
    p23 = __byte_perm(lo, hi, 0x7362);
}

struct PfArgs {
    const uint8_t *data;
    const uint32_t *unit16;
    int64_t rows, NB;
    const uint8_t *xs;  // swizzled activations: [windows][ntiles * 128 rows][128 bytes]
    int32_t ntiles, m;   // token tiles of this pass, real activation rows of it
    const uint16_t *bias;
    void *out;           // [m][rows] of this pass
    int32_t out_f32;
    int *err;
};

__global__ void __launch_bounds__(kPfThreads, 1) prefill_sip_kernel(PfArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte aligned tiles (the swizzle pattern follows address bits 7-9)
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *btile = smem;                                    // [kPfBStages][128 rows][128 B]
    uint8_t *atile = btile + kPfBStages * kBTile;             // [kPfAStages][ntiles][128 rows][128 B]
    // per weight row, the escapes of its current block column: position | terminal << 16
    uint32_t *esc = reinterpret_cast<uint32_t *>(atile + kPfAStages * kPfMaxTiles * kATile);  // [128][kPfEsc]
    uint64_t *bar = reinterpret_cast<uint64_t *>(esc + kPfRows * kPfEsc);
    uint64_t *b_full = bar, *b_empty = bar + kPfBStages;
    uint64_t *a_full = bar + 2 * kPfBStages, *a_empty = a_full + kPfAStages;
    uint64_t *acc_done = a_empty + kPfAStages;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t NB = a.NB;
    const int32_t nwin = (int32_t)(NB * 16);
    const int32_t ncols = a.ntiles <= 1 ? 128 : (a.ntiles == 2 ? 256 : 512);
    pdl_launch_dependents();
    if (threadIdx.x == 0) {
        for (int s = 0; s < kPfBStages; ++s) {
            mbar_init(&b_full[s], 4);  // the four warps of the half that decodes the window
            mbar_init(&b_empty[s], 1);
        }
        for (int s = 0; s < kPfAStages; ++s) {
            mbar_init(&a_full[s], 1);
            mbar_init(&a_empty[s], 1);
        }
        mbar_init(acc_done, 1);
        mbar_fence_init();
    }
    if (warp == kPfMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(ncols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp < kPfDecWarps) {
        // ------------------------------------------------------ decode --
        const int i = threadIdx.x & (kPfRows - 1);  // weight row of the CTA
        const int half = threadIdx.x >> 7;          // windows w = half, half + 2, ...
        const int64_t row = (int64_t)blockIdx.x * kPfRows + i;
        const bool real = row < a.rows;
        const int64_t tile16 = row / 16;
        const uint32_t sw = (uint32_t)(i & 7);
        bool ok = true;
        // the row's block of a block column: its literal plane, escape index,
        // terminal stream, escape count and exponent tables
        struct Hdr {
            const uint8_t *lit;
            const uint16_t *idx;
            const uint8_t *term;
            uint32_t th0, th1, tl0, tl1;
            int nesc;
        };
        auto load_hdr = [&](int64_t bc, Hdr &h) {
            const uint8_t *base = a.data + (size_t)a.unit16[tile16 * NB + bc] * 16;
            const RowEntry e = reinterpret_cast<const RowEntry *>(base)[row & 15];
            const uint4 tab = *reinterpret_cast<const uint4 *>(base + kUnitRows * sizeof(RowEntry));
            h.th0 = tab.x;
            h.th1 = tab.y;
            h.tl0 = tab.z;
            h.tl1 = tab.w;
            h.lit = base + (size_t)e.off16 * 16;
            h.idx = reinterpret_cast<const uint16_t *>(h.lit + (((uint32_t)e.words * 4u + 15u) & ~15u));
            h.term = h.lit + 1408;
            h.nesc = e.nesc;
        };
        auto load_win = [&](const Hdr &h, int qb, uint4 (&L)[4], uint32_t (&c)[6]) {
            const uint4 *lp = reinterpret_cast<const uint4 *>(h.lit + 64 * qb);
#pragma unroll
            for (int j = 0; j < 4; ++j) L[j] = lp[j];
            const uint32_t *cp = reinterpret_cast<const uint32_t *>(h.lit + 1024);
#pragma unroll
            for (int j = 0; j < 4; ++j) c[j] = cp[4 * qb + j];
            c[4] = cp[64 + 2 * qb];
            c[5] = cp[64 + 2 * qb + 1];
        };
        // this thread's windows w = half, half + 2, ...: block column w / 16,
        // quad w % 16
        Hdr hc{}, hn{};
        uint4 Ln[4] = {};
        uint32_t cn[6] = {0, 0, 0, 0, 0, 0};
        int cur = 0;
        const int32_t wk0 = half;
        // this thread's share of its row's staged escapes: entries
        // [32 half, 32 half + 32) of a block column's list, prefetched a
        // block column ahead and written at each block column's start
        uint4 sh_idx[4] = {};
        uint4 sh_term[2] = {};
        auto load_share = [&](const Hdr &h) {
            const uint4 *ip = reinterpret_cast<const uint4 *>(h.idx + 32 * half);
            const uint4 *tp = reinterpret_cast<const uint4 *>(h.term + 32 * half);
#pragma unroll
            for (int j = 0; j < 4; ++j) sh_idx[j] = ip[j];
#pragma unroll
            for (int j = 0; j < 2; ++j) sh_term[j] = tp[j];
        };
        auto store_share = [&]() {
            uint32_t *d = esc + i * kPfEsc + 32 * half;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const uint32_t iw = (&sh_idx[j >> 3].x)[(j >> 1) & 3];
                const uint32_t tw = (&sh_term[j >> 4].x)[(j >> 2) & 3];
                d[j] = ((iw >> (16 * (j & 1))) & 0xFFFFu) | (((tw >> (8 * (j & 3))) & 0xFFu) << 16);
            }
        };
        auto decoders_sync = [&]() {
            asm volatile("bar.sync 1, %0;" ::"r"(kPfDecWarps * 32) : "memory");
        };
        if (real) {
            load_hdr(wk0 >> 4, hc);
            load_hdr(((wk0 >> 4) + 1) % NB, hn);
            load_win(hc, wk0 & 15, Ln, cn);
            load_share(hc);
        }
        store_share();
        decoders_sync();
        bool need_share = true;  // the next block column's share still to fetch
        for (int32_t w = half; w < nwin; w += 2) {
            const int s = w % kPfBStages, use = w / kPfBStages;
            const int32_t wk = w;
            const int qb = wk & 15;
            uint4 L[4];
            uint32_t cw[6];
#pragma unroll
            for (int j = 0; j < 4; ++j) L[j] = Ln[j];
#pragma unroll
            for (int j = 0; j < 6; ++j) cw[j] = cn[j];
            // the next window of this thread: its bytes fetched now (from the
            // next block column's row block when it starts one)
            const int32_t wk2 = w + 2;
            const bool more = wk2 < nwin;
            const bool newblk = more && (wk2 >> 4) != (wk >> 4);
            if (real && more) load_win(newblk ? hn : hc, wk2 & 15, Ln, cn);
            if (need_share && !newblk) {  // the next block column's escapes, a block column early
                if (real) load_share(hn);
                need_share = false;
            }
            if (use > 0 && ok && !mbar_wait(&b_empty[s], (uint32_t)((use - 1) & 1), a.err, kErrWaitEmpty)) ok = false;
            uint8_t *rowp = btile + s * kBTile + i * 128;
#pragma unroll
            for (int j = 0; j < 4; ++j) {  // 16 weights: quarter j of the quad
                uint32_t xa, xb;
                selectors16(cw[j], cw[4 + (j >> 1)], j, xa, xb);
                uint32_t p[8];
                // code 7 decodes to sign | exponent 0 | mantissa: the escape
                // patch below only ORs the terminal exponent in
                const uint32_t th1 = hc.th1 & 0x00FFFFFFu, tl1 = hc.tl1 & 0x00FFFFFFu;
                dec4(L[j].x, xa, hc.th0, th1, hc.tl0, tl1, p[0], p[1]);
                dec4(L[j].y, xa >> 16, hc.th0, th1, hc.tl0, tl1, p[2], p[3]);
                dec4(L[j].z, xb, hc.th0, th1, hc.tl0, tl1, p[4], p[5]);
                dec4(L[j].w, xb >> 16, hc.th0, th1, hc.tl0, tl1, p[6], p[7]);
                if (!real) {
#pragma unroll
                    for (int k = 0; k < 8; ++k) p[k] = 0u;
                }
                *reinterpret_cast<uint4 *>(rowp + (((2u * j) ^ sw) << 4)) = make_uint4(p[0], p[1], p[2], p[3]);
                *reinterpret_cast<uint4 *>(rowp + (((2u * j + 1u) ^ sw) << 4)) = make_uint4(p[4], p[5], p[6], p[7]);
            }
            // escapes of this window: the terminal exponent ORed in (the other
            // half's windows' escapes are passed over); the staged list, then
            // global memory past its kPfEsc entries
            if (real) {
                const uint32_t start = 64u * (uint32_t)qb, end = start + 64u;
                const uint32_t *el = esc + i * kPfEsc;
                const int lim = hc.nesc < kPfEsc ? hc.nesc : kPfEsc;
                while (cur < lim) {
                    const uint32_t e = el[cur];
                    const uint32_t pos = e & 1023u;
                    if (pos >= end) break;
                    if (pos >= start) {
                        const uint32_t k = pos - start;
                        *reinterpret_cast<uint16_t *>(rowp + ((((k >> 3) ^ sw) << 4) | ((k & 7u) << 1))) |=
                            (uint16_t)(((e >> 16) & 0xFFu) << 7);
                    }
                    ++cur;
                }
                if (cur >= kPfEsc)
                    while (cur < hc.nesc) {
                        const uint32_t pos = hc.idx[cur] & 1023u;
                        if (pos >= end) break;
                        if (pos >= start) {
                            const uint32_t k = pos - start;
                            *reinterpret_cast<uint16_t *>(rowp + ((((k >> 3) ^ sw) << 4) | ((k & 7u) << 1))) |=
                                (uint16_t)((uint32_t)hc.term[cur] << 7);
                        }
                        ++cur;
                    }
            }
            fence_proxy_async_smem();  // these generic writes, before the tensor core's async reads
            __syncwarp();
            if ((threadIdx.x & 31) == 0) mbar_arrive(&b_full[s]);
            if (newblk) {  // this thread's next window starts a block column
                decoders_sync();  // every decoder done with the staged escapes
                store_share();
                decoders_sync();
                hc = hn;
                cur = 0;
                if (real) load_hdr(((wk2 >> 4) + 1) % NB, hn);
                need_share = true;
            }
        }
        // ---------------------------------------------------- epilogue --
        // warps 0-3 (warp w reads tensor-memory lanes 32w .. 32w + 31)
        if (warp < 4) {
        if (ok && !mbar_wait(acc_done, 0u, a.err, kErrWaitFull)) ok = false;
        tmem_fence_after();
        for (int tt = 0; tt < a.ntiles; ++tt) {
            const int tok = tt * kPfTok + warp * 32 + lane;
            for (int c0 = 0; c0 < kPfRows; c0 += 32) {
                uint32_t r[32];
                tmem_load32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(tt * kPfRows + c0), r);
                if (!ok || tok >= a.m) continue;
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int64_t orow = (int64_t)blockIdx.x * kPfRows + c0 + j;
                    if (orow >= a.rows) break;
                    float y = __uint_as_float(r[j]);
                    if (a.bias) y += bf16_bits_to_f32(a.bias[orow]);
                    if (a.out_f32)
                        reinterpret_cast<float *>(a.out)[(int64_t)tok * a.rows + orow] = y;
                    else
                        reinterpret_cast<uint16_t *>(a.out)[(int64_t)tok * a.rows + orow] = f32_to_bf16_bits(y);
                }
            }
        }
        tmem_fence_before();
        }
    } else if (warp == kPfActWarp) {
        // -------------------------------------------------- activations --
        if (lane == 0) {
            pdl_wait();  // the swizzled activations come from the kernel before this one
            const uint32_t bytes = (uint32_t)a.ntiles * kATile;
            bool ok = true;
            for (int32_t w = 0; w < nwin && ok; ++w) {
                const int s = w % kPfAStages, use = w / kPfAStages;
                if (use > 0 && !mbar_wait(&a_empty[s], (uint32_t)((use - 1) & 1), a.err, kErrWaitEmpty)) ok = false;
                if (!ok) break;
                mbar_arrive_expect_tx(&a_full[s], bytes);
                bulk_g2s(atile + s * kPfMaxTiles * kATile, a.xs + (size_t)w * bytes, bytes, &a_full[s]);
            }
        }
    } else {
        // ---------------------------------------------------------- MMA --
        bool ok = true;
        for (int32_t w = 0; w < nwin; ++w) {
            const int sb = w % kPfBStages, sa = w % kPfAStages;
            if (ok && !mbar_wait(&a_full[sa], (uint32_t)((w / kPfAStages) & 1), a.err, kErrWaitFull)) ok = false;
            if (ok && !mbar_wait(&b_full[sb], (uint32_t)((w / kPfBStages) & 1), a.err, kErrWaitFull)) ok = false;
            tmem_fence_after();
            if (lane == 0) {
                if (ok) {
                    const uint32_t bb = smem_addr(btile + sb * kBTile);
                    const uint32_t ab = smem_addr(atile + sa * kPfMaxTiles * kATile);
#pragma unroll
                    for (int k = 0; k < kPfWin / 16; ++k)
                        for (int tt = 0; tt < a.ntiles; ++tt)
                            umma_bf16(tmem + (uint32_t)(tt * kPfRows), sw128_desc(ab + tt * kATile + 32 * k),
                                      sw128_desc(bb + 32 * k), (w > 0 || k > 0) ? 1u : 0u);
                }
                umma_commit(&b_empty[sb]);  // frees the stages once these MMAs have read them
                umma_commit(&a_empty[sa]);
            }
            __syncwarp();
        }
        if (lane == 0) umma_commit(acc_done);
        __syncwarp();
    }
    // every warp: the epilogue's tensor-memory reads done before the free
    __syncthreads();
    if (warp == kPfMmaWarp) {
        tmem_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
    }
}

// X [m][C] bf16 (row stride ldx) -> window-major 128-byte-swizzled tiles
// [C / 64][ntiles * 128][128 bytes]; rows past m are zero.
__global__ void x_swizzle_kernel(const uint16_t *__restrict__ x, int64_t ldx, int32_t m, int32_t ntiles, int64_t C,
                                 uint8_t *__restrict__ xs) {
    const int64_t rows = (int64_t)ntiles * kPfTok;
    const int64_t chunks = (C / 8) * rows;  // 16-byte chunks
    for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < chunks; q += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = q % rows, kc = q / rows;  // token row, 8-weight chunk of K
        const int64_t w = kc >> 3, c = kc & 7;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < m) v = *reinterpret_cast<const uint4 *>(x + r * ldx + kc * 8);
        *reinterpret_cast<uint4 *>(xs + (w * rows + r) * 128 + ((c ^ (r & 7)) << 4)) = v;
    }
}

}  // namespace

int64_t prefill_workspace_bytes(const dm_tensor *t, int64_t M) {
    const int64_t m = std::min<int64_t>(M, (int64_t)kPfMaxTiles * kPfTok);
    const int64_t ntiles = (m + kPfTok - 1) / kPfTok;
    return t->L.C * ntiles * kPfTok * 2;
}

int launch_prefill_sip(const dm_tensor *t, const uint16_t *x, int64_t M, const uint16_t *bias, void *out,
                       int out_f32, uint8_t *work, int64_t work_bytes, void *stream, std::string &msg) {
    const TensorLayout &L = t->L;
    if (!L.fast_sip) {
        msg = "dm_prefill: needs a sip tensor (the fast path)";
        return DM_EINVAL;
    }
    if (work_bytes < prefill_workspace_bytes(t, M) || (reinterpret_cast<uintptr_t>(work) & 15) ||
        (reinterpret_cast<uintptr_t>(x) & 15)) {
        msg = "dm_prefill: workspace too small or activations / workspace not 16-byte aligned";
        return DM_EINVAL;
    }
    const int smem = kPfBStages * kBTile + kPfAStages * kPfMaxTiles * kATile + kPfRows * kPfEsc * 4 + 1024 + 256;
    // a per-device attribute: one bit per device (64 and up: every launch)
    static std::atomic<uint64_t> attr{0};
    const uint64_t dev_bit = t->device >= 0 && t->device < 64 ? 1ull << t->device : 0ull;
    if (!dev_bit || !(attr.load() & dev_bit)) {
        cudaError_t e = cudaFuncSetAttribute(prefill_sip_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) {
            msg = std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e);
            return DM_ECUDA;
        }
        attr.fetch_or(dev_bit);
    }
    const int64_t grid = (L.rows + kPfRows - 1) / kPfRows;
    for (int64_t m0 = 0; m0 < M; m0 += (int64_t)kPfMaxTiles * kPfTok) {
        const int32_t m = (int32_t)std::min<int64_t>(M - m0, (int64_t)kPfMaxTiles * kPfTok);
        const int32_t ntiles = (m + kPfTok - 1) / kPfTok;
        const int64_t chunks = (L.C / 8) * ntiles * kPfTok;
        const int blocks = (int)std::min<int64_t>((chunks + 255) / 256, (int64_t)t->sms * 16);
        x_swizzle_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(x + m0 * L.C, L.C, m, ntiles, L.C, work);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) {
            msg = std::string("x_swizzle_kernel: ") + cudaGetErrorString(e);
            return DM_ECUDA;
        }
        PfArgs a{};
        a.data = t->d_data;
        a.unit16 = t->d_unit16;
        a.rows = L.rows;
        a.NB = L.NB;
        a.xs = work;
        a.ntiles = ntiles;
        a.m = m;
        a.bias = bias;
        a.out = reinterpret_cast<uint8_t *>(out) + (size_t)m0 * L.rows * (out_f32 ? 4 : 2);
        a.out_f32 = out_f32;
        a.err = t->S.err;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)grid);
        cfg.blockDim = dim3(kPfThreads);
        cfg.dynamicSmemBytes = (size_t)smem;
        cfg.stream = (cudaStream_t)stream;
        cudaLaunchAttribute attr1[1];
        attr1[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr1[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr1;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, prefill_sip_kernel, a);
        if (e != cudaSuccess) {
            msg = std::string("prefill_sip_kernel: ") + cudaGetErrorString(e);
            return DM_ECUDA;
        }
    }
    return DM_OK;
}

}  // namespace dm
