// The prefill path on sm_100a: Y[M, rows] = X[M, C] @ W^T for a prefill
// chunk (the module routes M >= 9 here) with W a sip tensor, the weights
// decoded into shared memory and contracted on the 5th-generation tensor
// cores (tcgen05.mma, fp32 accumulators in tensor memory).
//
// Reference: the dense arm (radix_kernel_gpu.py:615-636 `_dense`, swap.py:
// 361-378) decodes the whole weight to HBM, then runs one bf16 GEMM. The
// result contract is the same: fp32 accumulate, the bias added in fp32, one
// rounding; here the decoded weight never leaves the SM.
//
// Design:
//   * A TILE is 128 weight rows (the MMA's M: the decoded weights are the A
//     operand) by a GROUP of up to 512 activation rows (the B operand), over
//     the whole K. A group is one or two HALVES of at most 256 activation rows
//     (the MMA's N), each with its own 256-column fp32 accumulator in tensor
//     memory, so every weight window is decoded ONCE for all the group's
//     activation rows (at M = 512, half the decode work of 256-row tiles).
//     With one half, the two accumulators alternate between tiles and a
//     tile's epilogue runs under the next tile's MMAs; with two, the first
//     half drains while the second half's last MMAs run.
//   * Persistent stream-K over K windows of 64: one CTA per SM; the windows of
//     every tile, tile after tile (a weight row tile's groups next to each
//     other, so its compressed bytes come from L2 the second time), are split
//     evenly over the CTAs. A CTA's first and last tiles may be shared with
//     its neighbours (PIECES); it runs those first. Per quarter of a shared
//     tile's rows, the pieces count their arrivals; every piece but the last
//     writes its fp32 partial and marks it ready, and the last adds the
//     others' partials and its own accumulator in CTA order (deterministic)
//     straight from tensor memory to the outputs.
//   * Warps 0-15 decode: four lanes per weight row (lane t takes weights
//     [16t, 16t + 16) of every window), from the loader's code planes with
//     the GEMV's byte-parallel table lookups (an escape, code 7, decodes to
//     +0), into the 128-byte-swizzled K-major tile the tensor core reads. The
//     escaped weights are then rewritten whole from the loader's escape
//     index (their positions) and the row's terminal stream (their
//     exponents, by rank): a row's four lanes share its window's escapes, no
//     bit scans. The compressed operands of the next four windows are staged
//     by cp.async into a shared-memory ring (literal plane, code words, bit-2
//     words), so no lane waits on a load of its own in flight.
//   * Warp 20 loads each activation window (one TMA tensor copy per half, no
//     multicast) in the same swizzled layout; lane 0 of warp 21 owns the MMA
//     issue (kind::f16, M = 128, N = half width, K = 16) and commits each
//     window to the barriers that free its stages; warp 21 owns the tensor
//     memory.
//   * Warps 16-19 read the accumulators (tcgen05.ld, a lane per weight row),
//     add the bias in fp32, round once and store; or write a piece's partial
//     (activation-row major, so a warp's store is one 128-byte line).
//   * Every wait is bounded (the device error word records a wait that gave
//     up); the tensor memory is freed on every path.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <string>

#include "dm_device.cuh"
#include "dm_internal.h"

namespace dm {

namespace {

constexpr int kPfRows = 128;       // weight rows per tile (MMA M)
constexpr int kHalfMax = 256;      // activation rows per half, at most (MMA N)
constexpr int kGroupMax = 512;     // activation rows per group (two halves)
constexpr int kWStages = 3;        // decoded weight windows in flight
constexpr int kMaxXStages = 6;     // activation half-windows in flight, at most
constexpr int kDecWarps = 16;      // eight weight rows per warp, four lanes per row
constexpr int kEpi0 = 16;          // warps 16-19: the epilogue (tensor-memory lane quarters 0-3)
constexpr int kProd = 20;          // warp 20: activation TMA
constexpr int kMma = 21;           // warp 21: tensor memory and MMA issue
constexpr int kPfThreads = 22 * 32;
constexpr int kAhead = 4;          // windows of compressed operands in flight (a cp.async ring)
constexpr int kLitStage = kPfRows * 64;   // literal plane: 64 bytes per row and window
constexpr int kCodeStage = kPfRows * 16;  // low-two-bit code words: four per row and window
constexpr int kBitStage = kPfRows * 8;    // bit-2 words: two per row and window
constexpr int kOpStage = kLitStage + kCodeStage + kBitStage;
constexpr int kWStage = kPfRows * 128;    // 16 KB: 128 rows x 64 bf16
constexpr int kAccCols = 256;             // tensor-memory columns per accumulator
constexpr int kMaxParts = 8;
constexpr int kNumBars = 2 * kMaxXStages + 2 * kWStages + 5;
constexpr int kFixedSmem = kWStages * kWStage + kAhead * kOpStage + kNumBars * 8 + 16 + kMaxParts * 16 + 80;
constexpr int kSmemLimit = 232448;        // the per-block opt-in maximum of sm_100
constexpr int kXBudget = kSmemLimit - 1024 - kFixedSmem;

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
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        :
        : "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_load16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// mbar_wait for a wait expected to be long: a try without a time hint, then a
// 256 ns sleep between tries (about 2^18 tries: tens of milliseconds), so the
// waiting lane takes almost no issue slots or shared-memory bandwidth.
__device__ __forceinline__ bool mbar_wait_backoff(uint64_t *bar, uint32_t parity, int *err, int code) {
    for (uint32_t i = 0; i < (1u << 18); ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(smem_addr(bar)), "r"(parity)
            : "memory");
        if (done) return true;
        __nanosleep(256);
    }
    if (err) atomicExch(err, code);
    return false;
}

// One 2-D TMA tile load global -> shared (no multicast), completing on `bar`.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int32_t x, int32_t y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// global -> shared, asynchronously (the LDGSTS path)
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Waits until at most `n` (0..3) of this thread's newest groups are pending.
__device__ __forceinline__ void cp_async_wait(int n) {
    if (n <= 0)
        asm volatile("cp.async.wait_group 0;" ::: "memory");
    else if (n == 1)
        asm volatile("cp.async.wait_group 1;" ::: "memory");
    else if (n == 2)
        asm volatile("cp.async.wait_group 2;" ::: "memory");
    else
        asm volatile("cp.async.wait_group 3;" ::: "memory");
}

// A release increment of a counter another CTA acquires.
__device__ __forceinline__ void red_add_release_gpu(uint32_t *p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// The selectors of 16 codes (one quarter of a 64-weight window) from a row
// block's code planes: v = the quarter's low-two-bit word, P = the bit-2 word
// it shares with its neighbour, rotated by (rl, rh) = (2, 1) for an even
// quarter and (0, 31) for an odd one (the GEMV's code_selectors).
__device__ __forceinline__ void selectors16(uint32_t v, uint32_t P, uint32_t rl, uint32_t rh, uint32_t &s0,
                                            uint32_t &s1) {
    s0 = (v & 0x33333333u) | (__funnelshift_l(P, P, rl) & 0x44444444u);
    s1 = ((v >> 2) & 0x33333333u) | (__funnelshift_l(P, P, rh) & 0x44444444u);
}

// Four weights -> two bf16 pairs (the GEMV's decode4); code 7 gives +0.
__device__ __forceinline__ void dec4(uint32_t L, uint32_t S, uint32_t th0, uint32_t th1, uint32_t tl0, uint32_t tl1,
                                     uint32_t &p01, uint32_t &p23) {
    const uint32_t eh = __byte_perm(th0, th1, S);
    const uint32_t el = __byte_perm(tl0, tl1, S);
    const uint32_t hi = lop3<0x64>(L, eh, 0x80808080u);
    const uint32_t lo = lop3<0x98>(L, el, 0x80808080u);
    p01 = __byte_perm(lo, hi, 0x5140);
    p23 = __byte_perm(lo, hi, 0x7362);
}

// Escapes (code 7) among the eight codes of a selector word: bit 4i is set
// where nibble i holds 7; the multiply gathers the eight bits into the top
// nibble (at most 8), which keeps the count off the XU pipe.
__device__ __forceinline__ uint32_t escapes8(uint32_t s) {
    return ((s & (s >> 1) & (s >> 2) & 0x11111111u) * 0x11111111u) >> 28;
}

struct PfArgs {
    const uint8_t *data;
    const uint2 *rowdir;     // [16-row padded rows][NB]: stream offset (16-byte units),
                             // nesc | part << 11 | escape-index offset (16-byte units) << 16
    int64_t rows, NB;
    int32_t M, ngrp, nt, nh; // real activation rows, groups, rows per half (MMA N), halves per group
    int64_t ntiles, W;       // tiles (row tiles x groups), all windows
    int32_t nwin;            // windows per tile
    int32_t nxs;             // activation stages
    uint32_t idesc;
    const uint16_t *bias;
    void *out;               // [M][rows]
    int32_t out_f32;
    float *part;             // [grid][2][nh * nt][128]: a CTA's partials of its first / last tile
    uint32_t *counters;      // [ntiles][8]: per row quarter, arrivals then ready partials; zero on entry
    int *err;
    uint32_t tabs[kMaxParts][4];
};

// The CTA's windows [x0, x1) of the whole sequence (tile-major), as PIECES:
// its first tile when partial, its whole tiles in order, then its last tile
// when partial. The last piece is the CTA's last work, so when it is the
// last of its tile's pieces to finish, its accumulator is still in tensor
// memory for the tile's fixup at the CTA's end.
struct Range {
    int64_t x0, x1;
    int32_t tA, tB, nwin;
    bool pA, pB;
    int32_t n;
    __device__ void init(int64_t c, int64_t G, int64_t W, int32_t nw) {
        nwin = nw;
        x0 = c * W / G;
        x1 = (c + 1) * W / G;
        n = 0;
        pA = pB = false;
        tA = tB = 0;
        if (x1 <= x0) return;
        tA = (int32_t)(x0 / nwin);
        tB = (int32_t)((x1 - 1) / nwin);
        if (tA == tB) {
            n = 1;
            return;
        }
        pA = x0 % nwin != 0;
        pB = x1 % nwin != 0;
        n = (pA ? 1 : 0) + (pB ? 1 : 0) + ((pB ? tB : tB + 1) - (pA ? tA + 1 : tA));
    }
    __device__ void piece(int32_t i, int32_t &t, int32_t &w0, int32_t &w1) const {
        if (tA == tB) {
            t = tA;
            w0 = (int32_t)(x0 - (int64_t)tA * nwin);
            w1 = (int32_t)(x1 - (int64_t)tA * nwin);
            return;
        }
        if (pA) {
            if (i == 0) {
                t = tA;
                w0 = (int32_t)(x0 - (int64_t)tA * nwin);
                w1 = nwin;
                return;
            }
            --i;
        }
        const int32_t first = pA ? tA + 1 : tA;
        const int32_t nwhole = (pB ? tB : tB + 1) - first;
        if (i < nwhole) {
            t = first + i;
            w0 = 0;
            w1 = nwin;
            return;
        }
        t = tB;
        w0 = 0;
        w1 = (int32_t)(x1 - (int64_t)tB * nwin);
    }
};

__device__ __forceinline__ int64_t cta_start(int64_t c, int64_t G, int64_t W) { return c * W / G; }

// The CTA whose windows hold window x.
__device__ __forceinline__ int64_t owner_of(int64_t x, int64_t G, int64_t W) {
    int64_t c = x * G / W;
    while (c + 1 < G && cta_start(c + 1, G, W) <= x) ++c;
    while (c > 0 && cta_start(c, G, W) > x) --c;
    return c;
}

// A position in the CTA's window sequence: piece pi, window w of tile t
// (weight row tile rt).
struct Cursor {
    int32_t pi, w, w1, t, rt;
    bool done;
    __device__ void at_piece(const Range &R, int32_t ngrp) {
        int32_t w0;
        R.piece(pi, t, w0, w1);
        w = w0;
        rt = t / ngrp;
    }
    __device__ void begin(const Range &R, int32_t ngrp) {
        pi = 0;
        done = R.n == 0;
        t = rt = w = w1 = 0;
        if (!done) at_piece(R, ngrp);
    }
    __device__ void next(const Range &R, int32_t ngrp) {
        if (++w < w1) return;
        if (++pi >= R.n) {
            done = true;
            return;
        }
        at_piece(R, ngrp);
    }
};

__global__ void __launch_bounds__(kPfThreads, 1) prefill_sip_kernel(const __grid_constant__ CUtensorMap xmap, PfArgs a) {
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned tiles (the swizzle pattern follows address bits 7-9)
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t xstage = (uint32_t)a.nt * 128u;  // one half of an activation window
    uint8_t *xs = smem;
    uint8_t *ws = xs + (size_t)a.nxs * xstage;
    uint8_t *ops = ws + kWStages * kWStage;  // [kAhead] x {literals [128][64], code words [128][16], bit-2 words [128][8]}
    uint64_t *bar = reinterpret_cast<uint64_t *>(ops + kAhead * kOpStage);
    uint64_t *x_full = bar, *x_empty = bar + kMaxXStages, *w_full = bar + 2 * kMaxXStages, *w_empty = w_full + kWStages;
    uint64_t *acc_full = w_empty + kWStages, *acc_empty = acc_full + 2, *drained = acc_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bar + kNumBars);
    uint32_t *tabs = tmem_slot + 4;  // [kMaxParts][4]
    // the shared tiles whose fixup this CTA runs at its end, per row quarter
    // (at most two: its first and last tiles): tile, and whether its own sum
    // is still in tensor memory
    int32_t *fix_n = reinterpret_cast<int32_t *>(tabs + kMaxParts * 4);  // [4]
    int32_t *fix_t = fix_n + 4, *fix_own = fix_t + 8;                       // [4][2]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t G = gridDim.x;
    Range R;
    R.init(blockIdx.x, G, a.W, a.nwin);
    if (threadIdx.x == 0) {
        for (int s = 0; s < kMaxXStages; ++s) {
            mbar_init(&x_full[s], 1);
            mbar_init(&x_empty[s], 1);
        }
        for (int s = 0; s < kWStages; ++s) {
            mbar_init(&w_full[s], kDecWarps);
            mbar_init(&w_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);
        }
        mbar_init(drained, 1);
        mbar_fence_init();
        for (int q = 0; q < 4; ++q) fix_n[q] = 0;
    }
    if (warp == kProd && lane < kMaxParts * 4) tabs[lane] = (&a.tabs[0][0])[lane];
    if (warp == kMma) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(2 * kAccCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int64_t NB = a.NB;

    if (warp < kDecWarps) {
        // ------------------------------------------------------ decode --
        // row r of the tile; lane t of the row's four decodes weights
        // [16t, 16t + 16) of every window
        const int tq = lane & 3;
        const int r = warp * 8 + (lane >> 2);
        const uint32_t sw = (uint32_t)(r & 7);
        const uint32_t st0 = (uint32_t)r * 128u + (((uint32_t)(2 * tq) ^ sw) << 4);
        const uint32_t st1 = (uint32_t)r * 128u + (((uint32_t)(2 * tq + 1) ^ sw) << 4);
        const uint32_t rl = (tq & 1) ? 0u : 2u, rh = (tq & 1) ? 31u : 1u;
        const uint32_t lit_at = (uint32_t)r * 64u + 16u * tq;
        const uint32_t code_at = kLitStage + (uint32_t)r * 16u + 4u * tq;
        const uint32_t bit_at = kLitStage + kCodeStage + (uint32_t)r * 8u + 4u * (tq >> 1);
        bool ok = true;
        // the load cursor runs kAhead windows before the decode position; a
        // window's compressed operands go to ring slot (window mod kAhead):
        // lane t its 16 literal bytes, lane 0 the row's four code words, lane
        // 1 its two bit-2 words; one cp.async group per window
        Cursor cl;
        cl.begin(R, a.ngrp);
        int32_t lseg_t = -1, lseg_bc = -1;
        uint32_t lbase16 = 0;
        bool lreal = false;
        int32_t nload = 0;
        auto dir_load = [&](int32_t rt, int32_t bc) -> uint2 {
            const int64_t row = (int64_t)rt * kPfRows + r;
            if (row >= a.rows) return make_uint2(0, 0);
            return __ldg(a.rowdir + row * NB + bc);
        };
        auto load_window = [&]() {
            const int32_t bc = cl.w >> 4;
            if (cl.t != lseg_t || bc != lseg_bc) {
                lseg_t = cl.t;
                lseg_bc = bc;
                lreal = (int64_t)cl.rt * kPfRows + r < a.rows;
                lbase16 = dir_load(cl.rt, bc).x;
            }
            if (lreal) {
                const uint32_t q = (uint32_t)(cl.w & 15);
                const uint8_t *blk = a.data + (size_t)lbase16 * 16;
                uint8_t *o = ops + (nload % kAhead) * kOpStage;
                cp_async16(o + lit_at, blk + 64 * q + 16 * tq);
                if (tq == 0) cp_async16(o + kLitStage + r * 16, blk + 1024 + 16 * q);
                if (tq == 1) cp_async8(o + kLitStage + kCodeStage + r * 8, blk + 1280 + 8 * q);
            }
            cp_async_commit();
            ++nload;
        };
#pragma unroll 1
        for (int i = 0; i < kAhead && !cl.done; ++i) {
            load_window();
            cl.next(R, a.ngrp);
        }
        uint32_t run = 0;  // escapes of this row block before the current window
        int32_t j = 0;     // window sequence number (its stage)
        Cursor cd;
        cd.begin(R, a.ngrp);
        int32_t dseg_t = -1, dseg_bc = -1;
        const uint8_t *blk = a.data;  // the decode position's row block
        const uint16_t *eidx = nullptr;
        uint32_t nesc = 0;
        bool real = false;
        uint32_t th0 = 0, th1 = 0, tl0 = 0, tl1 = 0;
        while (!cd.done) {
            const int32_t bc = cd.w >> 4;
            if (cd.t != dseg_t || bc != dseg_bc) {
                dseg_t = cd.t;
                dseg_bc = bc;
                run = 0;
                real = (int64_t)cd.rt * kPfRows + r < a.rows;
                const uint2 dir = dir_load(cd.rt, bc);  // an L1 hit: the load cursor read it a few windows ago
                blk = a.data + (size_t)dir.x * 16;
                nesc = dir.y & 0x7FFu;
                eidx = reinterpret_cast<const uint16_t *>(blk + (size_t)(dir.y >> 16) * 16);
                const uint32_t part = (dir.y >> 11) & 31u;
                const uint32_t *tb = tabs + 4 * (part < kMaxParts ? part : 0);
                th0 = tb[0];
                th1 = tb[1] & 0x00FFFFFFu;
                tl0 = tb[2];
                tl1 = tb[3] & 0x00FFFFFFu;
                // a piece that starts inside a block column: the block's
                // escapes before this window come first in rank (the escape
                // index is in block order)
                const uint32_t q0 = (uint32_t)(cd.w & 15);
                if (q0 > 0) {
                    uint32_t pre = 0;
                    if (real)
                        for (uint32_t i = tq; i < nesc; i += 4) pre += __ldg(eidx + i) < 64u * q0 ? 1u : 0u;
                    pre += __shfl_xor_sync(0xffffffffu, pre, 1);
                    pre += __shfl_xor_sync(0xffffffffu, pre, 2);
                    run = pre;
                }
            }
            // this window's group landed (every lane's: the escape rewrite
            // reads literal bytes another lane staged)
            cp_async_wait(nload - j - 1);
            __syncwarp();
            const int s = j % kWStages, use = j / kWStages;
            if (use > 0 && ok) {  // lane 0 polls; the warp barrier orders the others after it
                int got = 1;
                if (lane == 0) got = mbar_wait(&w_empty[s], (uint32_t)((use - 1) & 1), a.err, kErrWaitEmpty);
                ok = __shfl_sync(0xffffffffu, got, 0) != 0;
            }
            uint8_t *wst = ws + s * kWStage;
            const uint8_t *o = ops + (j % kAhead) * kOpStage;
            uint32_t tot = 0;
            if (real) {
                const uint4 L = *reinterpret_cast<const uint4 *>(o + lit_at);
                const uint32_t v = *reinterpret_cast<const uint32_t *>(o + code_at);
                const uint32_t P = *reinterpret_cast<const uint32_t *>(o + bit_at);
                uint32_t s0, s1, p0, p1, p2, p3, p4, p5, p6, p7;
                selectors16(v, P, rl, rh, s0, s1);
                dec4(L.x, s0, th0, th1, tl0, tl1, p0, p1);
                dec4(L.y, s0 >> 16, th0, th1, tl0, tl1, p2, p3);
                dec4(L.z, s1, th0, th1, tl0, tl1, p4, p5);
                dec4(L.w, s1 >> 16, th0, th1, tl0, tl1, p6, p7);
                *reinterpret_cast<uint4 *>(wst + st0) = make_uint4(p0, p1, p2, p3);
                *reinterpret_cast<uint4 *>(wst + st1) = make_uint4(p4, p5, p6, p7);
                tot = escapes8(s0) + escapes8(s1);
            } else {
                *reinterpret_cast<uint4 *>(wst + st0) = make_uint4(0u, 0u, 0u, 0u);
                *reinterpret_cast<uint4 *>(wst + st1) = make_uint4(0u, 0u, 0u, 0u);
            }
            // the row's escapes in this window: ranks [run, run + tot) of the
            // row block, their positions from the escape index, their
            // exponents from the terminal stream; lane t takes every fourth.
            // Ranks at or past nesc (a terminal stream cut short) stay +0.
            tot += __shfl_xor_sync(0xffffffffu, tot, 1);
            tot += __shfl_xor_sync(0xffffffffu, tot, 2);
            __syncwarp();  // the quarters' stores before the rewrites of single weights
            const uint32_t hi = min(run + tot, nesc);
            for (uint32_t i = run + tq; i < hi; i += 4) {
                const uint32_t pos = (uint32_t)__ldg(eidx + i) & 63u;
                const uint32_t ex = __ldg(blk + 1408 + i);
                const uint32_t lit = o[r * 64 + pos];
                *reinterpret_cast<uint16_t *>(wst + (uint32_t)r * 128u + ((((pos >> 3) ^ sw) << 4) | ((pos & 7u) << 1))) =
                    (uint16_t)(((lit & 0x80u) << 8) | (ex << 7) | (lit & 0x7Fu));
            }
            run += tot;
            fence_proxy_async_smem();  // these generic writes, before the tensor core's async reads
            __syncwarp();
            if (lane == 0) mbar_arrive(&w_full[s]);
            // every lane has read the ring slot: it takes the window kAhead ahead
            if (!cl.done) {
                load_window();
                cl.next(R, a.ngrp);
            }
            cd.next(R, a.ngrp);
            ++j;
        }
        cp_async_wait(0);
    } else if (warp >= kEpi0 && warp < kEpi0 + 4) {
        // ---------------------------------------------------- epilogue --
        const int qtr = warp - kEpi0;  // tensor-memory lanes 32 qtr .. 32 qtr + 31
        const int32_t GT = a.nh * a.nt;
        bool ok = true;
        uint32_t uses[2] = {0u, 0u};
        for (int32_t pi = 0; pi < R.n && ok; ++pi) {
            int32_t t, w0, w1;
            R.piece(pi, t, w0, w1);
            const bool whole = w0 == 0 && w1 == a.nwin;
            const bool final = pi == R.n - 1;
            const int64_t row = (int64_t)(t / a.ngrp) * kPfRows + qtr * 32 + lane;
            const int32_t tok0 = (t % a.ngrp) * GT;
            const float bv = (a.bias && row < a.rows) ? bf16_bits_to_f32(a.bias[row]) : 0.f;
            uint32_t *arrive = a.counters + t * 8 + qtr;
            uint32_t np = 1;
            if (!whole) {
                const int64_t tw = (int64_t)t * a.nwin;
                np = (uint32_t)(owner_of(tw + a.nwin - 1, G, a.W) - owner_of(tw, G, a.W) + 1);
            }
            // a piece's partial: [row quarter][activation row / 4][32 rows][4],
            // so a warp's float4 store of four activation rows is 512
            // consecutive bytes
            float *mine = a.part + (((int64_t)blockIdx.x * 2 + (t == R.tA ? 0 : 1)) * 4 + qtr) * GT * 32 + lane * 4;
            bool keep = false;
            for (int h = 0; h < a.nh && ok; ++h) {
                const int slot = a.nh == 2 ? h : (pi & 1);
                int got = 1;  // a long wait: lane 0 polls with a backoff, the others idle at the warp barrier
                if (lane == 0) got = mbar_wait_backoff(&acc_full[slot], uses[slot] & 1u, a.err, kErrWaitFull);
                ok = __shfl_sync(0xffffffffu, got, 0) != 0;
                ++uses[slot];
                tmem_fence_after();
                if (h == 0 && !whole && final) {
                    // the CTA's last piece of a shared tile: if it is the last
                    // of the tile's pieces to arrive, its sum stays in tensor
                    // memory and the CTA adds the others' partials at its end
                    uint32_t old = 0;
                    if (lane == 0) old = atom_add_acq_rel_gpu(arrive, 1u);
                    old = __shfl_sync(0xffffffffu, old, 0);
                    if (old == np - 1) {
                        keep = true;
                        if (lane == 0) {
                            const int k = fix_n[qtr]++;
                            fix_t[qtr * 2 + k] = t;
                            fix_own[qtr * 2 + k] = 1;
                        }
                        break;
                    }
                }
                const uint32_t tbase = tmem + ((uint32_t)(qtr * 32) << 16) + (uint32_t)(slot * kAccCols);
                for (int32_t c0 = 0; ok && c0 < a.nt; c0 += 16) {
                    uint32_t v[16];
                    tmem_load16(tbase + (uint32_t)c0, v);
                    const int32_t tl = h * a.nt + c0;
                    if (!whole) {
#pragma unroll
                        for (int i = 0; i < 4; ++i)
                            __stcg(reinterpret_cast<float4 *>(mine + (int64_t)(tl / 4 + i) * 128),
                                   make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                               __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3])));
                        continue;
                    }
                    if (row < a.rows)
#pragma unroll
                        for (int k = 0; k < 16; ++k) {
                            const int32_t tok = tok0 + tl + k;
                            if (tok >= a.M) break;
                            const float y = __uint_as_float(v[k]) + bv;
                            if (a.out_f32)
                                reinterpret_cast<float *>(a.out)[(int64_t)tok * a.rows + row] = y;
                            else
                                reinterpret_cast<uint16_t *>(a.out)[(int64_t)tok * a.rows + row] = f32_to_bf16_bits(y);
                        }
                }
                tmem_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[slot]);
            }
            if (!whole && !keep && ok) {
                // the partial is written: mark it ready; a piece that is not
                // the CTA's last counts its arrival only now, and if it is
                // the tile's last, the CTA runs the tile's fixup at its end
                __syncwarp();
                if (lane == 0) {
                    red_add_release_gpu(arrive + 4, 1u);
                    if (!final && atom_add_acq_rel_gpu(arrive, 1u) == np - 1) {
                        const int k = fix_n[qtr]++;
                        fix_t[qtr * 2 + k] = t;
                        fix_own[qtr * 2 + k] = 0;
                    }
                }
            }
        }
    } else if (warp == kProd) {
        // -------------------------------------------------- activations --
        // one stage per half window: stage k holds half k mod nh of window
        // k / nh of the CTA's sequence
        if (lane == 0) {
            const int32_t GT = a.nh * a.nt;
            bool ok = true;
            int32_t k = 0;
            Cursor cu;
            for (cu.begin(R, a.ngrp); !cu.done && ok; cu.next(R, a.ngrp)) {
                const int32_t y0 = (cu.t - cu.rt * a.ngrp) * GT;
                for (int h = 0; h < a.nh && ok; ++h, ++k) {
                    const int s = k % a.nxs, use = k / a.nxs;
                    if (use > 0 && !mbar_wait(&x_empty[s], (uint32_t)((use - 1) & 1), a.err, kErrWaitEmpty)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&x_full[s], xstage);
                    tma_load_2d(xs + (size_t)s * xstage, &xmap, cu.w * 64, y0 + h * a.nt, &x_full[s]);
                }
            }
            // every copy issued lands before the CTA exits (the last use of
            // each stage: its phase has completed, or completes now)
            for (int32_t i = max(0, k - a.nxs); i < k; ++i)
                mbar_wait(&x_full[i % a.nxs], (uint32_t)((i / a.nxs) & 1), a.err, kErrWaitDrain);
        }
    } else {
        // ---------------------------------------------------------- MMA --
        // lane 0 alone waits and issues (the other lanes idle at the warp
        // barrier instead of polling the barriers with it)
        if (lane == 0) {
            bool ok = true;
            int32_t j = 0, k = 0;
            uint32_t uses[2] = {0u, 0u};
            for (int32_t pi = 0; pi < R.n; ++pi) {
                int32_t t, w0, w1;
                R.piece(pi, t, w0, w1);
                for (int32_t w = w0; w < w1; ++w, ++j) {
                    const int sw = j % kWStages;
                    if (ok && !mbar_wait(&w_full[sw], (uint32_t)((j / kWStages) & 1), a.err, kErrWaitFull)) ok = false;
                    const uint32_t wb = smem_addr(ws + sw * kWStage);
                    for (int h = 0; h < a.nh; ++h, ++k) {
                        const int slot = a.nh == 2 ? h : (pi & 1);
                        const int sx = k % a.nxs;
                        if (ok && !mbar_wait(&x_full[sx], (uint32_t)((k / a.nxs) & 1), a.err, kErrWaitFull)) ok = false;
                        if (w == w0 && uses[slot] > 0 && ok &&
                            !mbar_wait(&acc_empty[slot], (uint32_t)((uses[slot] - 1) & 1), a.err, kErrWaitEmpty))
                            ok = false;
                        tmem_fence_after();
                        if (ok) {
                            const uint32_t xb = smem_addr(xs + (size_t)sx * xstage);
#pragma unroll
                            for (int kk = 0; kk < 4; ++kk)
                                umma_bf16(tmem + (uint32_t)(slot * kAccCols), sw128_desc(wb + 32 * kk),
                                          sw128_desc(xb + 32 * kk), a.idesc, (w > w0 || kk > 0) ? 1u : 0u);
                        }
                        umma_commit(&x_empty[sx]);  // frees the half's stage once its MMAs have read it
                        if (w == w1 - 1) {
                            umma_commit(&acc_full[slot]);  // this half's accumulator is complete
                            ++uses[slot];
                        }
                    }
                    umma_commit(&w_empty[sw]);
                }
            }
            // every MMA issued has completed before the tensor memory is freed
            umma_commit(drained);
            mbar_wait(drained, 0u, a.err, kErrWaitDrain);
        }
        __syncwarp();
    }
    // every warp: the main loops are done and every MMA has completed
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    if (warp < kEpi0 + 4) {
        // ------------------------------------------------------- fixup --
        // the shared tiles this CTA arrived last at: the 16 decode warps and
        // the 4 epilogue warps, five per row quarter (a warp reads only its
        // own quarter of tensor memory), add every piece's sum in CTA order
        const int q = warp & 3;
        const int kq = warp < kEpi0 ? warp >> 2 : 4;
        const int32_t GT = a.nh * a.nt;
        for (int k = 0; k < fix_n[q]; ++k) {
            const int32_t t = fix_t[q * 2 + k];
            const bool own = fix_own[q * 2 + k] != 0;
            const int64_t tw = (int64_t)t * a.nwin;
            const int64_t cf = owner_of(tw, G, a.W), cl = owner_of(tw + a.nwin - 1, G, a.W);
            const uint32_t need = (uint32_t)(cl - cf + 1) - (own ? 1u : 0u);
            int got = 1;
            if (lane == 0) {  // every other piece's partial is written
                got = 0;
                for (uint32_t i = 0; i < (1u << 22); ++i) {
                    if (ld_acquire_gpu(a.counters + t * 8 + 4 + q) >= need) {
                        got = 1;
                        break;
                    }
                    __nanosleep(64);
                }
                if (!got) atomicExch(a.err, kErrWaitFull);
            }
            if (!__shfl_sync(0xffffffffu, got, 0)) continue;
            const int64_t row = (int64_t)(t / a.ngrp) * kPfRows + q * 32 + lane;
            const int32_t tok0 = (t % a.ngrp) * GT;
            const float bv = (a.bias && row < a.rows) ? bf16_bits_to_f32(a.bias[row]) : 0.f;
            for (int32_t tl = 16 * kq; tl < GT; tl += 80) {
                const int h = tl / a.nt;
                const uint32_t col = (uint32_t)((a.nh == 2 ? h : ((R.n - 1) & 1)) * kAccCols + tl % a.nt);
                float acc[16];
                for (int64_t c = cf; c <= cl; ++c) {
                    float v[16];
                    if (own && c == (int64_t)blockIdx.x) {
                        uint32_t u[16];
                        tmem_load16(tmem + ((uint32_t)(q * 32) << 16) + col, u);
#pragma unroll
                        for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(u[i]);
                    } else {
                        const int sc = t == cta_start(c, G, a.W) / a.nwin ? 0 : 1;
                        const float4 *pp = reinterpret_cast<const float4 *>(
                            a.part + ((c * 2 + sc) * 4 + q) * GT * 32 + (int64_t)(tl / 4) * 128 + lane * 4);
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const float4 f = __ldcg(pp + i * 32);
                            v[4 * i] = f.x;
                            v[4 * i + 1] = f.y;
                            v[4 * i + 2] = f.z;
                            v[4 * i + 3] = f.w;
                        }
                    }
#pragma unroll
                    for (int i = 0; i < 16; ++i) acc[i] = c == cf ? v[i] : acc[i] + v[i];
                }
                if (row < a.rows)
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int32_t tok = tok0 + tl + i;
                        if (tok >= a.M) break;
                        const float y = acc[i] + bv;
                        if (a.out_f32)
                            reinterpret_cast<float *>(a.out)[(int64_t)tok * a.rows + row] = y;
                        else
                            reinterpret_cast<uint16_t *>(a.out)[(int64_t)tok * a.rows + row] = f32_to_bf16_bits(y);
                    }
            }
        }
    }
    // every warp: the tensor-memory reads done before the free
    tmem_fence_before();
    __syncthreads();
    if (warp == kMma) {
        tmem_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * kAccCols) : "memory");
    }
}

// cuTensorMapEncodeTiled, from the driver through the runtime (no link-time
// dependency on libcuda).
using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_tiled(std::string &msg) {
    static std::once_flag once;
    static EncodeTiled fn = nullptr;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    });
    if (!fn) msg = "dm_prefill: cuTensorMapEncodeTiled is not available from the driver";
    return fn;
}

// The launch geometry of a prefill over M activation rows: groups of at most
// 512 activation rows of equal size, one or two halves each (a multiple of 16
// rows, the tensor-memory loads' width).
struct PfPlan {
    int32_t nt, nh, ngrp, nxs;
    int64_t nrt, ntiles, nwin, W, grid;
    int64_t counter_bytes, part_bytes, smem;
};

PfPlan plan_prefill(const dm_tensor *t, int64_t M) {
    PfPlan P{};
    P.ngrp = (int32_t)((M + kGroupMax - 1) / kGroupMax);
    const int64_t per = (M + P.ngrp - 1) / P.ngrp;
    P.nh = per > kHalfMax ? 2 : 1;
    P.nt = (int32_t)(((per + P.nh - 1) / P.nh + 15) / 16 * 16);
    const int64_t xstage = (int64_t)P.nt * 128;  // one half window
    P.nxs = (int32_t)std::min<int64_t>(kMaxXStages, kXBudget / xstage);
    P.nrt = (t->L.rows + kPfRows - 1) / kPfRows;
    P.ntiles = P.nrt * P.ngrp;
    P.nwin = t->L.NB * 16;
    P.W = P.ntiles * P.nwin;
    P.grid = std::min<int64_t>(t->sms, P.W);
    P.counter_bytes = (P.ntiles * 8 * (int64_t)sizeof(uint32_t) + 255) / 256 * 256;
    P.part_bytes = P.grid * 2 * kPfRows * (int64_t)P.nh * P.nt * (int64_t)sizeof(float);
    P.smem = 1024 + P.nxs * xstage + kFixedSmem;
    return P;
}

}  // namespace

int64_t prefill_workspace_bytes(const dm_tensor *t, int64_t M) {
    const PfPlan P = plan_prefill(t, M);
    return P.counter_bytes + P.part_bytes;
}

int launch_prefill_sip(const dm_tensor *t, const uint16_t *x, int64_t M, const uint16_t *bias, void *out,
                       int out_f32, uint8_t *work, int64_t work_bytes, void *stream, std::string &msg) {
    const TensorLayout &L = t->L;
    if (!L.fast_sip || !t->d_rowdir) {
        msg = "dm_prefill: needs a sip tensor (the fast path)";
        return DM_EINVAL;
    }
    if (L.nparts > kMaxParts) {
        msg = "dm_prefill: a fused tensor of more than " + std::to_string(kMaxParts) + " parts";
        return DM_EINVAL;
    }
    if (M > (int64_t)INT32_MAX / 2) {
        msg = "dm_prefill: too many activation rows";
        return DM_EINVAL;
    }
    if (work_bytes < prefill_workspace_bytes(t, M) || (reinterpret_cast<uintptr_t>(work) & 255) ||
        (reinterpret_cast<uintptr_t>(x) & 15)) {
        msg = "dm_prefill: workspace too small or not 256-byte aligned, or activations not 16-byte aligned";
        return DM_EINVAL;
    }
    if (L.units == 0) return DM_OK;
    const PfPlan P = plan_prefill(t, M);
    if (P.nxs < 2 || P.smem > kSmemLimit) {
        msg = "dm_prefill: the shared-memory plan does not fit";
        return DM_EINVAL;
    }
    EncodeTiled enc = encode_tiled(msg);
    if (!enc) return DM_ECUDA;
    CUtensorMap xmap;
    const cuuint64_t gdim[2] = {(cuuint64_t)L.C, (cuuint64_t)M};
    const cuuint64_t gstride[1] = {(cuuint64_t)L.C * 2};
    const cuuint32_t box[2] = {64u, (cuuint32_t)P.nt};
    const cuuint32_t estride[2] = {1u, 1u};
    CUresult cr = enc(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t *>(x), gdim, gstride, box, estride,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) {
        msg = "dm_prefill: cuTensorMapEncodeTiled failed (" + std::to_string((int)cr) + ")";
        return DM_ECUDA;
    }
    // a per-device attribute: one bit per device (64 and up: every launch)
    static std::atomic<uint64_t> attr{0};
    const uint64_t dev_bit = t->device >= 0 && t->device < 64 ? 1ull << t->device : 0ull;
    if (!dev_bit || !(attr.load() & dev_bit)) {
        cudaError_t e = cudaFuncSetAttribute(prefill_sip_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
        if (e != cudaSuccess) {
            msg = std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e);
            return DM_ECUDA;
        }
        attr.fetch_or(dev_bit);
    }
    uint32_t *counters = reinterpret_cast<uint32_t *>(work);
    cudaError_t e = cudaMemsetAsync(counters, 0, (size_t)P.counter_bytes, (cudaStream_t)stream);
    if (e != cudaSuccess) {
        msg = std::string("dm_prefill: cudaMemsetAsync: ") + cudaGetErrorString(e);
        return DM_ECUDA;
    }
    PfArgs a{};
    a.data = t->d_data;
    a.rowdir = reinterpret_cast<const uint2 *>(t->d_rowdir);
    a.rows = L.rows;
    a.NB = L.NB;
    a.M = (int32_t)M;
    a.ngrp = P.ngrp;
    a.nt = P.nt;
    a.nh = P.nh;
    a.ntiles = P.ntiles;
    a.nwin = (int32_t)P.nwin;
    a.W = P.W;
    a.nxs = P.nxs;
    a.idesc = idesc_f16(kPfRows, P.nt);
    a.bias = bias;
    a.out = out;
    a.out_f32 = out_f32;
    a.counters = counters;
    a.part = reinterpret_cast<float *>(work + P.counter_bytes);
    a.err = t->S.err;
    for (int p = 0; p < kMaxParts; ++p)
        for (int k = 0; k < 4; ++k) a.tabs[p][k] = L.part_tabs[p][k];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)P.grid);
    cfg.blockDim = dim3(kPfThreads);
    cfg.dynamicSmemBytes = (size_t)P.smem;
    cfg.stream = (cudaStream_t)stream;
    cfg.numAttrs = 0;
    e = cudaLaunchKernelEx(&cfg, prefill_sip_kernel, xmap, a);
    if (e != cudaSuccess) {
        msg = std::string("prefill_sip_kernel: ") + cudaGetErrorString(e);
        return DM_ECUDA;
    }
    return DM_OK;
}

}  // namespace dm
