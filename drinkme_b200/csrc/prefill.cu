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
//     operand) by up to 256 activation rows (the MMA's N: the activations are
//     the B operand), over the whole K; its fp32 accumulator takes 256 of the
//     CTA's 512 tensor-memory columns, so two accumulators alternate and one
//     tile's epilogue runs under the next tile's MMAs.
//   * Persistent stream-K over K windows of 64: one CTA per SM; the windows of
//     every tile, tile after tile (a weight row tile's activation tiles next to
//     each other, so its compressed bytes come from L2 the second time), are
//     split evenly over the CTAs. A CTA's first and last tiles may be shared
//     with its neighbours (PIECES); it runs those first. A piece's fp32
//     partial goes to the workspace, and for each quarter of the tile's rows
//     the last piece to arrive (an acquire-release counter) adds every
//     piece's partial in CTA order and writes the outputs.
//   * Warps 0-7 decode: a lane pair per weight row, lane h taking weights
//     [32h, 32h + 32) of each window, from the loader's code planes with the
//     GEMV's byte-parallel table lookups (escaped weights come out as sign |
//     0 | mantissa), into the 128-byte-swizzled K-major tile the tensor core
//     reads. An escaped weight's terminal exponent is its rank among the row
//     block's escapes: the lane pair counts code-7 nibbles as it goes and
//     rewrites each escaped weight whole from its literal byte and the row's
//     terminal stream, staged per block column in shared memory. The
//     compressed operands of the next four windows are staged by cp.async
//     into a shared-memory ring (the lanes hold no loads in flight, so the
//     per-window barrier release and proxy fence never wait for them); the
//     row-block directory entry of the next block column is prefetched a
//     block column ahead.
//   * Warp 12 loads each activation window with one TMA tensor copy (no
//     multicast) in the same swizzled layout; lane 0 of warp 13 owns the MMA
//     issue (kind::f16, M = 128, N = tokens, K = 16) and commits each window
//     to the barriers that free its stages; warp 13 owns the tensor memory.
//   * Warps 8-11 read the accumulators (tcgen05.ld, a lane per weight row),
//     add the bias in fp32, round once and store; or write a piece's partial
//     (activation-row major, so a warp's store is one 128-byte line). Only one
//     lane of a warp polls a barrier.
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

constexpr int kPfRows = 128;      // weight rows per tile (MMA M)
constexpr int kPfTokMax = 256;    // activation rows per tile, at most (MMA N)
constexpr int kXStages = 3;       // activation windows in flight
constexpr int kWStages = 3;       // decoded weight windows in flight
constexpr int kPfDecWarps = 8;    // a lane pair per weight row, 16 rows per warp
constexpr int kPfEpi0 = 8;        // warps 8-11: the epilogue (tensor-memory lane quarters 0-3)
constexpr int kPfProd = 12;       // warp 12: activation TMA
constexpr int kPfMma = 13;        // warp 13: tensor memory and MMA issue
constexpr int kPfThreads = 14 * 32;
constexpr int kAhead = 4;         // windows of compressed operands in flight (a cp.async ring)
constexpr int kOpRow = 96;        // per row and window: 64 literal bytes, 4 code words, 2 bit-2 words
constexpr int kOpStage = kPfRows * kOpRow;
constexpr int kWStage = kPfRows * 128;    // 16 KB: 128 rows x 64 bf16
constexpr int kXStage = kPfTokMax * 128;  // 32 KB: 256 rows x 64 bf16
constexpr int kTermRing = 4;              // block columns of staged terminal bytes
constexpr int kTermRow = 64;              // terminal bytes staged per row (the rest read from HBM)
constexpr int kTermStage = kPfRows * kTermRow;
constexpr int kAccCols = 256;             // tensor-memory columns per accumulator
constexpr int kMaxParts = 8;

constexpr int kOffX = 0;
constexpr int kOffW = kOffX + kXStages * kXStage;
constexpr int kOffOp = kOffW + kWStages * kWStage;
constexpr int kOffTerm = kOffOp + kAhead * kOpStage;
constexpr int kOffBar = kOffTerm + kTermRing * kTermStage;
constexpr int kNumBars = 2 * kXStages + 2 * kWStages + 5;
constexpr int kOffTmem = kOffBar + kNumBars * 8;
constexpr int kOffTabs = kOffTmem + 16;
constexpr int kSmemBytes = kOffTabs + kMaxParts * 16 + 1024;  // + alignment slack

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
// 256 ns sleep between tries (about 2^16 tries: tens of milliseconds), so the
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

// 16 bytes global -> shared, asynchronously (the LDGSTS path, L2 only).
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
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

// The selectors of 16 codes (quarter t of a 64-weight window) from a row
// block's code planes: v = its low-two-bit word, P = its bit-2 word (the
// GEMV's code_selectors).
__device__ __forceinline__ void selectors16(uint32_t v, uint32_t P, uint32_t rl, uint32_t rh, uint32_t &s0,
                                            uint32_t &s1) {
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

// Bit 4i set where nibble i of a selector word holds code 7 (an escape).
__device__ __forceinline__ uint32_t escape_nibbles(uint32_t s) { return s & (s >> 1) & (s >> 2) & 0x11111111u; }

struct PfArgs {
    const uint8_t *data;
    const uint2 *rowdir;     // [16-row padded rows][NB]: stream offset (16-byte units), nesc | part << 16
    int64_t rows, NB;
    int32_t M, ntok, ntt;    // real activation rows, activation tiles, activation rows per tile (MMA N)
    int32_t nparts;
    int64_t ntiles, W;       // tiles (row tiles x activation tiles), all windows
    int32_t nwin;            // windows per tile
    uint32_t idesc;
    const uint16_t *bias;
    void *out;               // [M][rows]
    int32_t out_f32;
    float *part;             // [grid][2][128][ntt]: a CTA's partials of its first / last tile
    int *counters;           // [ntiles][4], zero on entry
    int *err;
    uint32_t tabs[kMaxParts][4];
};

// The CTA's windows [x0, x1) of the whole sequence (tile-major), as PIECES:
// its first tile when partial, its last tile when partial, then its whole
// tiles in order.
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
        if (pB) {
            if (i == 0) {
                t = tB;
                w0 = 0;
                w1 = (int32_t)(x1 - (int64_t)tB * nwin);
                return;
            }
            --i;
        }
        t = (pA ? tA + 1 : tA) + i;
        w0 = 0;
        w1 = nwin;
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
    __device__ void at_piece(const Range &R, int32_t ntok) {
        R.piece(pi, t, w, w1);
        rt = t / ntok;
    }
    __device__ void begin(const Range &R, int32_t ntok) {
        pi = 0;
        done = R.n == 0;
        t = rt = w = w1 = 0;
        if (!done) at_piece(R, ntok);
    }
    __device__ void next(const Range &R, int32_t ntok) {
        if (++w < w1) return;
        if (++pi >= R.n) {
            done = true;
            return;
        }
        at_piece(R, ntok);
    }
    // the first window (and its weight row tile) of the next block column
    // (segment) after this one
    __device__ bool next_segment(const Range &R, int32_t ntok, int32_t &rt2, int32_t &w2) const {
        const int32_t e = ((w >> 4) + 1) << 4;
        if (e < w1) {
            rt2 = rt;
            w2 = e;
            return true;
        }
        if (pi + 1 >= R.n) return false;
        int32_t t2, x;
        R.piece(pi + 1, t2, w2, x);
        rt2 = t2 / ntok;
        return true;
    }
};

__global__ void __launch_bounds__(kPfThreads, 1) prefill_sip_kernel(const __grid_constant__ CUtensorMap xmap, PfArgs a) {
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned tiles (the swizzle pattern follows address bits 7-9)
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *xs = smem + kOffX;
    uint8_t *ws = smem + kOffW;
    uint8_t *ops = smem + kOffOp;     // [kAhead][128 rows][kOpRow]: compressed operands in flight
    uint8_t *term = smem + kOffTerm;  // [kTermRing][128 rows][64 bytes]
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + kOffBar);
    uint64_t *x_full = bar, *x_empty = bar + kXStages, *w_full = bar + 2 * kXStages, *w_empty = w_full + kWStages;
    uint64_t *acc_full = w_empty + kWStages, *acc_empty = acc_full + 2, *drained = acc_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kOffTmem);
    uint32_t *tabs = reinterpret_cast<uint32_t *>(smem + kOffTabs);  // [kMaxParts][4]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t G = gridDim.x;
    Range R;
    R.init(blockIdx.x, G, a.W, a.nwin);
    if (threadIdx.x == 0) {
        for (int s = 0; s < kXStages; ++s) {
            mbar_init(&x_full[s], 1);
            mbar_init(&x_empty[s], 1);
        }
        for (int s = 0; s < kWStages; ++s) {
            mbar_init(&w_full[s], kPfDecWarps);
            mbar_init(&w_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);
        }
        mbar_init(drained, 1);
        mbar_fence_init();
    }
    if (warp == kPfProd && lane < kMaxParts * 4) tabs[lane] = (&a.tabs[0][0])[lane];
    if (warp == kPfMma) {
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

    if (warp < kPfDecWarps) {
        // ------------------------------------------------------ decode --
        // a lane pair per weight row; lane h decodes weights [32h, 32h + 32)
        // of every window (the GEMV's quarters 2h and 2h + 1 of a quad)
        const int r = warp * 16 + (lane >> 1);
        const int h = lane & 1;
        const uint32_t sw = (uint32_t)(r & 7);
        bool ok = true;
        // the load cursor runs kAhead windows before the decode position,
        // staging each window's compressed operands by cp.async into ring
        // slot (window mod kAhead) of this row: nothing the decoder waits on
        // is a load in flight of its own (a release or a proxy fence would
        // wait for those)
        Cursor cl;
        cl.begin(R, a.ntok);
        // segments the load cursor has entered; the ring of staged terminal
        // bytes has kTermRing slots, and the load cursor is at most three
        // segment starts ahead of the decode position (within kAhead = 4
        // windows: a piece start, the next piece's start, one block column
        // boundary), so no slot is overwritten while in use
        int32_t seg_load = -1;
        int32_t seg_t = -1, seg_bc = -1;
        uint2 dir_cur = make_uint2(0, 0), dir_next = make_uint2(0, 0);
        bool has_next = false;
        int32_t nxt_rt = 0, nxt_w = 0;
        auto dir_load = [&](int32_t rt, int32_t bc) -> uint2 {
            const int64_t row = (int64_t)rt * kPfRows + r;
            if (row >= a.rows) return make_uint2(0, 0);
            return __ldg(a.rowdir + row * NB + bc);
        };
        // the load cursor's window into ring slot `nload` mod kAhead: a new
        // segment takes the prefetched directory entry, prefetches the next
        // one and stages its terminal bytes (lane h: bytes [32h, 32h + 32));
        // one cp.async group per window. Per row and window the slot holds
        // the 64 literal bytes, the four code-plane words and the two bit-2
        // words.
        int32_t nload = 0;  // windows the load cursor has issued
        auto load_window = [&]() {
            const int32_t bc = cl.w >> 4;
            const bool exists = (int64_t)cl.rt * kPfRows + r < a.rows;
            if (cl.t != seg_t || bc != seg_bc) {
                if (has_next && nxt_rt == cl.rt && (nxt_w >> 4) == bc)
                    dir_cur = dir_next;
                else
                    dir_cur = dir_load(cl.rt, bc);
                has_next = cl.next_segment(R, a.ntok, nxt_rt, nxt_w);
                if (has_next) dir_next = dir_load(nxt_rt, nxt_w >> 4);
                ++seg_load;
                seg_t = cl.t;
                seg_bc = bc;
                if (exists) {
                    uint8_t *dst = term + (seg_load & (kTermRing - 1)) * kTermStage + r * kTermRow + 32 * h;
                    const uint8_t *src = a.data + (size_t)dir_cur.x * 16 + 1408 + 32 * h;
                    cp_async16(dst, src);
                    cp_async16(dst + 16, src + 16);
                }
            }
            if (exists) {
                const int q = cl.w & 15;
                const uint8_t *lit = a.data + (size_t)dir_cur.x * 16;
                uint8_t *o = ops + (nload % kAhead) * kOpStage + r * kOpRow;
                cp_async16(o + 32 * h, lit + 64 * q + 32 * h);
                cp_async16(o + 32 * h + 16, lit + 64 * q + 32 * h + 16);
                cp_async8(o + 64 + 8 * h, lit + 1024 + 16 * q + 8 * h);
                cp_async4(o + 80 + 4 * h, lit + 1024 + 256 + 8 * q + 4 * h);
            }
            cp_async_commit();
            ++nload;
        };
#pragma unroll 1
        for (int i = 0; i < kAhead && !cl.done; ++i) {
            load_window();
            cl.next(R, a.ntok);
        }
        int32_t seg_dec = -1;  // segment of the decode position
        uint32_t run = 0;      // escapes of this row block before the current window
        int32_t j = 0;         // window sequence number (its stage)
        Cursor cd;
        cd.begin(R, a.ntok);
        int32_t dseg_t = -1, dseg_bc = -1;
        uint2 dir = make_uint2(0, 0);  // the decode position's row block: stream offset, nesc | part << 16
        bool real = false;             // its row exists
        // decode window j (ring slot j mod kAhead), then load the window
        // kAhead ahead into the slot it frees
        while (!cd.done) {
            const int32_t bc = cd.w >> 4;
            if (cd.t != dseg_t || bc != dseg_bc) {
                ++seg_dec;
                dseg_t = cd.t;
                dseg_bc = bc;
                run = 0;
                real = (int64_t)cd.rt * kPfRows + r < a.rows;
                dir = dir_load(cd.rt, bc);  // an L1 hit: the load cursor read it a few windows ago
                // a piece that starts inside a block column: the escapes of
                // the block's earlier windows come before this window's ranks;
                // lane h counts whole windows h, h + 2, ... below q0, two
                // windows' loads at a time
                const int q0 = cd.w & 15;
                if (q0 > 0) {
                    uint32_t pre = 0;
                    if (real) {
                        const uint8_t *cb = a.data + (size_t)dir.x * 16 + 1024;
                        for (int base = h; base < q0; base += 4) {
                            uint4 cw[2];
                            uint2 pw[2];
#pragma unroll
                            for (int i = 0; i < 2; ++i) {
                                const int qq = base + 2 * i;
                                if (qq < q0) {
                                    cw[i] = __ldg(reinterpret_cast<const uint4 *>(cb + 16 * qq));
                                    pw[i] = __ldg(reinterpret_cast<const uint2 *>(cb + 256 + 8 * qq));
                                }
                            }
#pragma unroll
                            for (int i = 0; i < 2; ++i) {
                                if (base + 2 * i < q0) {
                                    uint32_t s0, s1, s2, s3;
                                    selectors16(cw[i].x, pw[i].x, 2u, 1u, s0, s1);
                                    selectors16(cw[i].y, pw[i].x, 0u, 31u, s2, s3);
                                    pre += __popc(escape_nibbles(s0)) + __popc(escape_nibbles(s1)) +
                                           __popc(escape_nibbles(s2)) + __popc(escape_nibbles(s3));
                                    selectors16(cw[i].z, pw[i].y, 2u, 1u, s0, s1);
                                    selectors16(cw[i].w, pw[i].y, 0u, 31u, s2, s3);
                                    pre += __popc(escape_nibbles(s0)) + __popc(escape_nibbles(s1)) +
                                           __popc(escape_nibbles(s2)) + __popc(escape_nibbles(s3));
                                }
                            }
                        }
                    }
                    run = pre + __shfl_xor_sync(0xffffffffu, pre, 1);
                }
            }
            // this window's group (and, at a segment start, its terminals) landed
            cp_async_wait(nload - j - 1);
            __syncwarp();
            const int s = j % kWStages, use = j / kWStages;
            if (use > 0 && ok) {  // lane 0 polls; the warp barrier orders the others after it
                int got = 1;
                if (lane == 0) got = mbar_wait(&w_empty[s], (uint32_t)((use - 1) & 1), a.err, kErrWaitEmpty);
                ok = __shfl_sync(0xffffffffu, got, 0) != 0;
            }
            uint8_t *rowp = ws + s * kWStage + r * 128;
            const uint8_t *o = ops + (j % kAhead) * kOpStage + r * kOpRow;
            const uint32_t part = dir.y >> 16;
            const uint32_t nesc = dir.y & 0xFFFFu;
            const uint32_t *tb = tabs + 4 * (part < kMaxParts ? part : 0);
            // code 7 decodes to sign | exponent 0 | mantissa; escaped weights
            // are rewritten whole below
            const uint32_t th0 = tb[0], th1 = tb[1] & 0x00FFFFFFu, tl0 = tb[2], tl1 = tb[3] & 0x00FFFFFFu;
            uint32_t p[16];
            uint32_t e0 = 0, e1 = 0, e2 = 0, e3 = 0;
            if (real) {
                const uint4 L0 = *reinterpret_cast<const uint4 *>(o + 32 * h);
                const uint4 L1 = *reinterpret_cast<const uint4 *>(o + 32 * h + 16);
                const uint2 c = *reinterpret_cast<const uint2 *>(o + 64 + 8 * h);
                const uint32_t P = *reinterpret_cast<const uint32_t *>(o + 80 + 4 * h);
                uint32_t s0, s1, s2, s3;
                selectors16(c.x, P, 2u, 1u, s0, s1);   // quarter 2h (even)
                selectors16(c.y, P, 0u, 31u, s2, s3);  // quarter 2h + 1 (odd)
                dec4(L0.x, s0, th0, th1, tl0, tl1, p[0], p[1]);
                dec4(L0.y, s0 >> 16, th0, th1, tl0, tl1, p[2], p[3]);
                dec4(L0.z, s1, th0, th1, tl0, tl1, p[4], p[5]);
                dec4(L0.w, s1 >> 16, th0, th1, tl0, tl1, p[6], p[7]);
                dec4(L1.x, s2, th0, th1, tl0, tl1, p[8], p[9]);
                dec4(L1.y, s2 >> 16, th0, th1, tl0, tl1, p[10], p[11]);
                dec4(L1.z, s3, th0, th1, tl0, tl1, p[12], p[13]);
                dec4(L1.w, s3 >> 16, th0, th1, tl0, tl1, p[14], p[15]);
                e0 = escape_nibbles(s0);
                e1 = escape_nibbles(s1);
                e2 = escape_nibbles(s2);
                e3 = escape_nibbles(s3);
            } else {
#pragma unroll
                for (int k = 0; k < 16; ++k) p[k] = 0u;
            }
#pragma unroll
            for (int k = 0; k < 4; ++k)
                *reinterpret_cast<uint4 *>(rowp + ((((uint32_t)(4 * h + k)) ^ sw) << 4)) =
                    make_uint4(p[4 * k], p[4 * k + 1], p[4 * k + 2], p[4 * k + 3]);
            // escapes: rank among the row block's escapes -> terminal
            // exponent; the weight is written whole from its literal byte
            // (independent loads and one store each, no read-modify-write)
            const uint32_t mine = __popc(e0) + __popc(e1) + __popc(e2) + __popc(e3);
            const uint32_t other = __shfl_xor_sync(0xffffffffu, mine, 1);
            uint32_t rank = run + (h ? other : 0u);
            run += mine + other;
            if (mine) {
                const uint8_t *ts = term + (seg_dec & (kTermRing - 1)) * kTermStage + r * kTermRow;
                const uint8_t *lb = o + 32 * h;
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    uint32_t m = g == 0 ? e0 : (g == 1 ? e1 : (g == 2 ? e2 : e3));
                    while (m) {
                        const uint32_t k = 8u * g + ((uint32_t)(__ffs(m) - 1) >> 2);  // weight of the 32
                        m &= m - 1;
                        uint16_t w16 = 0;  // past a truncated terminal stream: +0, as the GEMV decodes it
                        if (rank < nesc) {
                            const uint32_t ex = rank < (uint32_t)kTermRow ? ts[rank]
                                                                          : a.data[(size_t)dir.x * 16 + 1408 + rank];
                            const uint32_t lit = lb[k];
                            w16 = (uint16_t)(((lit & 0x80u) << 8) | (ex << 7) | (lit & 0x7Fu));
                        }
                        *reinterpret_cast<uint16_t *>(
                            rowp + (((((uint32_t)(4 * h) + (k >> 3)) ^ sw) << 4) | ((k & 7u) << 1))) = w16;
                        ++rank;
                    }
                }
            }
            fence_proxy_async_smem();  // these generic writes, before the tensor core's async reads
            __syncwarp();
            if (lane == 0) mbar_arrive(&w_full[s]);
            // every lane has read its slot: it takes the window kAhead ahead
            if (!cl.done) {
                load_window();
                cl.next(R, a.ntok);
            }
            cd.next(R, a.ntok);
            ++j;
        }
        cp_async_wait(0);
    } else if (warp >= kPfEpi0 && warp < kPfEpi0 + 4) {
        // ---------------------------------------------------- epilogue --
        const int qtr = warp - kPfEpi0;  // tensor-memory lanes 32 qtr .. 32 qtr + 31
        bool ok = true;
        for (int32_t pi = 0; pi < R.n; ++pi) {
            int32_t t, w0, w1;
            R.piece(pi, t, w0, w1);
            const int b = pi & 1;
            if (ok) {  // a long wait: lane 0 polls with a backoff, the others idle at the warp barrier
                int got = 1;
                if (lane == 0) got = mbar_wait_backoff(&acc_full[b], (uint32_t)((pi >> 1) & 1), a.err, kErrWaitFull);
                ok = __shfl_sync(0xffffffffu, got, 0) != 0;
            }
            tmem_fence_after();
            const bool whole = w0 == 0 && w1 == a.nwin;
            const int64_t row = (int64_t)(t / a.ntok) * kPfRows + qtr * 32 + lane;
            const int32_t tok0 = (t % a.ntok) * a.ntt;
            const float bv = (a.bias && row < a.rows) ? bf16_bits_to_f32(a.bias[row]) : 0.f;
            const int slot = t == R.tA ? 0 : 1;
            // a piece's partial: [activation row][weight row], so each store of
            // one activation row by the warp's 32 lanes (rows) is one 128-byte line
            float *mine = a.part + ((int64_t)blockIdx.x * 2 + slot) * a.ntt * kPfRows + qtr * 32 + lane;
            for (int32_t c0 = 0; c0 < a.ntt; c0 += 16) {
                uint32_t v[16];
                tmem_load16(tmem + ((uint32_t)(qtr * 32) << 16) + (uint32_t)(b * kAccCols + c0), v);
                if (!ok) continue;
                if (whole) {
                    if (row < a.rows)
#pragma unroll
                        for (int k = 0; k < 16; ++k) {
                            const int32_t tok = tok0 + c0 + k;
                            if (tok >= a.M) break;
                            const float y = __uint_as_float(v[k]) + bv;
                            if (a.out_f32)
                                reinterpret_cast<float *>(a.out)[(int64_t)tok * a.rows + row] = y;
                            else
                                reinterpret_cast<uint16_t *>(a.out)[(int64_t)tok * a.rows + row] = f32_to_bf16_bits(y);
                        }
                } else {
#pragma unroll
                    for (int k = 0; k < 16; ++k) __stcg(mine + (int64_t)(c0 + k) * kPfRows, __uint_as_float(v[k]));
                }
            }
            tmem_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
            if (whole || !ok) continue;
            // a shared tile: the last of its pieces to arrive (per row quarter)
            // adds every piece's partial in CTA order
            const int64_t tw = (int64_t)t * a.nwin;
            const int64_t cf = owner_of(tw, G, a.W), cl = owner_of(tw + a.nwin - 1, G, a.W);
            __syncwarp();
            int last = 0;
            if (lane == 0) {
                const uint32_t old = atom_add_acq_rel_gpu(reinterpret_cast<uint32_t *>(a.counters + t * 4 + qtr), 1u);
                last = old == (uint32_t)(cl - cf);
                if (last) a.counters[t * 4 + qtr] = 0;
            }
            last = __shfl_sync(0xffffffffu, last, 0);
            if (!last) continue;
            for (int32_t c0 = 0; c0 < a.ntt; c0 += 16) {
                float acc[16];
                for (int64_t c = cf; c <= cl; ++c) {
                    const int sc = t == cta_start(c, G, a.W) / a.nwin ? 0 : 1;
                    const float *pp = a.part + (c * 2 + sc) * a.ntt * kPfRows + (int64_t)c0 * kPfRows + qtr * 32 + lane;
#pragma unroll
                    for (int k = 0; k < 16; ++k) {
                        const float x = __ldcg(pp + k * kPfRows);
                        acc[k] = c == cf ? x : acc[k] + x;
                    }
                }
                if (row < a.rows)
#pragma unroll
                    for (int k = 0; k < 16; ++k) {
                        const int32_t tok = tok0 + c0 + k;
                        if (tok >= a.M) break;
                        const float y = acc[k] + bv;
                        if (a.out_f32)
                            reinterpret_cast<float *>(a.out)[(int64_t)tok * a.rows + row] = y;
                        else
                            reinterpret_cast<uint16_t *>(a.out)[(int64_t)tok * a.rows + row] = f32_to_bf16_bits(y);
                    }
            }
        }
    } else if (warp == kPfProd) {
        // -------------------------------------------------- activations --
        if (lane == 0) {
            const uint32_t bytes = (uint32_t)a.ntt * 128u;
            bool ok = true;
            int32_t j = 0;
            Cursor cu;
            for (cu.begin(R, a.ntok); !cu.done && ok; cu.next(R, a.ntok), ++j) {
                const int s = j % kXStages, use = j / kXStages;
                if (use > 0 && !mbar_wait(&x_empty[s], (uint32_t)((use - 1) & 1), a.err, kErrWaitEmpty)) ok = false;
                if (!ok) break;
                mbar_arrive_expect_tx(&x_full[s], bytes);
                tma_load_2d(xs + s * kXStage, &xmap, cu.w * 64, (cu.t - cu.rt * a.ntok) * a.ntt, &x_full[s]);
            }
            // every copy issued lands before the CTA exits (the last use of
            // each stage: its phase has completed, or completes now)
            for (int32_t i = std::max<int32_t>(0, j - kXStages); i < j; ++i)
                mbar_wait(&x_full[i % kXStages], (uint32_t)((i / kXStages) & 1), a.err, kErrWaitDrain);
        }
    } else {
        // ---------------------------------------------------------- MMA --
        // lane 0 alone waits and issues (the other lanes idle at the warp
        // barrier instead of polling the barriers with it)
        if (lane == 0) {
            bool ok = true;
            int32_t j = 0;
            for (int32_t pi = 0; pi < R.n; ++pi) {
                int32_t t, w0, w1;
                R.piece(pi, t, w0, w1);
                const int b = pi & 1;
                if (pi >= 2 && ok && !mbar_wait(&acc_empty[b], (uint32_t)(((pi >> 1) - 1) & 1), a.err, kErrWaitEmpty))
                    ok = false;
                tmem_fence_after();
                for (int32_t w = w0; w < w1; ++w, ++j) {
                    const int sx = j % kXStages, sw = j % kWStages;
                    if (ok && !mbar_wait(&x_full[sx], (uint32_t)((j / kXStages) & 1), a.err, kErrWaitFull)) ok = false;
                    if (ok && !mbar_wait(&w_full[sw], (uint32_t)((j / kWStages) & 1), a.err, kErrWaitFull)) ok = false;
                    tmem_fence_after();
                    if (ok) {
                        const uint32_t wb = smem_addr(ws + sw * kWStage), xb = smem_addr(xs + sx * kXStage);
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            umma_bf16(tmem + (uint32_t)(b * kAccCols), sw128_desc(wb + 32 * k), sw128_desc(xb + 32 * k),
                                      a.idesc, (w > w0 || k > 0) ? 1u : 0u);
                    }
                    umma_commit(&w_empty[sw]);  // frees the stages once these MMAs have read them
                    umma_commit(&x_empty[sx]);
                }
                umma_commit(&acc_full[b]);
            }
            // every MMA issued has completed before the tensor memory is freed
            umma_commit(drained);
            mbar_wait(drained, 0u, a.err, kErrWaitDrain);
        }
        __syncwarp();
    }
    // every warp: the epilogue's tensor-memory reads done before the free
    tmem_fence_before();
    __syncthreads();
    if (warp == kPfMma) {
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

// The launch geometry of a prefill over M activation rows.
struct PfPlan {
    int32_t ntt, ntok;
    int64_t nrt, ntiles, nwin, W, grid;
    int64_t counter_bytes, part_bytes;
};

PfPlan plan_prefill(const dm_tensor *t, int64_t M) {
    PfPlan P{};
    P.ntt = (int32_t)std::min<int64_t>(kPfTokMax, (M + 15) / 16 * 16);  // whole 16-column tensor-memory loads
    P.ntok = (int32_t)((M + P.ntt - 1) / P.ntt);
    P.nrt = (t->L.rows + kPfRows - 1) / kPfRows;
    P.ntiles = P.nrt * P.ntok;
    P.nwin = t->L.NB * 16;
    P.W = P.ntiles * P.nwin;
    P.grid = std::min<int64_t>(t->sms, P.W);
    P.counter_bytes = (P.ntiles * 4 * (int64_t)sizeof(int) + 255) / 256 * 256;
    P.part_bytes = P.grid * 2 * kPfRows * P.ntt * (int64_t)sizeof(float);
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
    EncodeTiled enc = encode_tiled(msg);
    if (!enc) return DM_ECUDA;
    CUtensorMap xmap;
    const cuuint64_t gdim[2] = {(cuuint64_t)L.C, (cuuint64_t)M};
    const cuuint64_t gstride[1] = {(cuuint64_t)L.C * 2};
    const cuuint32_t box[2] = {64u, (cuuint32_t)P.ntt};
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
        cudaError_t e = cudaFuncSetAttribute(prefill_sip_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
        if (e != cudaSuccess) {
            msg = std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e);
            return DM_ECUDA;
        }
        attr.fetch_or(dev_bit);
    }
    int *counters = reinterpret_cast<int *>(work);
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
    a.ntok = P.ntok;
    a.ntt = P.ntt;
    a.nparts = L.nparts;
    a.ntiles = P.ntiles;
    a.nwin = (int32_t)P.nwin;
    a.W = P.W;
    a.idesc = idesc_f16(kPfRows, P.ntt);
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
    cfg.dynamicSmemBytes = (size_t)kSmemBytes;
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
