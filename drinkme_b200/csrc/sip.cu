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
//   * A CTA = 1 producer warp, 4 groups of 4 consumer warps and 1 epilogue
//     warp, one CTA per SM. The CTA is a stream-K WORKER: the units (16 rows x
//     1 block column, see layout.cpp) of the tensor in tile-major order are
//     split over the CTAs by a table of starts (the last CTAs to be
//     dispatched get a little less). Consecutive CTAs therefore share at most
//     one tile at each boundary; the CTA processes those (at most two)
//     PARTIAL tiles first and its whole tiles after them. Small tensors use
//     whole tiles per CTA instead.
//   * The producer stages each unit with ONE 1-D bulk copy (the TMA engine)
//     into a ring of shared-memory slots, completing an mbarrier; the
//     activations of every block column are either resident for the launch
//     (RES) or staged with each unit (one 2 KB bulk copy per activation
//     row). Unit i of the CTA's sequence goes to group i mod 4; the 4 warps
//     of the group share it, each decoding a quarter of its k range.
//   * A consumer decodes its unit straight into MMA operands: the weights
//     are the A operand (m = 16 output rows) of mma.m16n8k16 bf16 with fp32
//     accumulate, the activations the B operand (n = 8 = up to 8 activation
//     rows). Lane (g, t) decodes rows g and g + 8 of the unit at
//     k = 64q + 16t + [0, 16); warp w of a group takes q in [4w, 4w + 4).
//   * Decode is byte-parallel: the tier-0 codes come from the loader's two
//     code planes as PRMT selectors (a mask, a rotate and an OR per 8 codes),
//     then one PRMT per 4 weights looks four exponents up in an 8-byte
//     table, and two LOP3 + two PRMT merge sign, exponent and mantissa into
//     the bf16 pairs of the MMA operand. The table's escape entry makes a
//     weight whose code is 7 decode to exactly +0.
//   * Escaped weights (about 2% of a N(0, 0.02) tensor) are added back as
//     fp32 corrections: the loader's escape index lists each block's escape
//     positions; the group's lanes split each row's escapes between them.
//   * A group accumulates its units of a tile in registers (each unit's MMA
//     chains start from zero; unit sums added in unit order), sums its four
//     warps in warp order at the tile's end and deposits the result in a
//     small ring of tile slots; a group with no unit in a tile deposits
//     zeros. The EPILOGUE warp sums a tile's four group deposits in group
//     order and writes a whole tile's outputs; a partial tile's sum goes
//     through scratch instead: each CTA writes its sum, the last to arrive (an
//     atomic counter that it resets) adds them in CTA order and writes the
//     outputs. As the partial tiles come first, those round trips overlap
//     the CTA's remaining units, and the consumers never wait on them.
//   * Every sum has a fixed order that depends on the tensor alone (not on
//     M nor the number of staging slots), so results are deterministic and
//     activation row m of an M-row call is bitwise the M=1 call on row m.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <string>
#include <vector>

#include "dm_device.cuh"
#include "dm_internal.h"

namespace dm {

constexpr int kMaxGrid = 256;  // CTAs of one launch, at most (one per SM)

struct alignas(16) SipArgs {
    const uint8_t *data;
    const uint32_t *unit16;
    int64_t units, rows, NB;
    const uint16_t *x;  // virtual activation rows [Mv][x_stride] bf16
    int64_t x_stride;
    int32_t Mv, nsplit, M_out;
    const uint16_t *bias;
    void *out;
    int32_t out_f32;
    float *partials;  // [grid][2][128]: a CTA's sums of its first / last tile
    int *counters;    // [tiles], zero between launches
    int *err;
    int32_t slot_bytes, x_off, nslots, dir_cap;
    int32_t xres_bytes;  // > 0: the activations of every block column resident in shared memory
    int32_t tile_split;  // 1: CTAs own whole tiles (no tile is shared), else units are split by weight
    int32_t starts[kMaxGrid + 1];  // CTA w owns units [starts[w], starts[w + 1])
    // row-sharded outputs gathered over NVLink (world > 0): every output is
    // also stored into each rank's gathered buffer [M][world * slot] at
    // rank * slot + row; the last CTA then raises each rank's flag of this
    // linear to the new launch count. Before staging activations, every CTA
    // waits for the flags of the linear its input depends on.
    int32_t world, rank;
    int64_t gslot;
    void *peer_out[DM_MAX_RANKS];
    uint32_t *peer_flags[DM_MAX_RANKS];
    uint32_t *gen, *done;
    const uint32_t *wait_flags, *wait_gen;
    uint32_t *abort;
    uint32_t wait_polls;  // polls of one flag wait before it gives up
    int32_t grid;         // CTAs of this linear (a chain launch may have more)
    int32_t wait_prev;    // chain: the awaited flags are the previous launch's (the link waits on a later link)
    int32_t prefetch;     // units after the staged ones asked into L2 before the dependency wait
    // a one-rank chain: the awaited link's CTA count (never reset: grid per
    // launch) and its grid, polled directly instead of a flag
    const uint32_t *wait_done;
    int32_t wait_grid;
};

// A GROUP of kGroupWarps consumer warps shares each staged unit: warp w of
// the group decodes quads [4w, 4w + 4) (k in [256w, 256w + 256)) of every
// row of the unit, and every 16th escape from w * 4 on. The CTA has kGroups
// groups (always: the sums' order must not depend on the launch).
constexpr int kGroupWarps = 4;
constexpr int kGroups = 4;
constexpr int kTileRing = 4;  // tile slots between the groups and the epilogue warp
// Block columns whose activations may stay resident: wider tensors (a 25600
// column down projection) measured faster staging activations per unit.
constexpr int kMaxResidentCols = 16;
constexpr int kSipThreads = 32 * (2 + kGroups * kGroupWarps);
// Staging slots of the unit ring, at most: with activations staged per unit
// six beat five, seven and eight on the 25600-column down projection.
constexpr int kMaxSlots = 6;
// Units fewer than the average that the last stream-K worker gets (part_sum).
constexpr double kSkewUnits = 4.0;
// Units past the first staged ones whose weights a CTA asks into L2 before it
// waits for its activations. Off by default: measured on the Qwen3 8B and
// 32B stacks, 4, 8 and 16 units each made the step 3-9 % slower, per-linear
// launches and chains alike (the extra requests compete with the previous
// linear's tail instead of filling it).
constexpr int kPrefetchUnits = 0;

// The stream-K split: worker b's share of the U units is proportional to
// wt(b) = 4096 for b <= b0 and 4096 - r (b - b0) after. CTAs are dispatched
// in index order as the previous launch's CTAs leave their SMs, so the last
// ones start after that launch has ended, too late to stage their first
// units under it, and get a smaller share (r = 0: an even split).
static inline int64_t part_sum(int64_t w, int64_t b0, int64_t r) {
    const int64_t m = w - 1 - b0;
    return 4096 * w - (m > 0 ? r * (m * (m + 1) / 2) : 0);
}
// The CTA that owns unit u (the last w with starts[w] <= u), from a CTA
// whose range is near.
__device__ __forceinline__ int64_t worker_of(const SipArgs &a, int64_t u, int64_t from, int64_t W) {
    int64_t c = from;
    while (c > 0 && a.starts[c] > u) --c;
    while (c + 1 < W && a.starts[c + 1] <= u) ++c;
    return c;
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

// The selectors of lane t's 16 codes from the unit's code planes (the
// loader's sip_code_planes): nibble w of s0 = code of weight w (w < 8), of
// s1 = code of weight 8 + w. The lane's bit-2 bits sit at 4w + 2 after a
// rotation by rl (weights 0..7) or rh (8..15): rl = t odd ? 0 : 2, rh = t
// odd ? 31 : 1.
__device__ __forceinline__ void code_selectors(uint32_t v, uint32_t P, uint32_t rl, uint32_t rh, uint32_t &s0,
                                               uint32_t &s1) {
    s0 = (v & 0x33333333u) | (__funnelshift_l(P, P, rl) & 0x44444444u);
    s1 = ((v >> 2) & 0x33333333u) | (__funnelshift_l(P, P, rh) & 0x44444444u);
}

// One row's quad: 16 weights at k = 64q + 16t + [0, 16) -> four bf16-pair
// registers per half (p01[j] = weights 4j, 4j+1; p23[j] = weights 4j+2, 4j+3).
__device__ __forceinline__ void decode_quad(const uint8_t *lit, const uint32_t *codes, int q, int t, uint32_t rl,
                                            uint32_t rh, uint32_t th0, uint32_t th1, uint32_t tl0, uint32_t tl1,
                                            uint32_t p01[4], uint32_t p23[4]) {
    const uint4 L = *reinterpret_cast<const uint4 *>(lit + 64 * q + 16 * t);
    uint32_t s0, s1;
    code_selectors(codes[4 * q + t], codes[64 + 2 * q + (t >> 1)], rl, rh, s0, s1);
    decode4(L.x, s0, th0, th1, tl0, tl1, p01[0], p23[0]);
    decode4(L.y, s0 >> 16, th0, th1, tl0, tl1, p01[1], p23[1]);
    decode4(L.z, s1, th0, th1, tl0, tl1, p01[2], p23[2]);
    decode4(L.w, s1 >> 16, th0, th1, tl0, tl1, p01[3], p23[3]);
}

// One quad of both of this lane's rows (g and g + 8) into the MMA chain: the
// weights are the A operand (16 rows x 16 k), the activations the B operand
// (16 k x 8 activation rows; lanes g < Mv hold activation row g).
__device__ __forceinline__ void quad(const uint8_t *lit0, const uint32_t *t00, const uint8_t *lit1,
                                     const uint32_t *t01, const uint8_t *xg, int q, int t, uint32_t rl, uint32_t rh,
                                     bool has_x,
                                     uint32_t th0, uint32_t th1, uint32_t tl0, uint32_t tl1, float &d0, float &d1,
                                     float &d2, float &d3) {
    uint4 X0 = make_uint4(0, 0, 0, 0), X1 = make_uint4(0, 0, 0, 0);
    if (has_x) {
        X0 = *reinterpret_cast<const uint4 *>(xg + 128 * q + 32 * t);
        X1 = *reinterpret_cast<const uint4 *>(xg + 128 * q + 32 * t + 16);
    }
    uint32_t a01[4], a23[4], c01[4], c23[4];
    decode_quad(lit0, t00, q, t, rl, rh, th0, th1, tl0, tl1, a01, a23);
    decode_quad(lit1, t01, q, t, rl, rh, th0, th1, tl0, tl1, c01, c23);
    mma_bf16_16816(d0, d1, d2, d3, a01[0], c01[0], a23[0], c23[0], X0.x, X0.y);
    mma_bf16_16816(d0, d1, d2, d3, a01[1], c01[1], a23[1], c23[1], X0.z, X0.w);
    mma_bf16_16816(d0, d1, d2, d3, a01[2], c01[2], a23[2], c23[2], X1.x, X1.y);
    mma_bf16_16816(d0, d1, d2, d3, a01[3], c01[3], a23[3], c23[3], X1.z, X1.w);
}

// Output o = (row r, activation row m) of tile `tile` from the tile's sums
// S[v][16] (virtual row v = m * nsplit + s): the nsplit virtual rows added in
// order, the bias in fp32, one rounding.
template <typename Sum>
__device__ __forceinline__ void store_output(const SipArgs &a, int64_t tile, int o, Sum S) {
    const int r = o & 15, m = o >> 4;
    const int64_t row = tile * kUnitRows + r;
    if (row >= a.rows) return;
    float y = S(m * a.nsplit * 16 + r);
    for (int s = 1; s < a.nsplit; ++s) y += S((m * a.nsplit + s) * 16 + r);
    if (a.bias) y += bf16_bits_to_f32(a.bias[row]);
    if (a.world > 0) {
        // into every rank's gathered output (this GPU's own included)
        const int64_t at = (int64_t)m * a.world * a.gslot + (int64_t)a.rank * a.gslot + row;
        if (a.out_f32) {
            for (int r = 0; r < a.world; ++r) reinterpret_cast<float *>(a.peer_out[r])[at] = y;
        } else {
            const uint16_t b = f32_to_bf16_bits(y);
            for (int r = 0; r < a.world; ++r) reinterpret_cast<uint16_t *>(a.peer_out[r])[at] = b;
        }
        return;
    }
    if (a.out_f32)
        reinterpret_cast<float *>(a.out)[m * a.rows + row] = y;
    else
        reinterpret_cast<uint16_t *>(a.out)[m * a.rows + row] = f32_to_bf16_bits(y);
}

// The wait for the flags of the linear this launch's input depends on: each
// rank's flag word reaches this rank's own launch count of that linear
// (bounded; gives up with an error code). In a chain launch (E > 0: the
// chain's launch count after this launch) the target is E for a link earlier
// in the chain and E - 1 for a later one (its output of the previous launch).
// One rank: the flags never leave this GPU, GPU scope suffices.
__device__ __forceinline__ void wait_inputs(const SipArgs &a, uint32_t E) {
    if (a.world <= 0) return;
    if (E && a.wait_done) {
        // one rank: the awaited link is done when all its CTAs have counted
        // themselves for this launch (E - 1 for the previous launch's)
        const uint32_t want = (a.wait_prev ? E - 1u : E) * (uint32_t)a.wait_grid;
        uint32_t i = 0;
        while ((int32_t)(ld_acquire_gpu(a.wait_done) - want) < 0)
            if (++i > a.wait_polls || (i % 64 == 0 && ld_acquire_gpu(a.abort) != 0u)) {
                atomicExch(a.err, kErrWaitPeer);
                atomicExch(a.abort, 1u);
                return;
            }
        fence_proxy_async_global();
        return;
    }
    if (a.wait_flags == nullptr) return;
    const uint32_t want = E ? (a.wait_prev ? E - 1u : E) : ld_acquire_gpu(a.wait_gen);
    if (want == 0u) return;  // a chain's first launch: no earlier output to wait for
    for (int r = 0; r < a.world; ++r) {
        uint32_t i = 0;
        while ((int32_t)((a.world == 1 ? ld_acquire_gpu(a.wait_flags + r) : ld_acquire_sys(a.wait_flags + r)) -
                         want) < 0) {
            // a rank gave up before: do not wait again
            if (++i > a.wait_polls || (i % 64 == 0 && ld_acquire_gpu(a.abort) != 0u)) {
                atomicExch(a.err, kErrWaitPeer);
                atomicExch(a.abort, 1u);
                return;
            }
        }
    }
    fence_proxy_async_global();
}

// After this CTA's last output (called by one lane, after a __syncwarp of
// the warp that stored them): the CTA count of the launch; the last CTA,
// having acquired every count, raises every rank's flag of this linear to
// the new launch count (E in a chain launch) behind one fence.
__device__ __forceinline__ void signal_outputs(const SipArgs &a, uint32_t E) {
    if (a.world <= 0) return;
    if (E && a.world == 1) {
        // a one-rank chain: the count itself is what later links poll; it
        // grows by the grid every launch (never reset)
        if (atom_add_acq_rel_gpu(a.done, 1u) + 1u == E * (uint32_t)a.grid) *a.gen = E;
        return;
    }
    // the count needs GPU scope only: the last CTA's system-scope fence
    // below carries every CTA's stores (ordered before it here) to the peers
    if (atom_add_acq_rel_gpu(a.done, 1u) + 1u != (uint32_t)a.grid) return;
    *a.done = 0u;
    const uint32_t g = E ? E : *a.gen + 1u;
    *a.gen = g;
    if (a.world == 1) {
        fence_acq_rel_gpu();
        st_relaxed_gpu(a.peer_flags[0] + a.rank, g);
        return;
    }
    // one system-scope fence releases every flag store after it (a release
    // store per rank would wait for the outstanding NVLink stores each time)
    fence_acq_rel_sys();
    for (int r = 0; r < a.world; ++r) st_relaxed_sys(a.peer_flags[r] + a.rank, g);
}

// Full barriers per staging slot. A group takes every 4th position of the
// ring, so it can reach slot p % S before the slot's previous position p - S
// (another group's) has landed; with one barrier per slot its phase parity
// would then name an older, completed phase. Position p arms barrier set
// (p / S) % L of its slot: a group at p has consumed p - 4, so every position
// up to p - 4 is staged, hence (L - 1) * S >= 4 puts p - (L - 1) * S among
// them and the set's previous use p - L * S has been consumed, and landed.
__host__ __device__ __forceinline__ int full_sets(int S) { return S >= kGroups ? 2 : (kGroups + S - 1) / S + 1; }

__device__ __forceinline__ void group_sync(int group) {
    asm volatile("bar.sync %0, %1;" ::"r"(1 + group), "r"(kGroupWarps * 32) : "memory");
}

// One row's escapes (this lane's share) added to its corrections.
template <int MV>
__device__ __forceinline__ void escapes(const uint8_t *lit, RowEntry e, const uint8_t *xs, int j0, float corr[MV]) {
    const int ne = e.nesc;
    if (ne <= j0) return;
    const uint8_t *term = lit + 1408;
    const uint16_t *idx = reinterpret_cast<const uint16_t *>(lit + (((uint32_t)e.words * 4u + 15u) & ~15u));
    for (int j = j0; j < ne; j += 4 * kGroupWarps) {
        const uint32_t pos = idx[j];
        const uint32_t ex = term[j];
        const uint32_t lb = lit[pos];
        const float wv = __uint_as_float(((lb & 0x80u) << 24) | (ex << 23) | ((lb & 0x7Fu) << 16));
        const uint8_t *xp = xs + pos * 2;
#pragma unroll
        for (int v = 0; v < MV; ++v)
            corr[v] = fmaf(bf16_bits_to_f32(*reinterpret_cast<const uint16_t *>(xp + v * kXRowStride)), wv, corr[v]);
    }
}

// The CTA's unit sequence: its first tile's units when that tile is partial
// (segment A), its last tile's when partial (B), then its whole tiles (C).
// Position p of the sequence -> unit and tile sequence number.
struct Seq {
    int64_t a0, b0, c0;     // first unit of A, B, C
    int32_t nA, nAB, n;     // |A|, |A| + |B|, |A| + |B| + |C|
    int32_t tsB, tsC;       // sequence numbers of B's tile and C's first tile
    int32_t ntiles;
    int64_t tA, tB, tC;     // tile ids of A, B and C's first tile
    __device__ void init(int64_t cu0, int64_t cu1, int64_t NB) {
        const int64_t f = cu0 / NB, l = (cu1 - 1) / NB;
        const bool pa = cu0 > f * NB || cu1 < (f + 1) * NB;
        const bool pb = l != f && cu1 < (l + 1) * NB;
        const int64_t a1 = pa ? std::min(cu1, (f + 1) * NB) : cu0;
        a0 = cu0;
        b0 = pb ? l * NB : cu1;
        c0 = a1;
        const int64_t c1 = pb ? l * NB : cu1;
        nA = (int32_t)(a1 - cu0);
        nAB = nA + (int32_t)(pb ? cu1 - l * NB : 0);
        n = (int32_t)(cu1 - cu0);
        tsB = nA > 0 ? 1 : 0;
        tsC = tsB + (nAB > nA ? 1 : 0);
        ntiles = tsC + (int32_t)((c1 - c0) / NB);
        tA = f;
        tB = l;
        tC = c0 / NB;
    }
    __device__ __forceinline__ int64_t tile_of(int32_t ts) const {
        return ts < tsB ? tA : (ts < tsC ? tB : tC + (ts - tsC));
    }
};

// The barriers of a linear's shared-memory plan: full [L][S], empty [S],
// tfull and tempty [kTileRing], x_ready [kMaxResidentCols], contiguous.
__device__ __forceinline__ uint64_t *sip_barriers(const SipArgs &a, uint8_t *smem) {
    return reinterpret_cast<uint64_t *>(smem + (size_t)a.nslots * a.slot_bytes + a.xres_bytes);
}

// One linear's GEMV by this CTA (the kernel body; every role returns here).
// RES: the activations of every block column are resident in shared memory
// (loaded once per launch) instead of staged with each unit. E: 0 for a
// launch of its own, else the chain's launch count after this launch.
template <int MV, bool RES>
__device__ __forceinline__ void sip_run(const SipArgs &a, uint8_t *smem, uint32_t E) {
    constexpr int kP = 16 * MV;  // floats of one tile partial [MV][16]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = a.nslots;
    // resident activations [NB][Mv][kXRowStride] (when xres_bytes > 0)
    uint8_t *xres = smem + (size_t)S * a.slot_bytes;
    const int L = full_sets(S);
    uint64_t *full = reinterpret_cast<uint64_t *>(xres + a.xres_bytes);  // [L][S]
    uint64_t *empty = full + L * S;       // [S]
    uint64_t *tfull = empty + S;          // [kTileRing]: 16 warp deposits
    uint64_t *tempty = tfull + kTileRing;  // [kTileRing]: the epilogue warp's release
    uint64_t *x_ready = tempty + kTileRing;  // [kMaxResidentCols]: a block column's resident activations landed
    float *pwb = reinterpret_cast<float *>(x_ready + kMaxResidentCols);  // [kGroups][2][kGroupWarps][kP]
    float *tslot = pwb + kGroups * 2 * kGroupWarps * kP;          // [kTileRing][kGroups][kP]
    float *ebuf = tslot + kTileRing * kGroups * kP;               // [kP] the epilogue's tile sum
    uint32_t *dir = reinterpret_cast<uint32_t *>(ebuf + kP);     // this CTA's unit starts
    const int64_t U = a.units, W = a.grid, NB = a.NB;
    const int64_t T = (U + NB - 1) / NB;
    const int64_t cu0 = a.starts[blockIdx.x], cu1 = a.starts[blockIdx.x + 1];
    const bool dir_in_smem = (cu1 - cu0 + 1) <= a.dir_cap;
    Seq q;
    q.init(cu0, cu1, NB);
    pdl_launch_dependents();
    if (threadIdx.x == 0) {
        for (int i = 0; i < L * S; ++i) mbar_init(&full[i], 1);
        for (int i = 0; i < S; ++i) mbar_init(&empty[i], kGroupWarps);
        for (int i = 0; i < kTileRing; ++i) {
            mbar_init(&tfull[i], kGroups * kGroupWarps);
            mbar_init(&tempty[i], 1);
        }
        if constexpr (RES)
            for (int i = 0; i < NB; ++i) mbar_init(&x_ready[i], 1);
        mbar_fence_init();
    }
    if (warp == 0 && dir_in_smem)
        for (int64_t i = lane; i <= cu1 - cu0; i += 32) dir[i] = a.unit16[cu0 + i];
    __syncthreads();
    // position p -> unit
    auto unit_at = [&](int32_t p) -> int64_t {
        return p < q.nA ? q.a0 + p : (p < q.nAB ? q.b0 + (p - q.nA) : q.c0 + (p - q.nAB));
    };

    if (warp == 0) {
        // ---------------------------------------------------- producer --
        if (lane == 0) {
            // unit u (block column col) into slot `slot`, completing on full
            // barrier fb; positions walk units with no division: consecutive
            // within a segment, a segment's first unit starting a tile
            auto advance = [&](int32_t np, int64_t &u, int32_t &col) {
                if (np == q.nA || np == q.nAB) {
                    u = unit_at(np);
                    col = 0;
                } else {
                    ++u;
                    if (++col == NB) col = 0;
                }
            };
            const int64_t u0 = unit_at(0);
            const int32_t col0 = (int32_t)(u0 % NB);
            auto stage_w = [&](int64_t u, int slot, uint64_t *fb) {
                const uint32_t q0 = dir_in_smem ? dir[u - cu0] : a.unit16[u];
                const uint32_t q1 = dir_in_smem ? dir[u + 1 - cu0] : a.unit16[u + 1];
                const uint32_t ubytes = (q1 - q0) * 16u;
                mbar_arrive_expect_tx(fb, ubytes + (RES ? 0u : (uint32_t)a.Mv * 2048u));
                bulk_g2s(smem + (size_t)slot * a.slot_bytes, a.data + (size_t)q0 * 16, ubytes, fb);
            };
            auto stage_x = [&](int32_t col, int slot, uint64_t *fb) {
                if constexpr (RES) return;  // the block columns' activations are resident
                const uint16_t *xb = a.x + (size_t)col * 1024;
                uint8_t *dst = smem + (size_t)slot * a.slot_bytes + a.x_off;
                for (int v = 0; v < a.Mv; ++v) bulk_g2s(dst + v * kXRowStride, xb + v * a.x_stride, 2048u, fb);
            };
            // the first S units' weights do not depend on the kernel before
            // this one: stage them, wait for it, then add their activations
            const int32_t first = std::min<int32_t>(S, q.n);
            {
                int64_t u = u0;
                int32_t col = col0;
                for (int32_t p = 0; p < first; ++p) {
                    if (p > 0) advance(p, u, col);
                    stage_w(u, p, &full[p]);
                }
                // the next units' weights into L2 meanwhile
                const int32_t pf = std::min<int32_t>(q.n, first + a.prefetch);
                for (int32_t p = first; p < pf; ++p) {
                    advance(p, u, col);
                    const uint32_t q0 = dir_in_smem ? dir[u - cu0] : a.unit16[u];
                    const uint32_t q1 = dir_in_smem ? dir[u + 1 - cu0] : a.unit16[u + 1];
                    bulk_prefetch_l2(a.data + (size_t)q0 * 16, (q1 - q0) * 16u);
                }
            }
            pdl_wait();
            wait_inputs(a, E);
            if constexpr (RES) {
                // the block columns this CTA's units touch (its units are
                // consecutive: min(n, NB) columns from A's first), each once
                // on its own barrier, in the order the units first need them;
                // every copy issued here is waited for by a consumer
                int64_t b = q.a0 % NB;
                const int64_t ncols = std::min<int64_t>(NB, q.n);
                for (int64_t i = 0; i < ncols; ++i) {
                    mbar_arrive_expect_tx(&x_ready[b], (uint32_t)a.Mv * 2048u);
                    for (int v = 0; v < a.Mv; ++v)
                        bulk_g2s(xres + (b * a.Mv + v) * kXRowStride, a.x + b * 1024 + v * a.x_stride, 2048u,
                                 &x_ready[b]);
                    if (++b == NB) b = 0;
                }
            }
            int64_t u = u0;
            int32_t col = col0;
            for (int32_t p = 0; p < first; ++p) {
                if (p > 0) advance(p, u, col);
                stage_x(col, p, &full[p]);
            }
            int slot = 0, fset = L > 1 ? 1 : 0;  // position first = S: slot 0 of set 1
            uint32_t epar = 0;  // parity of the empty phase to wait for
            bool ok = true;
            for (int32_t p = first; p < q.n && ok; ++p) {
                advance(p, u, col);
                if (!mbar_wait(&empty[slot], epar, a.err, kErrWaitEmpty)) ok = false;
                if (ok) {
                    uint64_t *fb = &full[fset * S + slot];
                    stage_w(u, slot, fb);
                    stage_x(col, slot, fb);
                }
                if (++slot == S) {
                    slot = 0;
                    epar ^= 1u;
                    if (++fset == L) fset = 0;
                }
            }
            // drain: every copy this producer issued lands before the CTA exits
            for (int32_t p = std::max<int32_t>(0, q.n - S); p < q.n && ok; ++p)
                mbar_wait(&full[((p / S) % L) * S + p % S], (uint32_t)((p / S / L) & 1), a.err, kErrWaitDrain);
        }
        return;
    }

    if (warp == 1 + kGroups * kGroupWarps) {
        if constexpr (MV == 0) {
            return;  // decode: nothing to sum
        } else {
            // ---------------------------------------------------- epilogue --
            bool ok = true;
            for (int32_t ts = 0; ts < q.ntiles; ++ts) {
                const int ring = ts % kTileRing;
                if (ok && !mbar_wait(&tfull[ring], (uint32_t)((ts / kTileRing) & 1), a.err, kErrWaitFull)) ok = false;
                float T[(kP + 31) / 32];
    #pragma unroll
                for (int i = 0; i < (kP + 31) / 32; ++i) {
                    const int e = lane + 32 * i;
                    float v = 0.f;
                    if (e < kP) {
                        const float *sl = tslot + ring * kGroups * kP + e;
                        v = sl[0];
    #pragma unroll
                        for (int gg = 1; gg < kGroups; ++gg) v += sl[gg * kP];
                    }
                    T[i] = v;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[ring]);
                const int64_t tl = q.tile_of(ts);
                bool store = ts >= q.tsC;
                if (!store) {
                    // a tile shared with other CTAs: this CTA's sum to scratch,
                    // the last of them to arrive adds all in CTA order
                    const int cs = (tl == cu0 / NB) ? 0 : 1;
                    float *mine = a.partials + ((int64_t)blockIdx.x * 2 + cs) * 128;
    #pragma unroll
                    for (int i = 0; i < (kP + 31) / 32; ++i)
                        if (lane + 32 * i < kP) mine[lane + 32 * i] = T[i];
                    // the warp's partial, released by lane 0's count; the last to
                    // count acquires every other CTA's partial with it
                    __syncwarp();
                    const int64_t cf = worker_of(a, tl * NB, blockIdx.x, W);
                    const int64_t cl = worker_of(a, (tl + 1) * NB - 1, blockIdx.x, W);
                    int last = 0;
                    if (lane == 0) {
                        const uint32_t old = atom_add_acq_rel_gpu(reinterpret_cast<uint32_t *>(a.counters + tl), 1u);
                        last = (old == (uint32_t)(cl - cf));
                        if (last) a.counters[tl] = 0;
                    }
                    last = __shfl_sync(0xffffffffu, last, 0);
                    if (last) {
                        for (int64_t c = cf; c <= cl; ++c) {
                            const int sc = (tl == a.starts[c] / NB) ? 0 : 1;
                            const float *pp = a.partials + (c * 2 + sc) * 128;
    #pragma unroll
                            for (int i = 0; i < (kP + 31) / 32; ++i)
                                if (lane + 32 * i < kP) {
                                    const float x = __ldcg(pp + lane + 32 * i);
                                    T[i] = (c == cf) ? x : T[i] + x;
                                }
                        }
                        store = true;
                    }
                }
                if (store) {
    #pragma unroll
                    for (int i = 0; i < (kP + 31) / 32; ++i)
                        if (lane + 32 * i < kP) ebuf[lane + 32 * i] = T[i];
                    __syncwarp();
                    for (int o = lane; o < 16 * a.M_out; o += 32) store_output(a, tl, o, [&](int e) { return ebuf[e]; });
                    __syncwarp();
                }
            }
            __syncwarp();
            if (lane == 0) signal_outputs(a, E);
            return;
        }
    }

    // ------------------------------------------------------- consumers --
    const int gi = (warp - 1) / kGroupWarps, wi = (warp - 1) % kGroupWarps;
    const int g = lane >> 2, t = lane & 3;
    if constexpr (MV == 0) {
        // DECODE: each unit's weights straight to the bf16 output [rows][C]:
        // the group's stores, one group barrier, then the escaped weights'
        // true values over their +0 (every group barrier is kept even after a
        // failed wait, so none is left short)
        uint16_t *out = reinterpret_cast<uint16_t *>(a.out);
        const int64_t C = NB * 1024;
        const uint32_t rl = (t & 1) ? 0u : 2u, rh = (t & 1) ? 31u : 1u;
        const int q0 = 4 * wi, j0 = 4 * wi + t;
        // no activations order these stores after the kernel before this
        // one (launched early by programmatic dependent launch, it may still
        // read or write the output's memory): wait for it explicitly
        pdl_wait();
        bool ok = true;
        int slot = gi % S, set = (gi / S) % L;
        uint32_t par = (uint32_t)((gi / S / L) & 1);
        for (int32_t p = gi; p < q.n; p += kGroups) {
            const int64_t u = unit_at(p);
            const int64_t tile = u / NB, bcol = u - tile * NB;
            const int64_t r0 = tile * kUnitRows + g, r1 = r0 + 8;
            if (ok && !mbar_wait(&full[set * S + slot], par, a.err, kErrWaitFull)) ok = false;
            const uint8_t *base = smem + (size_t)slot * a.slot_bytes;
            const RowEntry e0 = reinterpret_cast<const RowEntry *>(base)[g];
            const RowEntry e1 = reinterpret_cast<const RowEntry *>(base)[g + 8];
            const uint8_t *lit0 = base + (size_t)e0.off16 * 16;
            const uint8_t *lit1 = base + (size_t)e1.off16 * 16;
            if (ok) {
                const uint4 tab = *reinterpret_cast<const uint4 *>(base + kUnitRows * sizeof(RowEntry));
                const uint32_t *t00 = reinterpret_cast<const uint32_t *>(lit0 + 1024);
                const uint32_t *t01 = reinterpret_cast<const uint32_t *>(lit1 + 1024);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    uint32_t a01[4], a23[4], c01[4], c23[4];
                    decode_quad(lit0, t00, q0 + k, t, rl, rh, tab.x, tab.y, tab.z, tab.w, a01, a23);
                    decode_quad(lit1, t01, q0 + k, t, rl, rh, tab.x, tab.y, tab.z, tab.w, c01, c23);
                    const int64_t col = bcol * 1024 + 64 * (q0 + k) + 16 * t;
                    if (r0 < a.rows) {
                        uint4 *d = reinterpret_cast<uint4 *>(out + r0 * C + col);
                        d[0] = make_uint4(a01[0], a23[0], a01[1], a23[1]);
                        d[1] = make_uint4(a01[2], a23[2], a01[3], a23[3]);
                    }
                    if (r1 < a.rows) {
                        uint4 *d = reinterpret_cast<uint4 *>(out + r1 * C + col);
                        d[0] = make_uint4(c01[0], c23[0], c01[1], c23[1]);
                        d[1] = make_uint4(c01[2], c23[2], c01[3], c23[3]);
                    }
                }
            }
            group_sync(gi);
            if (ok) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const RowEntry e = h ? e1 : e0;
                    const uint8_t *lit = h ? lit1 : lit0;
                    const int64_t row = h ? r1 : r0;
                    const uint8_t *term = lit + 1408;
                    const uint16_t *idx = reinterpret_cast<const uint16_t *>(lit + (((uint32_t)e.words * 4u + 15u) & ~15u));
                    if (row < a.rows)
                        for (int j = j0; j < (int)e.nesc; j += 4 * kGroupWarps) {
                            const uint32_t pos = idx[j] & 1023u;
                            const uint32_t lb = lit[pos];
                            out[row * C + bcol * 1024 + pos] =
                                (uint16_t)(((lb & 0x80u) << 8) | ((uint32_t)term[j] << 7) | (lb & 0x7Fu));
                        }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[slot]);
            }
            slot += kGroups;
            while (slot >= S) {
                slot -= S;
                if (++set == L) {
                    set = 0;
                    par ^= 1u;
                }
            }
        }
        return;
    } else {

    // D[rows g, g + 8][activation rows 2t, 2t + 1] over this warp's k range, the tile so far
    float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
    float cg[MV], cg8[MV];  // rows g and g + 8: escape corrections (this lane's share)
#pragma unroll
    for (int v = 0; v < MV; ++v) cg[v] = cg8[v] = 0.f;
    int buf = 0;
    bool ok = true;

    // the tile ring slot of tile sequence number ts, once the epilogue warp
    // has released its previous use
    auto tile_slot = [&](int32_t ts) -> float * {
        const int ring = ts % kTileRing, use = ts / kTileRing;
        if (use > 0 && ok && !mbar_wait(&tempty[ring], (uint32_t)((use - 1) & 1), a.err, kErrWaitEmpty)) ok = false;
        return tslot + (ring * kGroups + gi) * kP;
    };
    // this group's sum of tile ts (its warps' partials in warp order) into
    // the tile ring; the two partial buffers alternate, so one barrier will do
    auto flush = [&](int32_t ts) {
#pragma unroll
        for (int v = 0; v < MV; ++v) {
            float s = cg[v], s8 = cg8[v];
            s += __shfl_xor_sync(0xffffffffu, s, 1);
            s += __shfl_xor_sync(0xffffffffu, s, 2);
            s8 += __shfl_xor_sync(0xffffffffu, s8, 1);
            s8 += __shfl_xor_sync(0xffffffffu, s8, 2);
            cg[v] = s;
            cg8[v] = s8;
        }
        float *grp = pwb + (gi * 2 + buf) * kGroupWarps * kP;
        float *pw = grp + wi * kP;
        if (t == 0) {
#pragma unroll
            for (int v = 0; v < MV; ++v) {
                pw[v * 16 + g] = cg[v];
                pw[v * 16 + g + 8] = cg8[v];
            }
        }
        __syncwarp();
        if (2 * t < MV) {
            pw[2 * t * 16 + g] += acc0;
            pw[2 * t * 16 + g + 8] += acc2;
        }
        if (2 * t + 1 < MV) {
            pw[(2 * t + 1) * 16 + g] += acc1;
            pw[(2 * t + 1) * 16 + g + 8] += acc3;
        }
        group_sync(gi);
        float *dst = tile_slot(ts);
        for (int e = wi * 32 + lane; e < kP; e += kGroupWarps * 32) {
            float v = grp[e];
#pragma unroll
            for (int k = 1; k < kGroupWarps; ++k) v += grp[k * kP + e];
            dst[e] = v;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&tfull[ts % kTileRing]);
        buf ^= 1;
        acc0 = acc1 = acc2 = acc3 = 0.f;
#pragma unroll
        for (int v = 0; v < MV; ++v) cg[v] = cg8[v] = 0.f;
    };
    // a tile without units of this group: zeros
    auto deposit_zero = [&](int32_t ts) {
        float *dst = tile_slot(ts);
        for (int e = wi * 32 + lane; e < kP; e += kGroupWarps * 32) dst[e] = 0.f;
        __syncwarp();
        if (lane == 0) mbar_arrive(&tfull[ts % kTileRing]);
    };

    const uint32_t rl = (t & 1) ? 0u : 2u, rh = (t & 1) ? 31u : 1u;
    const bool has_x = g < MV;
    const int q0 = 4 * wi, j0 = 4 * wi + t;
    int32_t cur = -1;  // tile sequence number of the group's current tile
    uint32_t xin = 0;  // bit b: block column b's resident activations have landed
    int slot = gi % S, set = (gi / S) % L;
    uint32_t par = (uint32_t)((gi / S / L) & 1);
    int32_t cq = -1, cts = 0;  // in segment C: the unit's offset in its tile, its tile's number
    const int32_t nb = (int32_t)NB;
    const int32_t bcA = (int32_t)(q.a0 % NB);  // block column of A's first unit
    for (int32_t p = gi; p < q.n; p += kGroups) {
        int32_t ts, bc;  // the unit's tile sequence number and block column
        if (p < q.nA) {
            ts = 0;
            bc = bcA + p;
        } else if (p < q.nAB) {
            ts = q.tsB;
            bc = p - q.nA;
        } else {
            if (cq < 0) {
                cq = (p - q.nAB) % nb;
                cts = (p - q.nAB) / nb;
            } else {
                cq += kGroups;
                while (cq >= nb) {
                    cq -= nb;
                    ++cts;
                }
            }
            ts = q.tsC + cts;
            bc = cq;
        }
        if (ts != cur) {
            if (cur >= 0) flush(cur);
            for (int32_t z = cur + 1; z < ts; ++z) deposit_zero(z);
            cur = ts;
        }
        if (ok && !mbar_wait(&full[set * S + slot], par, a.err, kErrWaitFull)) ok = false;
        if (RES && !((xin >> bc) & 1u)) {
            if (ok && !mbar_wait(&x_ready[bc], 0u, a.err, kErrWaitFull)) ok = false;
            xin |= 1u << bc;
        }
        if (ok) {
            const uint8_t *base = smem + (size_t)slot * a.slot_bytes;
            // the exponent tables of the unit's part (high part th0/th1, low tl0/tl1)
            const uint4 tab = *reinterpret_cast<const uint4 *>(base + kUnitRows * sizeof(RowEntry));
            const uint32_t th0 = tab.x, th1 = tab.y, tl0 = tab.z, tl1 = tab.w;
            const RowEntry e0 = reinterpret_cast<const RowEntry *>(base)[g];
            const RowEntry e1 = reinterpret_cast<const RowEntry *>(base)[g + 8];
            const uint8_t *lit0 = base + (size_t)e0.off16 * 16;
            const uint8_t *lit1 = base + (size_t)e1.off16 * 16;
            const uint32_t *t00 = reinterpret_cast<const uint32_t *>(lit0 + 1024);
            const uint32_t *t01 = reinterpret_cast<const uint32_t *>(lit1 + 1024);
            const uint8_t *xs = RES ? xres + bc * (MV * kXRowStride) : base + a.x_off;
            const uint8_t *xg = xs + g * kXRowStride;
            float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
            float f0 = 0.f, f1 = 0.f, f2 = 0.f, f3 = 0.f;
            quad(lit0, t00, lit1, t01, xg, q0 + 0, t, rl, rh, has_x, th0, th1, tl0, tl1, d0, d1, d2, d3);
            quad(lit0, t00, lit1, t01, xg, q0 + 1, t, rl, rh, has_x, th0, th1, tl0, tl1, f0, f1, f2, f3);
            quad(lit0, t00, lit1, t01, xg, q0 + 2, t, rl, rh, has_x, th0, th1, tl0, tl1, d0, d1, d2, d3);
            quad(lit0, t00, lit1, t01, xg, q0 + 3, t, rl, rh, has_x, th0, th1, tl0, tl1, f0, f1, f2, f3);
            // escapes of rows g and g + 8: the group's warps take every 16th one, lane t every 4th of those
            escapes<MV>(lit0, e0, xs, j0, cg);
            escapes<MV>(lit1, e1, xs, j0, cg8);
            acc0 += d0;
            acc0 += f0;
            acc1 += d1;
            acc1 += f1;
            acc2 += d2;
            acc2 += f2;
            acc3 += d3;
            acc3 += f3;
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
        slot += kGroups;
        while (slot >= S) {
            slot -= S;
            if (++set == L) {
                set = 0;
                par ^= 1u;
            }
        }
    }
    if (cur >= 0) flush(cur);
    for (int32_t z = cur + 1; z < q.ntiles; ++z) deposit_zero(z);
    }
}

template <int MV, bool RES>
__global__ void __launch_bounds__(kSipThreads, 1) sip_gemv_kernel(const __grid_constant__ SipArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    sip_run<MV, RES>(a, smem, 0u);
}

// A CHAIN: a sequence of GEMVs (links) in one persistent launch, one CTA per
// SM. Each CTA runs its share of link 0, then of link 1, ...: the link's
// arguments are copied into shared memory behind the largest link's plan,
// its barriers set up, the body run, its barriers retired. A link whose
// activations are another link's output waits (bounded) on that link's flags
// before staging them, exactly as a launch of its own waits on its
// predecessor; its first units' weights are staged before the wait, under the
// previous link's tail. words[0] counts the chain's launches (each link's
// flags are raised to it), words[1] the CTAs that have left this launch: the
// last one raises words[0], after every CTA has read it. Needs every CTA
// resident at once (a cooperative launch).
// A link's arguments global -> shared, 16 bytes per thread, asynchronously
// (LDGSTS): the next link's copy lands while this one runs.
__device__ __forceinline__ void chain_args_prefetch(const SipArgs *src, SipArgs *dst) {
    const uint8_t *s = reinterpret_cast<const uint8_t *>(src);
    uint8_t *d = reinterpret_cast<uint8_t *>(dst);
    for (int k = threadIdx.x; k < (int)(sizeof(SipArgs) / 16); k += kSipThreads)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(d + 16 * k)), "l"(s + 16 * k)
                     : "memory");
    asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int MV>
__global__ void __launch_bounds__(kSipThreads, 1) sip_chain_kernel(const SipArgs *links, int32_t n, uint32_t *words,
                                                                   int32_t args_off) {
    extern __shared__ __align__(128) uint8_t smem[];
    SipArgs *buf = reinterpret_cast<SipArgs *>(smem + args_off);  // [2]: this link's and the next one's
    uint32_t *launches = reinterpret_cast<uint32_t *>(buf + 2);
    if (threadIdx.x == 0) *launches = ld_acquire_gpu(words);
    chain_args_prefetch(links, buf);
    for (int32_t i = 0; i < n; ++i) {
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncthreads();  // link i's arguments landed; the previous link is done in this CTA
        if (i + 1 < n) chain_args_prefetch(links + i + 1, buf + ((i + 1) & 1));
        const SipArgs *sa = buf + (i & 1);
        if ((int32_t)blockIdx.x >= sa->grid) continue;
        const uint32_t E = *launches + 1u;
        if (sa->xres_bytes > 0)
            sip_run<MV, true>(*sa, smem, E);
        else
            sip_run<MV, false>(*sa, smem, E);
        __syncthreads();
        if (threadIdx.x == 0) {
            // retire the link's barriers: its shared memory is the next link's
            uint64_t *b = sip_barriers(*sa, smem);
            const int S = sa->nslots, nb = full_sets(S) * S + S + 2 * kTileRing;
            const int nres = sa->xres_bytes > 0 ? (int)sa->NB : 0;
            for (int k = 0; k < nb + nres; ++k) mbar_inval(b + k);
        }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    if (threadIdx.x == 0 && atom_add_acq_rel_gpu(words + 1, 1u) + 1u == gridDim.x) {
        words[1] = 0u;
        st_relaxed_gpu(words, *launches + 1u);
    }
}

// Staging slots of a launch with resident activations: five, six at M = 1
// for tensors of 8 or more block columns. Fewer slots than fit: on the Qwen3
// 8B and 32B shapes 5-6 slots beat 7-8 by 3-8 % (and 4 lose up to 10 %).
inline int resident_slots(int Mv, int64_t NB) { return Mv == 1 && NB >= 8 ? 6 : 5; }

// Shared-memory plan for a launch: the slot size, the number of slots and
// whether the activations of every block column stay resident (one copy per
// launch instead of one per unit; chosen whenever the tensor has at most
// `max_res` block columns and they fit beside the resident launch's slots).
// `slots` > 0 asks for that many slots (fewer when they do not fit); 0 takes
// the measured rule. Any number of slots is correct (full_sets). Fixed
// part: the barriers, the groups' partial buffers, the tile ring, the
// epilogue's sum and the directory.
int sip_shared_bytes(const dm_tensor *t, int Mv, int slots, int max_res, int *slot_bytes, int *nslots,
                     int *xres_bytes, int dir_cap, int reserve) {
    const int unit = (t->L.max_unit_bytes + 127) & ~127;
    const int budget = 227 * 1024 - reserve;
    const int kP = 16 * Mv;
    const int fixed = (3 * kMaxSlots + 2 * kTileRing + kMaxResidentCols) * 8 +
                      (kGroups * 2 * kGroupWarps + kTileRing * kGroups + 1) * kP * 4 + (dir_cap + 1) * 4 + 128;
    const int sb1 = unit + Mv * kXRowStride;
    const int n1 = std::min(slots > 0 ? slots : kMaxSlots, (budget - fixed) / sb1);
    const int64_t xr = Mv >= 1 && t->L.NB <= std::min(max_res, kMaxResidentCols)
                           ? ((t->L.NB * Mv * kXRowStride + 127) & ~(int64_t)127)
                           : 0;
    const int want = slots > 0 ? slots : resident_slots(Mv, t->L.NB);
    if (xr > 0 && (int64_t)budget - fixed - xr >= (int64_t)want * unit) {
        *slot_bytes = unit;
        *nslots = want;
        *xres_bytes = (int)xr;
        return want * unit + (int)xr + fixed;
    }
    if (n1 < 1) return -1;
    *slot_bytes = sb1;
    *nslots = n1;
    *xres_bytes = 0;
    return n1 * sb1 + fixed;
}

// The launch a GEMV (Mv virtual activation rows; 0: decode) of this tensor
// makes under its launch knobs (dm_tensor_set_launch): the CTA split, the
// stream-K weights, the staging slots and the shared-memory plan.
struct SipPlan {
    int64_t grid = 0, per_cta = 0;
    int tile_split = 0;
    int32_t part_b0 = 0, part_r = 0;
    int dir_cap = 0, smem = 0, slot_bytes = 0, nslots = 0, xres_bytes = 0;
};

static int plan_sip(const dm_tensor *t, int Mv, SipPlan &P, std::string &msg, int reserve = 0) {
    const dm::TensorLayout &L = t->L;
    const LaunchKnobs &K = t->K;
    // One CTA per SM, each a stream-K worker owning at least one unit; or,
    // CTAs that own whole tiles when the busiest of them would decode fewer
    // units than a stream-K worker plus its cross-CTA fixup (worth about
    // three units when a CTA's range holds under two tiles, four under one;
    // measured on the Qwen3 8B and 32B shapes). The split depends on the
    // tensor (and its knobs) alone.
    const int64_t tiles = L.tiles;
    const int64_t gridA = std::min<int64_t>(t->sms, L.units), gridB = std::min<int64_t>(t->sms, tiles);
    const int64_t perA = (L.units + gridA - 1) / gridA;
    const int64_t costA = perA + (perA < L.NB ? 4 : (perA < 2 * L.NB ? 3 : 0));
    const int64_t costB = (tiles + gridB - 1) / gridB * L.NB;
    P.tile_split = K.split == kSplitTiles ? 1 : (K.split == kSplitStreamK ? 0 : (costB < costA ? 1 : 0));
    P.grid = P.tile_split ? gridB : gridA;
    // the stream-K split's weights: the last 40 % of the CTAs down to `skew`
    // units fewer than the average for the very last (none when the average
    // is under 8 units)
    const double skew = K.skew >= 0 ? (double)K.skew : kSkewUnits;
    P.part_b0 = P.part_r = 0;
    if (!P.tile_split && P.grid > 8 && perA >= 8 && skew > 0) {
        P.part_b0 = (int32_t)(P.grid * 6 / 10);
        const double delta = std::min(0.5, skew * (double)P.grid / (double)L.units);
        P.part_r = (int32_t)std::llround(4096.0 * delta / (double)(P.grid - 1 - P.part_b0));
    }
    P.per_cta = P.tile_split
                    ? (tiles + P.grid - 1) / P.grid * L.NB
                    : (P.part_r ? (L.units * 4096 + part_sum(P.grid, P.part_b0, P.part_r) - 1) /
                                          part_sum(P.grid, P.part_b0, P.part_r) + 1
                                : perA);
    P.dir_cap = (int)std::min<int64_t>(4096, P.per_cta + 2);
    P.smem = sip_shared_bytes(t, Mv, K.slots, K.resident >= 0 ? K.resident : kMaxResidentCols, &P.slot_bytes,
                              &P.nslots, &P.xres_bytes, P.dir_cap, reserve);
    if (P.smem < 0) {
        msg = "sip kernel: a unit does not fit in shared memory";
        return DM_EINVAL;
    }
    return DM_OK;
}

int gemv_plan(const dm_tensor *t, int Mv, dm_launch_plan *out, std::string &msg) {
    SipPlan P;
    if (int rc = plan_sip(t, Mv, P, msg)) return rc;
    out->grid = (int32_t)P.grid;
    out->split = P.tile_split ? kSplitTiles : kSplitStreamK;
    out->slots = P.nslots;
    out->resident = P.xres_bytes > 0 ? 1 : 0;
    out->smem_bytes = P.smem;
    out->skew_step = P.part_r;
    return DM_OK;
}

int launch_gemv_sip(const dm_tensor *t, const uint16_t *xv, int64_t x_stride, int Mv, int nsplit, int M_out,
                    const uint16_t *bias, void *out, int out_f32, void *stream, std::string &msg) {
    return launch_gemv_sip_with(t, xv, x_stride, Mv, nsplit, M_out, bias, out, out_f32, t->S.partials,
                                t->S.counters, t->S.err, t->S.max_workers, stream, msg, nullptr);
}

// The sip GEMV for activations of either dtype at any element alignment:
// bf16 rows that start on a 16-byte boundary go to the kernel as they are
// (its bulk copies need 16-byte aligned sources); other bf16 rows are first
// copied into `xbuf`, and fp32 rows are split there into three bf16 pieces
// (hi, mid, lo) read as three virtual rows. `xbuf` holds `xcap` bf16
// elements, 16-byte aligned; rows go through it a chunk at a time, one launch
// per chunk. Activation row m's result is the same bits whatever the chunk:
// every sum's order depends on the tensor alone.
int gemv_sip_rows(const dm_tensor *t, const void *x, int x_f32, int64_t M, const uint16_t *bias, void *out,
                  int out_f32, uint16_t *xbuf, int64_t xcap, float *partials, int *counters, int64_t max_workers,
                  void *stream, std::string &msg) {
    const int64_t C = t->L.C;
    const size_t esz = out_f32 ? 4 : 2;
    const bool direct = !x_f32 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    if (direct)
        return launch_gemv_sip_with(t, reinterpret_cast<const uint16_t *>(x), C, (int)M, 1, (int)M, bias, out,
                                    out_f32, partials, counters, t->S.err, max_workers, stream, msg);
    // rows per chunk: fp32 rows take three bf16 rows of xbuf each (at most
    // two per launch: six virtual rows), bf16 rows one (at most six)
    const int64_t per = x_f32 ? std::min<int64_t>(2, xcap / (3 * C)) : std::min<int64_t>(6, xcap / C);
    if (per < 1) {
        msg = "sip kernel: an activation row of " + std::to_string(C) + " columns exceeds the " +
              std::to_string(xcap) + "-element staging buffer";
        return DM_EINVAL;
    }
    int rc = DM_OK;
    for (int64_t m0 = 0; m0 < M && rc == DM_OK; m0 += per) {
        const int64_t mm = std::min<int64_t>(per, M - m0);
        uint8_t *o = reinterpret_cast<uint8_t *>(out) + (size_t)m0 * t->L.rows * esz;
        if (x_f32) {
            rc = launch_split_f32(reinterpret_cast<const float *>(x) + m0 * C, C, mm, xbuf, stream, msg);
            if (rc == DM_OK)
                rc = launch_gemv_sip_with(t, xbuf, C, (int)(3 * mm), 3, (int)mm, bias, o, out_f32, partials, counters,
                                          t->S.err, max_workers, stream, msg);
        } else {
            rc = launch_copy_u16(reinterpret_cast<const uint16_t *>(x) + m0 * C, mm * C, xbuf, stream, msg);
            if (rc == DM_OK)
                rc = launch_gemv_sip_with(t, xbuf, C, (int)mm, 1, (int)mm, bias, o, out_f32, partials, counters,
                                          t->S.err, max_workers, stream, msg);
        }
    }
    return rc;
}

// The kernel arguments of one GEMV with caller-supplied scratch (partials
// for `max_workers` CTAs, per-tile counters that are zero on entry, the error
// word) under the tensor's launch plan. `reserve` bytes of shared memory are
// kept out of the plan (a chain launch keeps its link arguments there).
static int prepare_sip_args(const dm_tensor *t, const uint16_t *xv, int64_t x_stride, int Mv, int nsplit, int M_out,
                            const uint16_t *bias, void *out, int out_f32, float *partials, int *counters, int *err,
                            int64_t max_workers, const dm_gather *gather, SipArgs &a, SipPlan &P, std::string &msg,
                            int reserve = 0) {
    const dm::TensorLayout &L = t->L;
    if (Mv < 0 || Mv > kMaxVirtualRows) {  // 0: decode to bf16
        msg = "sip kernel: 1..8 virtual activation rows";
        return DM_EINVAL;
    }
    if (int rc = plan_sip(t, Mv, P, msg, reserve)) return rc;
    const int64_t tiles = L.tiles, grid = P.grid;
    if (grid > max_workers || grid > kMaxGrid) {
        msg = "sip kernel: " + std::to_string(grid) + " stream-K workers exceed the scratch's " +
              std::to_string(max_workers) + " (or the launch's " + std::to_string(kMaxGrid) + ")";
        return DM_EINVAL;
    }
    a = SipArgs{};
    a.data = t->d_data;
    a.unit16 = t->d_unit16;
    a.units = L.units;
    a.rows = L.rows;
    a.NB = L.NB;
    a.x = xv;
    a.x_stride = x_stride;
    a.Mv = Mv;
    a.nsplit = nsplit;
    a.M_out = M_out;
    a.bias = bias;
    a.out = out;
    a.out_f32 = out_f32;
    a.partials = partials;
    a.counters = counters;
    a.err = err;
    a.slot_bytes = P.slot_bytes;
    a.xres_bytes = P.xres_bytes;
    a.x_off = (L.max_unit_bytes + 127) & ~127;
    a.nslots = P.nslots;
    a.dir_cap = P.dir_cap;
    a.tile_split = P.tile_split;
    a.grid = (int32_t)grid;
    a.prefetch = Mv > 0 ? (t->K.prefetch >= 0 ? t->K.prefetch : kPrefetchUnits) : 0;
    for (int64_t w = 0; w <= grid; ++w)
        a.starts[w] = (int32_t)(P.tile_split ? (w * tiles / grid) * L.NB
                                             : L.units * part_sum(w, P.part_b0, P.part_r) /
                                                   part_sum(grid, P.part_b0, P.part_r));
    if (gather) {
        a.world = gather->world;
        a.rank = gather->rank;
        a.gslot = gather->slot;
        for (int r = 0; r < gather->world; ++r) {
            a.peer_out[r] = gather->peer_out[r];
            a.peer_flags[r] = gather->peer_flags[r];
        }
        a.gen = gather->gen;
        a.done = gather->done;
        a.wait_flags = gather->wait_flags;
        a.wait_gen = gather->wait_gen;
        a.abort = gather->abort;
        a.wait_polls = gather->wait_polls ? gather->wait_polls : kPeerPolls;
    }
    return DM_OK;
}

// The launch with caller-supplied scratch: dm_gemv passes the tensor's own,
// dm_gemv_noalloc a static device array.
int launch_gemv_sip_with(const dm_tensor *t, const uint16_t *xv, int64_t x_stride, int Mv, int nsplit, int M_out,
                         const uint16_t *bias, void *out, int out_f32, float *partials, int *counters, int *err,
                         int64_t max_workers, void *stream, std::string &msg, const dm_gather *gather) {
    SipArgs a;
    SipPlan P;
    if (int rc = prepare_sip_args(t, xv, x_stride, Mv, nsplit, M_out, bias, out, out_f32, partials, counters, err,
                                  max_workers, gather, a, P, msg))
        return rc;
    using Kern = void (*)(SipArgs);
    static const Kern kernels[2][kMaxVirtualRows + 1] = {
        {sip_gemv_kernel<0, false>, sip_gemv_kernel<1, false>, sip_gemv_kernel<2, false>, sip_gemv_kernel<3, false>,
         sip_gemv_kernel<4, false>, sip_gemv_kernel<5, false>, sip_gemv_kernel<6, false>, sip_gemv_kernel<7, false>,
         sip_gemv_kernel<8, false>},
        {nullptr, sip_gemv_kernel<1, true>, sip_gemv_kernel<2, true>, sip_gemv_kernel<3, true>,
         sip_gemv_kernel<4, true>, sip_gemv_kernel<5, true>, sip_gemv_kernel<6, true>, sip_gemv_kernel<7, true>,
         sip_gemv_kernel<8, true>}};
    // the shared-memory limit is a per-device attribute of each kernel: one
    // bit per device (devices 64 and up set it on every launch)
    static std::atomic<uint64_t> attr_set[2][kMaxVirtualRows + 1];
    const int res = P.xres_bytes > 0 ? 1 : 0;
    const uint64_t dev_bit = t->device >= 0 && t->device < 64 ? 1ull << t->device : 0ull;
    const Kern kern = kernels[res][Mv];
    if (kern == nullptr) {
        msg = "sip kernel: no resident-activation kernel without activations";
        return DM_EINVAL;
    }
    if (!dev_bit || !(attr_set[res][Mv].load() & dev_bit)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) {
            msg = std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e);
            return DM_ECUDA;
        }
        attr_set[res][Mv].fetch_or(dev_bit);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)P.grid);
    cfg.blockDim = dim3(kSipThreads);
    cfg.dynamicSmemBytes = (size_t)P.smem;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
    if (e != cudaSuccess) {
        msg = std::string("sip_gemv_kernel: ") + cudaGetErrorString(e);
        return DM_ECUDA;
    }
    return DM_OK;
}

// Room behind a chain's largest plan: two links' arguments (this one's and
// the next one's) and the launch count read at entry.
constexpr int kChainArgsBytes = (2 * (int)sizeof(SipArgs) + 16 + 127) & ~127;

int chain_prepare(const dm_chain_link *links, int32_t n, int64_t M, int32_t out_f32, std::vector<SipArgs> &args,
                  int *grid, int *smem, std::string &msg) {
    args.resize((size_t)n);
    *grid = 0;
    *smem = 0;
    for (int32_t i = 0; i < n; ++i) {
        const dm_chain_link &k = links[i];
        const std::string at = "dm_chain_create: link " + std::to_string(i) + ": ";
        if (!k.t || !k.x) {
            msg = at + "null tensor or activations";
            return DM_EINVAL;
        }
        if (!k.t->L.fast_sip) {
            msg = at + "needs a sip tensor (the fast path)";
            return DM_EINVAL;
        }
        if (k.t->device != links[0].t->device) {
            msg = at + "tensors on different devices";
            return DM_EINVAL;
        }
        if ((reinterpret_cast<uintptr_t>(k.x) & 15) != 0) {
            msg = at + "activations must be 16-byte aligned";
            return DM_EINVAL;
        }
        const dm_gather &g = k.g;
        if (g.world < 1 || g.world > DM_MAX_RANKS || g.rank < 0 || g.rank >= g.world) {
            msg = at + "rank outside a world of 1.." + std::to_string(DM_MAX_RANKS);
            return DM_EINVAL;
        }
        if (g.slot < k.t->L.rows) {
            msg = at + "slot smaller than this rank's rows";
            return DM_EINVAL;
        }
        for (int r = 0; r < g.world; ++r)
            if (!g.peer_out[r] || !g.peer_flags[r]) {
                msg = at + "null peer pointer";
                return DM_EINVAL;
            }
        if (!g.gen || !g.done || !g.abort) {
            msg = at + "counters incomplete";
            return DM_EINVAL;
        }
        if (k.wait < -1 || k.wait >= n) {
            msg = at + "wait index outside -1.." + std::to_string(n - 1);
            return DM_EINVAL;
        }
        if (k.wait >= 0 && (links[k.wait].g.world != g.world || links[k.wait].g.rank != g.rank)) {
            msg = at + "waits on a link of another world";
            return DM_EINVAL;
        }
        dm_gather gg = g;
        gg.wait_flags = k.wait >= 0 ? links[k.wait].g.peer_flags[g.rank] : nullptr;
        gg.wait_gen = nullptr;
        SipPlan P;
        if (int rc = prepare_sip_args(k.t, reinterpret_cast<const uint16_t *>(k.x), k.t->L.C, (int)M, 1, (int)M,
                                      reinterpret_cast<const uint16_t *>(k.bias), nullptr, out_f32, k.t->S.partials,
                                      k.t->S.counters, k.t->S.err, k.t->S.max_workers, &gg, args[(size_t)i], P, msg,
                                      kChainArgsBytes)) {
            msg = at + msg;
            return rc;
        }
        args[(size_t)i].wait_prev = k.wait >= i ? 1 : 0;
        *grid = std::max<int>(*grid, (int)P.grid);
        *smem = std::max<int>(*smem, (P.smem + 127) & ~127);
    }
    // one rank: a link polls its predecessor's CTA count itself
    for (int32_t i = 0; i < n; ++i)
        if (links[i].wait >= 0 && links[i].g.world == 1) {
            args[(size_t)i].wait_done = links[links[i].wait].g.done;
            args[(size_t)i].wait_grid = args[(size_t)links[i].wait].grid;
        }
    return DM_OK;
}

int launch_chain(const SipArgs *d_links, int32_t n, int Mv, int grid, int smem, uint32_t *words, int device,
                 void *stream, std::string &msg) {
    using Kern = void (*)(const SipArgs *, int32_t, uint32_t *, int32_t);
    static const Kern kernels[kMaxVirtualRows + 1] = {
        nullptr, sip_chain_kernel<1>, sip_chain_kernel<2>, sip_chain_kernel<3>, sip_chain_kernel<4>,
        sip_chain_kernel<5>, sip_chain_kernel<6>, sip_chain_kernel<7>, sip_chain_kernel<8>};
    static std::atomic<uint64_t> attr_set[kMaxVirtualRows + 1];
    if (Mv < 1 || Mv > kMaxVirtualRows) {
        msg = "dm_chain: 1..8 activation rows";
        return DM_EINVAL;
    }
    const Kern kern = kernels[Mv];
    const uint64_t dev_bit = device >= 0 && device < 64 ? 1ull << device : 0ull;
    if (!dev_bit || !(attr_set[Mv].load() & dev_bit)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) {
            msg = std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e);
            return DM_ECUDA;
        }
        attr_set[Mv].fetch_or(dev_bit);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kSipThreads);
    cfg.dynamicSmemBytes = (size_t)smem + kChainArgsBytes;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // the links wait on one another's CTAs
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, d_links, n, words, (int32_t)smem);
    if (e != cudaSuccess) {
        msg = std::string("sip_chain_kernel: ") + cudaGetErrorString(e);
        return DM_ECUDA;
    }
    return DM_OK;
}

int launch_decode_sip(const dm_tensor *t, uint16_t *out, void *stream, std::string &msg) {
    const TensorLayout &L = t->L;
    if (!L.fast_sip) {
        msg = "sip decode: not a sip tensor";
        return DM_EINVAL;
    }
    if ((reinterpret_cast<uintptr_t>(out) & 15) != 0) {
        msg = "dm_decode: output of a sip tensor must be 16-byte aligned";
        return DM_EINVAL;
    }
    if (L.units == 0) return DM_OK;
    // the GEMV kernel's pipeline in its decode mode (no activations)
    return launch_gemv_sip_with(t, nullptr, 0, 0, 1, 1, nullptr, out, 0, t->S.partials, t->S.counters, t->S.err,
                                t->S.max_workers, stream, msg);
}

}  // namespace dm

// ------------------------------------------------------------ the chain --

struct dm_chain {
    int32_t device = 0, n = 0, Mv = 0, grid = 0, smem = 0;
    dm::SipArgs *d_links = nullptr;
    uint32_t *d_words = nullptr;  // [0] the chain's launch count, [1] CTAs that have left the running launch
    void *d_alloc = nullptr;
};

namespace {

struct ChainDevice {
    int prev = -1;
    explicit ChainDevice(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~ChainDevice() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

int chain_fail(char *err, size_t len, int code, const std::string &msg) {
    dm::set_error(err, len, msg);
    return code;
}

}  // namespace

extern "C" int dm_chain_create(const dm_chain_link *links, int32_t n, int64_t M, int32_t out_dtype, dm_chain **out,
                               char *err, size_t err_len) {
    if (!links || !out || n < 1) return chain_fail(err, err_len, DM_EINVAL, "dm_chain_create: no links");
    *out = nullptr;
    if (M < 1 || M > DM_MC_MAX)
        return chain_fail(err, err_len, DM_EINVAL,
                          "radix gemv_mc: M=" + std::to_string(M) + " outside 1.." + std::to_string(DM_MC_MAX));
    if (out_dtype != DM_BF16 && out_dtype != DM_F32)
        return chain_fail(err, err_len, DM_EINVAL, "dm_chain_create: dtype must be DM_BF16 or DM_F32");
    if (!links[0].t) return chain_fail(err, err_len, DM_EINVAL, "dm_chain_create: link 0: null tensor or activations");
    std::vector<dm::SipArgs> args;
    int grid = 0, smem = 0;
    std::string msg;
    if (int rc = dm::chain_prepare(links, n, M, out_dtype == DM_F32, args, &grid, &smem, msg))
        return chain_fail(err, err_len, rc, msg);
    auto *c = new dm_chain;
    c->device = links[0].t->device;
    c->n = n;
    c->Mv = (int32_t)M;
    c->grid = grid;
    c->smem = smem;
    ChainDevice g(c->device);
    const size_t abytes = ((size_t)n * sizeof(dm::SipArgs) + 255) & ~(size_t)255;
    cudaError_t e = cudaMalloc(&c->d_alloc, abytes + 256);
    if (e == cudaSuccess) {
        c->d_links = reinterpret_cast<dm::SipArgs *>(c->d_alloc);
        c->d_words = reinterpret_cast<uint32_t *>(reinterpret_cast<uint8_t *>(c->d_alloc) + abytes);
        e = cudaMemcpy(c->d_links, args.data(), (size_t)n * sizeof(dm::SipArgs), cudaMemcpyHostToDevice);
    }
    if (e == cudaSuccess) e = cudaMemset(c->d_words, 0, 256);
    if (e != cudaSuccess) {
        if (c->d_alloc) cudaFree(c->d_alloc);
        delete c;
        return chain_fail(err, err_len, e == cudaErrorMemoryAllocation ? DM_ENOMEM : DM_ECUDA,
                          std::string("dm_chain_create: ") + cudaGetErrorString(e));
    }
    *out = c;
    return DM_OK;
}

extern "C" int dm_chain_run(const dm_chain *c, void *stream, char *err, size_t err_len) {
    if (!c) return chain_fail(err, err_len, DM_EINVAL, "dm_chain_run: null chain");
    ChainDevice g(c->device);
    std::string msg;
    if (int rc = dm::launch_chain(c->d_links, c->n, c->Mv, c->grid, c->smem, c->d_words, c->device, stream, msg))
        return chain_fail(err, err_len, rc, msg);
    return DM_OK;
}

extern "C" int dm_chain_destroy(dm_chain *c, char *err, size_t err_len) {
    if (!c) return chain_fail(err, err_len, DM_EINVAL, "dm_chain_destroy: null chain");
    ChainDevice g(c->device);
    cudaError_t e = cudaFree(c->d_alloc);
    delete c;
    if (e != cudaSuccess) return chain_fail(err, err_len, DM_ECUDA, std::string("dm_chain_destroy: ") + cudaGetErrorString(e));
    return DM_OK;
}
