// The pack encoder: uint16 BF16 bit patterns -> pack format 1 radix arrays,
// byte-identical to the reference's writers (src/drinkme/codec/radix.py:
// 77-136 `pack_array`; the native plan/encode of radix_native.cpp:57-166,
// which write the same bytes, pinned by the reference's
// tests/test_radix_pack.py).
//
// Format rules it follows (the algorithm has to be the reference's, the
// code is this library's own): the palette is the exponents ordered by
// frequency over the whole tensor, ties by the lower exponent, the first
// sum(2^w - 1) of them split across the nonterminal tiers; a weight whose
// exponent has palette rank k codes min(k - base, 2^w - 1) at each tier it
// reaches (the top code escapes to the next tier, over only the weights
// that escaped); the weights that escape every tier store their 8-bit
// exponent in the terminal stream; every stream is padded to whole
// little-endian uint32 words; the directory holds each block's first word.
#include <algorithm>
#include <array>
#include <atomic>
#include <cstring>
#include <numeric>
#include <thread>
#include <vector>

#include "dm_internal.h"

namespace {

int pool_size(int32_t threads, int64_t work) {
    unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    int64_t t = threads > 0 ? threads : (int64_t)hw;
    return (int)std::max<int64_t>(1, std::min<int64_t>(t, std::max<int64_t>(1, work / 64)));
}

template <class F>
void run_blocks(int64_t nblk, int32_t threads, F fn) {
    int nt = pool_size(threads, nblk);
    if (nt <= 1) {
        for (int64_t i = 0; i < nblk; ++i) fn(i);
        return;
    }
    std::atomic<int64_t> next(0);
    std::vector<std::thread> pool;
    for (int t = 0; t < nt; ++t)
        pool.emplace_back([&]() {
            for (;;) {
                int64_t s = next.fetch_add(256);
                if (s >= nblk) break;
                int64_t e = std::min(nblk, s + 256);
                for (int64_t i = s; i < e; ++i) fn(i);
            }
        });
    for (auto &th : pool) th.join();
}

struct Plan {
    int32_t covered = 0;
    std::array<uint16_t, 256> rank{};  // exponent -> palette rank (covered when absent)
};

inline int64_t cw(int64_t count, int64_t width) { return (count * width + 31) / 32; }

// Appends `width`-bit little-endian fields into a zeroed word stream.
struct FieldWriter {
    uint32_t *w;
    uint64_t bit = 0;
    explicit FieldWriter(uint32_t *words) : w(words) {}
    inline void put(uint32_t v, uint32_t width) {
        uint32_t lo = (uint32_t)(bit & 31);
        uint64_t wi = bit >> 5;
        w[wi] |= v << lo;
        if (lo + width > 32) w[wi + 1] |= v >> (32 - lo);
        bit += width;
    }
};

}  // namespace

namespace dm {

int check_pack_params(int64_t R, int64_t C, const int32_t *widths, int32_t nw, int32_t B, int32_t *covered,
                      std::string &msg) {
    if (R <= 0 || C <= 0) { msg = "expected a nonempty 2D uint16 array of bf16 bit patterns"; return 1; }
    if (B < 32 || B > 4096 || (B & (B - 1))) { msg = "block_size must be a power of two from 32 through 4096"; return 1; }
    if (nw < 2 || nw > 8 || widths[nw - 1] != 8) {
        msg = "radix needs 2..8 widths in 1..8, ending with the exponent width";
        return 1;
    }
    int32_t c = 0;
    for (int i = 0; i < nw; ++i)
        if (widths[i] < 1 || widths[i] > 8) {
            msg = "radix needs 2..8 widths in 1..8, ending with the exponent width";
            return 1;
        }
    for (int i = 0; i < nw - 1; ++i) c += (1 << widths[i]) - 1;
    if (c > 256) { msg = "radix tiers exceed the exponent alphabet"; return 1; }
    *covered = c;
    return 0;
}

void palette_from_histogram(const uint64_t *hist, int32_t covered, uint8_t *palette_out, uint16_t *rank) {
    std::array<int, 256> order;
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return hist[a] > hist[b]; });
    for (int e = 0; e < 256; ++e) rank[e] = (uint16_t)covered;
    for (int k = 0; k < covered; ++k) {
        palette_out[k] = (uint8_t)order[k];
        rank[order[k]] = (uint16_t)k;
    }
}

}  // namespace dm

extern "C" int dm_pack_plan(const uint16_t *bits, int64_t R, int64_t C, const int32_t *widths, int32_t nw,
                            int32_t B, int32_t threads, uint8_t *palette_out, uint32_t *offsets_out,
                            uint64_t *nwords, char *err, size_t err_len) {
    std::string msg;
    int32_t covered;
    if (!bits || !widths || !palette_out || !offsets_out || !nwords) {
        dm::set_error(err, err_len, "dm_pack_plan: null pointer");
        return DM_EINVAL;
    }
    if (dm::check_pack_params(R, C, widths, nw, B, &covered, msg)) { dm::set_error(err, err_len, msg); return DM_EINVAL; }
    const int64_t NB = (C + B - 1) / B, nblk = R * NB;
    // histogram over the whole tensor, one partial per row range
    int nt = pool_size(threads, R * C / 4096 + 1);
    std::vector<std::array<uint64_t, 256>> parts(nt);
    {
        std::vector<std::thread> pool;
        for (int t = 0; t < nt; ++t)
            pool.emplace_back([&, t]() {
                auto &h = parts[t];
                h.fill(0);
                int64_t r0 = R * t / nt, r1 = R * (t + 1) / nt;
                for (int64_t i = r0 * C; i < r1 * C; ++i) ++h[(bits[i] >> 7) & 0xFF];
            });
        for (auto &th : pool) th.join();
    }
    std::array<uint64_t, 256> hist{};
    for (auto &h : parts)
        for (int e = 0; e < 256; ++e) hist[e] += h[e];
    std::array<uint16_t, 256> rank;
    dm::palette_from_histogram(hist.data(), covered, palette_out, rank.data());
    // per-block word counts, then the directory
    std::vector<uint32_t> words(nblk);
    run_blocks(nblk, threads, [&](int64_t blk) {
        int64_t r = blk / NB, b = blk % NB, c0 = b * B, n = std::min<int64_t>(B, C - c0);
        const uint16_t *src = bits + r * C + c0;
        // how many weights reach each tier: count ranks past each tier's base
        std::array<uint32_t, 257> per_rank{};
        for (int64_t i = 0; i < n; ++i) ++per_rank[rank[(src[i] >> 7) & 0xFF]];
        int64_t total = cw(n, 8), active = n, base = 0;
        for (int t = 0; t < nw - 1; ++t) {
            total += cw(active, widths[t]);
            int64_t esc = (1 << widths[t]) - 1;
            for (int64_t k = base; k < base + esc; ++k) active -= per_rank[k];
            base += esc;
        }
        total += cw(active, 8);
        words[blk] = (uint32_t)total;
    });
    uint64_t acc = 0;
    offsets_out[0] = 0;
    for (int64_t blk = 0; blk < nblk; ++blk) {
        acc += words[blk];
        if (acc > UINT32_MAX) {
            dm::set_error(err, err_len, "radix payload exceeds the uint32 word directory");
            return DM_EINVAL;
        }
        offsets_out[blk + 1] = (uint32_t)acc;
    }
    *nwords = acc;
    return DM_OK;
}

extern "C" int dm_pack_encode(const uint16_t *bits, int64_t R, int64_t C, const int32_t *widths, int32_t nw,
                              int32_t B, int32_t threads, const uint8_t *palette, const uint32_t *offsets,
                              uint32_t *data, uint64_t nwords, char *err, size_t err_len) {
    std::string msg;
    int32_t covered;
    if (!bits || !widths || !palette || !offsets || !data) {
        dm::set_error(err, err_len, "dm_pack_encode: null pointer");
        return DM_EINVAL;
    }
    if (dm::check_pack_params(R, C, widths, nw, B, &covered, msg)) { dm::set_error(err, err_len, msg); return DM_EINVAL; }
    const int64_t NB = (C + B - 1) / B, nblk = R * NB;
    if (offsets[0] != 0 || offsets[nblk] != nwords) {
        dm::set_error(err, err_len, "directory endpoints");
        return DM_EINVAL;
    }
    std::array<uint16_t, 256> rank;
    rank.fill((uint16_t)covered);
    for (int k = 0; k < covered; ++k) rank[palette[k]] = (uint16_t)k;
    std::atomic<int> bad(0);
    run_blocks(nblk, threads, [&](int64_t blk) {
        int64_t r = blk / NB, b = blk % NB, c0 = b * B, n = std::min<int64_t>(B, C - c0);
        const uint16_t *src = bits + r * C + c0;
        uint32_t *out = data + offsets[blk];
        const int64_t avail = (int64_t)offsets[blk + 1] - (int64_t)offsets[blk];
        std::memset(out, 0, (size_t)avail * 4);
        std::vector<uint16_t> rk(n), ex(n);
        int64_t pos = 0;
        {
            FieldWriter fw(out);
            for (int64_t i = 0; i < n; ++i) {
                uint16_t v = src[i];
                fw.put((uint32_t)((v & 0x7F) | ((v >> 8) & 0x80)), 8);
                ex[i] = (uint16_t)((v >> 7) & 0xFF);
                rk[i] = rank[ex[i]];
            }
            pos = cw(n, 8);
        }
        int64_t active = n, base = 0;
        for (int t = 0; t < nw - 1 && !bad.load(std::memory_order_relaxed); ++t) {
            uint32_t w = (uint32_t)widths[t], esc = (1u << w) - 1;
            if (pos + cw(active, w) > avail) { bad = 1; return; }
            FieldWriter fw(out + pos);
            int64_t kept = 0;
            for (int64_t i = 0; i < active; ++i) {
                uint32_t code = (uint32_t)std::min<int64_t>((int64_t)rk[i] - base, esc);
                fw.put(code, w);
                if (code == esc) { rk[kept] = rk[i]; ex[kept] = ex[i]; ++kept; }
            }
            pos += cw(active, w);
            active = kept;
            base += esc;
        }
        if (pos + cw(active, 8) != avail) { bad = 1; return; }
        FieldWriter fw(out + pos);
        for (int64_t i = 0; i < active; ++i) fw.put(ex[i], 8);
    });
    if (bad) {
        dm::set_error(err, err_len, "terminal stream mismatch: the directory does not match these bits");
        return DM_EINVAL;
    }
    return DM_OK;
}
