// Host side of the loader: descriptor validation and the B200 device layout.
//
// The pack stays pack format 1 on disk (src/drinkme/codec/radix_pack.py:9-21).
// What changes is only where the bytes sit on the device: the reference keeps
// the payload verbatim plus a zero pad (swap.to_device_radix,
// src/drinkme/codec/swap.py:80-161); this loader regroups the same block
// words into UNITS of 16 rows x 1 block column, each unit contiguous and
// 16-byte aligned so one bulk copy stages it into shared memory:
//
//   unit  = [16 x RowEntry header][sip exponent tables, 16 bytes]
//           [row-block streams, each 16-byte aligned]
//           [sip fast path: per row, the escape index — the uint16 position
//            of every tier-0 escape (code 7) in block order, 16-byte aligned]
//           [sip fast path, ragged last tile only: one null block whose
//            weights all decode to +0]
//   units in tile-major order (tile = 16 rows; all block columns of a tile
//   before the next tile), then a zero tail pad as long as the widest block
//   (radix.block_word_bounds(B)[1] words), so no reader leaves the buffer.
//
// A FUSED tensor concatenates the rows of several packs sharing their
// columns (q, k and v; gate and up): each part keeps its own palette, whose
// tables ride in the header of every unit of its tiles.
#include <algorithm>
#include <atomic>
#include <cstring>
#include <thread>
#include <vector>

#include "dm_internal.h"

namespace dm {

static int64_t cw(int64_t count, int64_t width) { return (count * width + 31) / 32; }

int64_t block_words_most(int64_t n, const int32_t *widths, int32_t nw) {
    int64_t m = cw(n, 8);
    for (int i = 0; i < nw - 1; ++i) m += cw(n, widths[i]);
    return m + cw(n, 8);
}

static int64_t block_words_fewest(int64_t n, const int32_t *widths) { return cw(n, 8) + cw(n, widths[0]); }

template <class F>
static void parallel_for(int64_t n, F fn) {
    unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    int64_t threads = std::min<int64_t>(hw, std::max<int64_t>(1, n / 256));
    if (threads <= 1) {
        for (int64_t i = 0; i < n; ++i) fn(i);
        return;
    }
    std::atomic<int64_t> next(0);
    std::vector<std::thread> pool;
    for (int64_t t = 0; t < threads; ++t)
        pool.emplace_back([&]() {
            for (;;) {
                int64_t s = next.fetch_add(1024);
                if (s >= n) break;
                int64_t e = std::min(n, s + 1024);
                for (int64_t i = s; i < e; ++i) fn(i);
            }
        });
    for (auto &th : pool) th.join();
}

// radix.py:174-238 (validate) with its messages, plus the widths rule of
// radix.py:139-146.
int validate_pack(const uint8_t *palette, size_t npal, const uint32_t *offsets, size_t noff, size_t nwords,
                  int64_t R, int64_t C, const int32_t *widths, int32_t nw, int32_t B, std::string &msg) {
    if (R <= 0 || C <= 0) { msg = "invalid radix shape or raw flag"; return 1; }
    if (B < 32 || B > 4096 || (B & (B - 1))) { msg = "invalid radix block size"; return 1; }
    if (nw < 2 || nw > 8 || widths[nw - 1] != 8) {
        msg = "radix needs 2..8 widths in 1..8, ending with the exponent width";
        return 1;
    }
    int64_t covered = 0;
    for (int i = 0; i < nw; ++i)
        if (widths[i] < 1 || widths[i] > 8) {
            msg = "radix needs 2..8 widths in 1..8, ending with the exponent width";
            return 1;
        }
    for (int i = 0; i < nw - 1; ++i) covered += (1 << widths[i]) - 1;
    if (covered > 256) { msg = "radix tiers exceed the exponent alphabet"; return 1; }
    if ((int64_t)npal != covered) { msg = "invalid radix palette entries"; return 1; }
    bool seen[256] = {false};
    for (size_t i = 0; i < npal; ++i) {
        if (seen[palette[i]]) { msg = "invalid radix palette entries"; return 1; }
        seen[palette[i]] = true;
    }
    int64_t per_row = (C + B - 1) / B, nb = R * per_row;
    if ((int64_t)noff != nb + 1 || offsets[0] != 0 || (int64_t)offsets[nb] != (int64_t)nwords) {
        msg = "invalid radix block offsets";
        return 1;
    }
    for (int64_t i = 0; i < nb; ++i) {
        if (offsets[i + 1] <= offsets[i]) { msg = "invalid radix block offsets"; return 1; }
    }
    for (int64_t i = 0; i < nb; ++i) {
        int64_t n = std::min<int64_t>(B, C - (i % per_row) * B);
        int64_t len = (int64_t)offsets[i + 1] - (int64_t)offsets[i];
        int64_t fewest = block_words_fewest(n, widths), most = block_words_most(n, widths, nw);
        if (len < fewest) {
            msg = "invalid radix block offsets: block " + std::to_string(i) + " holds " + std::to_string(len) +
                  " word(s), fewer than the " + std::to_string(fewest) + " its literal plane and first tier take for " +
                  std::to_string(n) + " weights";
            return 1;
        }
        if (len > most) {
            msg = "invalid radix block offsets: block " + std::to_string(i) + " holds " + std::to_string(len) +
                  " words, more than the " + std::to_string(most) + " any block of " + std::to_string(n) +
                  " weights can use";
            return 1;
        }
    }
    return 0;
}

static inline uint32_t field_at(const uint32_t *w, int64_t avail, int64_t index, int32_t width) {
    int64_t bit = index * width;
    int64_t wi = bit >> 5;
    uint32_t lo = (uint32_t)(bit & 31);
    uint64_t a = wi < avail ? w[wi] : 0, b = wi + 1 < avail ? w[wi + 1] : 0;
    uint64_t v = (a >> lo) | (lo + width > 32 ? (b << (32 - lo)) : 0);
    return (uint32_t)(v & ((1u << width) - 1));
}

// The sip escape positions of one full 1024-weight block: tier-0 codes
// equal to 7, in block order. Counts only; positions written when out != 0.
static int sip_escapes(const uint32_t *tier0, uint16_t *out) {
    int count = 0;
    for (int g = 0; g < 32; ++g) {  // 32 codes per 3 words
        unsigned __int128 v = (unsigned __int128)tier0[3 * g] | ((unsigned __int128)tier0[3 * g + 1] << 32) |
                              ((unsigned __int128)tier0[3 * g + 2] << 64);
        unsigned __int128 f = v & (v >> 1) & (v >> 2);
        uint32_t m = 0;
        for (int j = 0; j < 32; ++j) m |= (uint32_t)((f >> (3 * j)) & 1) << j;
        while (m) {
            int j = __builtin_ctz(m);
            m &= m - 1;
            if (out) out[count] = (uint16_t)(32 * g + j);
            ++count;
        }
    }
    return count;
}

// The device form of a sip block's tier-0 codes (the pack's 3-bit stream,
// code k at bits 3k..3k+2, 96 words) for the kernels' decode: two planes in
// the same 384 bytes. The kernels decode 16 weights k = 64q + 16t + [0, 16)
// per lane and need their codes as nibbles; from these planes that takes a
// mask and an OR per 8 codes instead of a bit-spreading sequence.
//   words 0..63, word 4q + t: bits 2j, 2j + 1 = the low two bits of the code
//     of weight j / 2 (j even) or 8 + j / 2 (j odd) of lane t's 16;
//   words 64..95, word 64 + 2q + t / 2: bit 2 of those codes; weight w < 8
//     at bit 4w (t even) or 4w + 2 (t odd), weight 8 + w at 4w + 1 or 4w + 3.
static void sip_code_planes(const uint32_t *src, uint32_t *dst) {
    for (int i = 0; i < 96; ++i) dst[i] = 0;
    for (int k = 0; k < 1024; ++k) {
        const int b = 3 * k;
        const uint64_t two = (uint64_t)src[b >> 5] | ((b >> 5) + 1 < 96 ? (uint64_t)src[(b >> 5) + 1] << 32 : 0);
        const uint32_t c = (uint32_t)(two >> (b & 31)) & 7u;
        const int q = k >> 6, t = (k >> 4) & 3, w = k & 15;
        const int j = w < 8 ? 2 * w : 2 * (w - 8) + 1;
        dst[4 * q + t] |= (c & 3u) << (2 * j);
        const int pos = w < 8 ? 4 * w + ((t & 1) ? 2 : 0) : 4 * (w - 8) + ((t & 1) ? 3 : 1);
        dst[64 + 2 * q + (t >> 1)] |= ((c >> 2) & 1u) << pos;
    }
}

// One block of any radix profile decoded to bf16 bit patterns (radix.py:
// 241-278, the reference's CPU decode): the literal plane, then per
// nonterminal tier the codes of the weights still active (an escape code
// passes the weight on to the next tier), then the terminal exponents.
// Words the block does not hold read as zero.
static void decode_block(const uint32_t *blk, int64_t words, int64_t n, const uint8_t *palette,
                         const int32_t *widths, int32_t nw, uint16_t *out) {
    uint32_t lit[4096], expo[4096];
    int32_t active[4096];
    int64_t pos = 0;
    for (int64_t i = 0; i < n; ++i) lit[i] = field_at(blk, words, i, 8);
    pos += cw(n, 8);
    int64_t count = n, base = 0;
    for (int64_t i = 0; i < n; ++i) active[i] = (int32_t)i;
    for (int t = 0; t < nw - 1; ++t) {
        const int32_t w = widths[t];
        const uint32_t esc = (1u << w) - 1;
        int64_t kept = 0;
        for (int64_t i = 0; i < count; ++i) {
            const uint32_t code = field_at(blk + pos, words - pos, i, w);
            if (code == esc) {
                active[kept++] = active[i];
            } else {
                expo[active[i]] = palette[base + code];
            }
        }
        pos += cw(count, w);
        base += esc;
        count = kept;
    }
    for (int64_t i = 0; i < count; ++i) expo[active[i]] = field_at(blk + pos, words - pos, i, 8);
    for (int64_t i = 0; i < n; ++i)
        out[i] = (uint16_t)((lit[i] & 0x7Fu) | ((lit[i] >> 7) << 15) | (expo[i] << 7));
}

// Rows [P.row0, P.row1) of a validated pack as bf16 bit patterns.
void decode_rows(const PackPart &P, uint16_t *out) {
    const int64_t NB = (P.C + P.B - 1) / P.B, rows = P.row1 - P.row0;
    parallel_for(rows * NB, [&](int64_t i) {
        const int64_t r = P.row0 + i / NB, b = i % NB, gb = r * NB + b;
        const int64_t n = std::min<int64_t>(P.B, P.C - b * P.B);
        const int64_t start = P.offsets[gb], words = (int64_t)P.offsets[gb + 1] - start;
        decode_block(P.data + start, words, n, P.palette, P.widths, P.nw, out + (i / NB) * P.C + b * P.B);
    });
}

// radix_ops.read_bytes (radix_ops.py:435-441) of rows [row0, row1) of a
// pack: its payload words, its slice of the directory, the padded palette
// words (radix_pack.py:333-350) and, for more than one nonterminal tier,
// the uint16 schedule.
int64_t pack_read_bytes(const PackPart &P, int64_t *payload_words) {
    const int64_t NB = (P.C + P.B - 1) / P.B, b0 = P.row0 * NB, nb = (P.row1 - P.row0) * NB;
    const int64_t words = (int64_t)P.offsets[b0 + nb] - (int64_t)P.offsets[b0];
    int64_t pal_words = 0;
    for (int i = 0; i < P.nw - 1; ++i) pal_words += (((1 << P.widths[i]) - 1) + 3) / 4;
    if (payload_words) *payload_words = words;
    return words * 4 + (nb + 1) * 4 + pal_words * 4 + (P.nw > 2 ? nb * 2 : 0);
}

// radix_pack.py:376-411 (schedule_np) for one block: byte (k-1) = word
// length of nonterminal tier k (k >= 1); reads past `avail` are zero.
static uint16_t block_schedule(const uint32_t *blk, int64_t avail, int64_t n, const int32_t *widths, int32_t nw) {
    if (nw <= 2) return 0;
    int64_t pos = cw(n, 8), count = n;
    uint32_t header = 0;
    for (int t = 0; t < nw - 1; ++t) {
        int32_t w = widths[t];
        int64_t words = cw(count, w);
        if (t > 0) header |= (uint32_t)words << ((t - 1) * 8);
        if (t < nw - 2) {
            uint32_t esc = (1u << w) - 1;
            int64_t kept = 0;
            for (int64_t i = 0; i < count; ++i)
                if (field_at(blk + pos, avail - pos, i, w) == esc) ++kept;
            count = kept;
        }
        pos += words;
    }
    return (uint16_t)header;
}

static inline int64_t a16(int64_t bytes) { return (bytes + 15) & ~int64_t(15); }

// The sip exponent tables of a part (the kernels' PRMT lookups): high part
// p >> 1 with 0x80 at the escape code 7, low part (p & 1) << 7 with 0x7F at
// code 7, each eight bytes as two words.
static void sip_tables(const uint8_t *palette, uint32_t tab[4]) {
    uint8_t th[8], tl[8];
    for (int c = 0; c < 7; ++c) {
        th[c] = (uint8_t)(palette[c] >> 1);
        tl[c] = (uint8_t)((palette[c] & 1u) << 7);
    }
    th[7] = 0x80;  // escape marker: zeroes the sign in the high byte
    tl[7] = 0x7F;  // escape: zeroes the mantissa in the low byte
    tab[0] = th[0] | (th[1] << 8) | (th[2] << 16) | ((uint32_t)th[3] << 24);
    tab[1] = th[4] | (th[5] << 8) | (th[6] << 16) | ((uint32_t)th[7] << 24);
    tab[2] = tl[0] | (tl[1] << 8) | (tl[2] << 16) | ((uint32_t)tl[3] << 24);
    tab[3] = tl[4] | (tl[5] << 8) | (tl[6] << 16) | ((uint32_t)tl[7] << 24);
}

int build_layout(const PackPart *parts, int nparts, TensorLayout &L, std::string &bytes, std::string &unit16,
                 std::string &msg, std::string *rowdir) {
    if (nparts < 1) { msg = "no tensor parts"; return 1; }
    const PackPart &P0 = parts[0];
    const int64_t C = P0.C;
    const int32_t B = P0.B, nw = P0.nw;
    const int32_t *widths = P0.widths;
    for (int p = 0; p < nparts; ++p) {
        const PackPart &P = parts[p];
        if (P.row0 < 0 || P.row1 > P.R || P.row1 <= P.row0) { msg = "invalid row range"; return 1; }
        if (P.C != C || P.B != B || P.nw != nw || std::memcmp(P.widths, widths, sizeof(int32_t) * nw) != 0) {
            msg = "fused tensor parts must share columns, block size and tier widths";
            return 1;
        }
    }
    L = TensorLayout();
    L.C = C; L.B = B; L.nw = nw; L.nparts = nparts;
    for (int i = 0; i < nw; ++i) L.widths[i] = widths[i];
    L.covered = (int32_t)P0.npal;
    std::memcpy(L.palette, P0.palette, P0.npal);
    L.NB = (C + B - 1) / B;
    L.fast_sip = nw == 2 && widths[0] == 3 && B == 1024 && C % 1024 == 0;
    std::vector<int64_t> rowoff(nparts + 1, 0);
    for (int p = 0; p < nparts; ++p) {
        const int64_t n = parts[p].row1 - parts[p].row0;
        if (nparts > 1 && p + 1 < nparts && n % kUnitRows != 0) {
            msg = "fused tensor parts other than the last need a multiple of 16 rows";
            return 1;
        }
        rowoff[p + 1] = rowoff[p] + n;
    }
    if (nparts > 1 && !L.fast_sip) {
        msg = "fused tensors are served by the sip kernel: every part sip, 1024-weight blocks, rows of whole blocks";
        return 1;
    }
    L.R = nparts == 1 ? P0.R : rowoff[nparts];
    L.row0 = nparts == 1 ? P0.row0 : 0;
    L.rows = rowoff[nparts];
    L.tiles = (L.rows + kUnitRows - 1) / kUnitRows;
    L.units = L.tiles * L.NB;
    {  // padded palette words of the first part (radix_pack.py:333-350)
        int32_t wpos = 0, base = 0;
        std::vector<uint8_t> t;
        for (int i = 0; i < nw - 1; ++i) {
            int32_t n = (1 << widths[i]) - 1, padded = ((n + 3) / 4) * 4;
            L.tier_table[i] = wpos;
            for (int k = 0; k < padded; ++k) t.push_back(k < n ? P0.palette[base + k] : 0);
            base += n;
            wpos += padded / 4;
        }
        L.npal_words = wpos;
        if (wpos > 24) { msg = "radix palette tables too large for the device kernels"; return 1; }
        std::memcpy(L.pal_words, t.data(), t.size());
    }
    const int64_t NB = L.NB, rows = L.rows, nblk = rows * NB;
    // global row -> (part, source block row)
    std::vector<int32_t> rpart(rows);
    std::vector<int64_t> rsrc(rows);
    for (int p = 0; p < nparts; ++p)
        for (int64_t r = rowoff[p]; r < rowoff[p + 1]; ++r) {
            rpart[r] = p;
            rsrc[r] = parts[p].row0 + (r - rowoff[p]);
        }
    for (int p = 0; p < nparts; ++p) {
        const PackPart &P = parts[p];
        const int64_t pb0 = P.row0 * NB, pnb = (P.row1 - P.row0) * NB;
        const int64_t words = (int64_t)P.offsets[pb0 + pnb] - (int64_t)P.offsets[pb0];
        L.payload_words += words;
        L.read_bytes += words * 4 + (pnb + 1) * 4 + (int64_t)L.npal_words * 4 + (nw > 2 ? pnb * 2 : 0);
    }
    std::vector<uint32_t> tabs((size_t)nparts * 4, 0);
    if (L.fast_sip)
        for (int p = 0; p < nparts; ++p) {
            sip_tables(parts[p].palette, &tabs[(size_t)p * 4]);
            if (p < 8) std::memcpy(L.part_tabs[p], &tabs[(size_t)p * 4], 16);
        }
    auto block_of = [&](int64_t i, const PackPart *&P, int64_t &gb) {
        const int64_t r = i / NB, b = i % NB;
        P = &parts[rpart[r]];
        gb = rsrc[r] * NB + b;
    };

    // pass 1: per block, escapes (fast path) and the schedule
    std::vector<uint16_t> nesc(nblk, 0), sched(nblk, 0);
    const bool fast = L.fast_sip;
    parallel_for(nblk, [&](int64_t i) {
        const PackPart *P;
        int64_t gb;
        block_of(i, P, gb);
        const uint32_t *blk = P->data + P->offsets[gb];
        int64_t words = (int64_t)P->offsets[gb + 1] - (int64_t)P->offsets[gb];
        int64_t n = std::min<int64_t>(B, C - (i % NB) * B);
        sched[i] = block_schedule(blk, (int64_t)P->nwords - (int64_t)P->offsets[gb], n, widths, nw);
        if (fast) {
            int e = sip_escapes(blk + 256, nullptr);
            // a block short of its terminal stream (validate cannot see it)
            // keeps every escape index inside its own words
            int avail = (int)std::max<int64_t>(0, (words - 352) * 4);
            nesc[i] = (uint16_t)std::min(e, avail);
        }
    });
    // unit sizes
    std::vector<int64_t> usize(L.units + 1, 0);
    const bool ragged = rows % kUnitRows != 0;
    for (int64_t u = 0; u < L.units; ++u) {
        int64_t tile = u / NB, b = u % NB, sz = kUnitHeader;
        bool absent = false;
        for (int s = 0; s < kUnitRows; ++s) {
            int64_t r = tile * kUnitRows + s;
            if (r >= rows) { absent = true; continue; }
            const int64_t i = r * NB + b;
            const PackPart *P;
            int64_t gb;
            block_of(i, P, gb);
            int64_t words = (int64_t)P->offsets[gb + 1] - (int64_t)P->offsets[gb];
            sz += a16(words * 4);
            if (fast) sz += a16((int64_t)nesc[i] * 2);
        }
        if (fast && absent && ragged) sz += 1408;
        usize[u] = sz;
        L.max_unit_bytes = (int32_t)std::max<int64_t>(L.max_unit_bytes, sz);
    }
    std::vector<int64_t> ustart(L.units + 1, 0);
    for (int64_t u = 0; u < L.units; ++u) ustart[u + 1] = ustart[u] + usize[u];
    const int64_t pad = a16(block_words_most(B, widths, nw) * 4 + 64);
    const int64_t total = ustart[L.units] + pad;
    if (ustart[L.units] / 16 > (int64_t)UINT32_MAX) { msg = "radix tensor too large for the unit directory"; return 1; }
    bytes.assign((size_t)total, '\0');
    unit16.assign((size_t)(L.units + 1) * 4, '\0');
    uint32_t *u16p = reinterpret_cast<uint32_t *>(&unit16[0]);
    for (int64_t u = 0; u <= L.units; ++u) u16p[u] = (uint32_t)(ustart[u] / 16);
    char *out = &bytes[0];
    parallel_for(L.units, [&](int64_t u) {
        int64_t tile = u / NB, b = u % NB;
        char *base = out + ustart[u];
        RowEntry *hdr = reinterpret_cast<RowEntry *>(base);
        if (fast) {
            const int p = rpart[std::min<int64_t>(tile * kUnitRows, rows - 1)];
            std::memcpy(base + kUnitRows * sizeof(RowEntry), &tabs[(size_t)p * 4], 16);
        }
        int64_t at = kUnitHeader;
        int64_t null_at = -1;
        for (int s = 0; s < kUnitRows; ++s) {
            int64_t r = tile * kUnitRows + s;
            if (r >= rows) continue;
            const int64_t i = r * NB + b;
            const PackPart *P;
            int64_t gb;
            block_of(i, P, gb);
            int64_t words = (int64_t)P->offsets[gb + 1] - (int64_t)P->offsets[gb];
            hdr[s].off16 = (uint16_t)(at / 16);
            hdr[s].words = (uint16_t)words;
            hdr[s].sched = sched[i];
            hdr[s].nesc = nesc[i];
            std::memcpy(base + at, P->data + P->offsets[gb], (size_t)words * 4);
            if (fast && words >= 352) {
                uint32_t planes[96];
                sip_code_planes(P->data + P->offsets[gb] + 256, planes);
                std::memcpy(base + at + 1024, planes, sizeof(planes));
            }
            at += a16(words * 4);
            if (fast) {
                std::vector<uint16_t> pos(1024);
                int e = sip_escapes(P->data + P->offsets[gb] + 256, pos.data());
                int keep = std::min<int>(e, nesc[i]);
                std::memcpy(base + at, pos.data(), (size_t)keep * 2);
                at += a16((int64_t)nesc[i] * 2);
            }
        }
        if (fast && ragged) {
            for (int s = 0; s < kUnitRows; ++s) {
                int64_t r = tile * kUnitRows + s;
                if (r < rows) continue;
                if (null_at < 0) {
                    null_at = at;
                    std::memset(base + at, 0, 1024);          // literals 0
                    std::memset(base + at + 1024, 0xFF, 384);  // every tier-0 code is 7: every weight escapes
                    at += 1408;
                }
                hdr[s].off16 = (uint16_t)(null_at / 16);
                hdr[s].words = 0;
                hdr[s].nesc = 0;
                hdr[s].sched = 0;
            }
        }
    });
    if (fast && rowdir) {
        // per row block (16-row padded rows x block columns): the absolute
        // offset of its streams in 16-byte units; its escape count (bits
        // 0-10), part index (bits 11-15) and the offset of its escape index
        // from the stream start in 16-byte units (bits 16-31) — the prefill
        // kernel's one-load directory
        const int64_t rows16 = L.tiles * kUnitRows;
        rowdir->assign((size_t)(rows16 * NB) * 8, '\0');
        uint32_t *rd = reinterpret_cast<uint32_t *>(&(*rowdir)[0]);
        parallel_for(L.units, [&](int64_t u) {
            const int64_t tile = u / NB, b = u % NB;
            const RowEntry *hdr = reinterpret_cast<const RowEntry *>(out + ustart[u]);
            for (int s = 0; s < kUnitRows; ++s) {
                const int64_t r = tile * kUnitRows + s;
                const uint32_t part = r < rows ? (uint32_t)rpart[r] : 0u;
                rd[(r * NB + b) * 2] = (uint32_t)(ustart[u] / 16) + hdr[s].off16;
                const uint32_t idx16 = (uint32_t)(a16((int64_t)hdr[s].words * 4) / 16);
                rd[(r * NB + b) * 2 + 1] = (uint32_t)hdr[s].nesc | ((part & 31u) << 11) | (idx16 << 16);
            }
        });
    }
    return 0;
}

}  // namespace dm
